// plattice_pd.cu -- explicit instantiation of the filter for one feature
// dimension.  Compiled once per pd in 1..16 with -DPL_PD=<pd>, so that the
// 16 x 8 (pd, vd) kernel instances build in parallel.
#include "plattice_impl.cuh"

#ifndef PL_PD
#error "compile with -DPL_PD=<1..16>"
#endif

namespace pl {
template cudaError_t run_forward<PL_PD>(const CallArgs&);
template cudaError_t run_backward<PL_PD>(const CallArgs&);
template cudaError_t run_filter<PL_PD>(const CallArgs&);
template cudaError_t run_feature_grad<PL_PD>(const CallArgs&);
template cudaError_t run_prepare<PL_PD>(const CallArgs&);
template cudaError_t run_export_keys<PL_PD>(const void*, const void*, const PlLayout&, int16_t*, int,
                                           cudaStream_t);
}  // namespace pl
