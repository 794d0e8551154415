// plattice_noalloc.cu -- the forward filter for callers that cannot allocate
// device memory.
//
// Some callers of this library cannot call cudaMalloc (or a caching
// allocator) at the point where they need the filter: code running while a
// memory pool is frozen or being defragmented, plugins whose host process owns
// every device allocation, real-time loops that forbid allocation after
// start-up, and embedders that have no allocator handle to pass down.  For
// them plattice_forward_noalloc runs the same forward filter as
// plattice_forward, with its lattice and scratch buffers carved out of one
// fixed array in the library's own device memory instead of buffers supplied
// by the caller.  The caller still passes the inputs and the outputs.
//
// The array is a file-scope static __device__ array of PL_NOALLOC_BYTES
// (64 MiB): every GPU on which the library is loaded holds it until the
// process exits.  An image whose workspace does not fit is rejected.
//
// Host code cannot use the array's name as a device address (it only names a
// host-side shadow of the symbol), so the first call in each CUDA context,
// with that context current, asks the runtime for the array's device address
// (cudaGetSymbolAddress) and keeps it for that context.  Make that first call
// -- or plattice_prepare -- before any stream capture begins.
//
// All calls on a device share the one array and it keeps whatever the last
// call left in it; the filter clears every part it needs to start at zero.
// Calls whose work overlaps on the GPU (other streams, other host threads)
// race on the array: issue them one after the other.
#include <cuda_runtime.h>
#include <stdio.h>

#include "../../include/plattice.h"
#include "plattice_layout.h"
#include "plattice_runtime.h"

#define PL_NOALLOC_BYTES (64ull << 20)

static __device__ __align__(256) unsigned char g_noalloc_arena[PL_NOALLOC_BYTES];

namespace pl {
int forward_images(float* weight_out, float* out, const float* values, const float* features, void* lattice,
                   size_t lattice_bytes, void* scratch, size_t scratch_bytes, int b, int pd, int vd, int w,
                   int h, void* stream, bool track, const char* call);
}

namespace {
thread_local char g_noalloc_err[192] = "";

// the array's device address in the current context
int arena(void** base) {
    const cudaError_t e = pl::symbol_address(reinterpret_cast<const void*>(&g_noalloc_arena), base);
    if (e != cudaSuccess) {
        snprintf(g_noalloc_err, sizeof(g_noalloc_err), "device address of the fixed array: %s",
                 cudaGetErrorName(e));
        return PLATTICE_ERR_CUDA;
    }
    return PLATTICE_OK;
}
}  // namespace

extern "C" {

size_t plattice_noalloc_capacity(void) { return (size_t)PL_NOALLOC_BYTES; }

const char* plattice_noalloc_error_detail(void) { return g_noalloc_err; }

int plattice_forward_noalloc(float* weight_out, float* out, const float* values, const float* features,
                             int pd, int vd, int w, int h, void* stream) {
    g_noalloc_err[0] = '\0';
    size_t lattice_bytes = 0, scratch_bytes = 0;
    int rc = plattice_workspace_sizes(h, w, pd, vd, &lattice_bytes, &scratch_bytes);
    if (rc != PLATTICE_OK) return rc;
    const size_t need = pl_align(lattice_bytes) + scratch_bytes;
    if (need > (size_t)PL_NOALLOC_BYTES) {
        snprintf(g_noalloc_err, sizeof(g_noalloc_err),
                 "image %dx%d (pd %d, vd %d) needs %zu bytes of workspace; the fixed array holds %llu",
                 h, w, pd, vd, need, (unsigned long long)PL_NOALLOC_BYTES);
        return PLATTICE_ERR_WORKSPACE;
    }
    if (h == 0 || w == 0) return PLATTICE_OK;
    void* base = nullptr;
    rc = arena(&base);
    if (rc != PLATTICE_OK) return rc;
    unsigned char* lattice = static_cast<unsigned char*>(base);
    unsigned char* scratch = lattice + pl_align(lattice_bytes);
    // no status ticket: the ring's pinned host memory would be an allocation
    return pl::forward_images(weight_out, out, values, features, lattice, lattice_bytes, scratch, scratch_bytes,
                              1, pd, vd, w, h, stream, false, "plattice_forward_noalloc");
}

int plattice_noalloc_status(int* status, int* m, void* stream) {
    void* base = nullptr;
    const int rc = arena(&base);
    if (rc != PLATTICE_OK) return rc;
    return plattice_lattice_info(base, status, m, nullptr, nullptr, stream);
}

}  // extern "C"
