// plattice_impl.cuh -- launch sequences of the forward and backward filter for
// one feature dimension PD (explicitly instantiated per PD in plattice_pd.cu,
// dispatched over pd at run time by plattice_capi.cu, over vd here).
#pragma once
#include <math.h>

#include "plattice_kernels.cuh"
#include "plattice_profile.h"

namespace pl {

struct CallArgs {
    const float* features;
    const float* values;     // forward values, or backward upstream gradient
    const float* weight_in;  // backward: saved normaliser
    float* out;
    float* wout;             // forward: normaliser output
    void* lattice;
    void* scratch;
    PlLayout lay;
    cudaStream_t stream;
    int sm_count;
    int lattice_state;       // backward: 0 rebuild, 1 fresh from forward, 2 reuse (re-zero)
    int cap_override_log2;
};

inline LatView lat_view(void* base, const PlLayout& L) {
    char* b = static_cast<char*>(base);
    LatView v;
    v.hdr = reinterpret_cast<LatticeHeader*>(b);
    v.tile_off = reinterpret_cast<int*>(b + L.off_tile_off);
    v.tile_cnt = reinterpret_cast<int*>(b + L.off_tile_cnt);
    v.slot_lid = reinterpret_cast<uint16_t*>(b + L.off_slot_lid);
    v.slot_w = reinterpret_cast<float*>(b + L.off_slot_w);
    v.staged_vid = reinterpret_cast<int*>(b + L.off_staged_vid);
    v.nbr = reinterpret_cast<int2*>(b + L.off_nbr);
    v.vb0 = reinterpret_cast<float*>(b + L.off_vb0);
    v.vb1 = reinterpret_cast<float*>(b + L.off_vb1);
    return v;
}

inline ScrView scr_view(void* base, const PlLayout& L) {
    char* b = static_cast<char*>(base);
    ScrView v;
    v.skeys = reinterpret_cast<uint4*>(b + L.off_skeys);
    v.svals = reinterpret_cast<float*>(b + L.off_svals);
    v.table = reinterpret_cast<uint4*>(b + L.off_table);
    v.vkeys = reinterpret_cast<uint4*>(b + L.off_vkeys);
    v.vf0 = reinterpret_cast<float*>(b + L.off_vf0);
    v.vf1 = reinterpret_cast<float*>(b + L.off_vf1);
    return v;
}

// Scale factors of permutohedral.cu:507-508, in float on the host as there.
inline EmbedConsts embed_consts(int pd) {
    EmbedConsts ec;
    for (int i = 0; i < PL_MAX_PD; ++i) ec.sf[i] = 0.0f;
    for (int i = 0; i < pd; ++i) {
        ec.sf[i] = (float)(pd + 1) * sqrtf(((1.0f / 6.0f) + 0.5f) / (float)((i + 1) * (i + 2)));
    }
    ec.rk = 1.0f / (float)(pd + 1);
    ec.kf = (float)(pd + 1);
    return ec;
}

inline Geo make_geo(const CallArgs& a) {
    Geo g;
    g.h = a.lay.h; g.w = a.lay.w; g.tiles_x = a.lay.tiles_x; g.tiles = a.lay.tiles;
    g.cap_max_log2 = a.lay.cap_max_log2;
    g.cap_override_log2 = a.cap_override_log2;
    return g;
}

// opt in to more than 48 KB of dynamic shared memory, once per device
template <int PD, int V>
cudaError_t prepare_tile_build() {
    static bool done[64] = {};
    constexpr int smem = tile_build_smem_bytes<PD>();
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !done[dev]) {
        e = cudaFuncSetAttribute(k_tile_build<PD, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) done[dev] = true;
    }
    return cudaSuccess;
}

// Build the lattice: tile dedup (+ forward splat when values != nullptr),
// table clear, global insert, blur neighbours.
template <int PD, int V>
cudaError_t build_lattice(const CallArgs& a, const Geo& geo, const LatView& Lv, const ScrView& Sv,
                          const float* values) {
    using C = Cfg<PD>;
    constexpr int CPF = pad_ch(V + 1), CPB = pad_ch(V);
    const cudaStream_t s = a.stream;
    const int grid = a.sm_count * 8;
    cudaError_t e = prepare_tile_build<PD, V>();
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(Lv.hdr, 0, sizeof(LatticeHeader), s);
    if (e != cudaSuccess) return e;
    const EmbedConsts ec = embed_consts(PD);
    PL_LAUNCH(STAGE_TILE_BUILD, s, k_tile_build<PD, V><<<a.lay.tiles, C::P, tile_build_smem_bytes<PD>(), s>>>(
        a.features, values, geo, ec, Lv, Sv));
    PL_LAUNCH(STAGE_CLEAR, s, k_clear<<<grid, 256, 0, s>>>(geo, Lv, Sv, C::CW, values ? CPF : 0, CPB));
    PL_LAUNCH(STAGE_INSERT, s, k_insert<PD, CPF><<<grid, 256, 0, s>>>(Lv, Sv, values ? 1 : 0));
    PL_LAUNCH(STAGE_NEIGHBORS, s, k_neighbors<PD><<<grid, 256, 0, s>>>(Lv, Sv));
    return cudaGetLastError();
}

template <int PD, int V>
cudaError_t forward_v(const CallArgs& a) {
    constexpr int CPF = pad_ch(V + 1);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    const ScrView Sv = scr_view(a.scratch, a.lay);
    cudaError_t e = build_lattice<PD, V>(a, geo, Lv, Sv, a.values);
    if (e != cudaSuccess) return e;
    const int grid = a.sm_count * 8;
    float* x = Sv.vf0;
    float* y = Sv.vf1;
    for (int ax = 0; ax <= PD; ++ax) {   // axis order 0..pd (permutohedral.cu:585)
        PL_LAUNCH(STAGE_BLUR_FWD, a.stream, k_blur<CPF><<<grid, 256, 0, a.stream>>>(x, y, Lv.nbr, Lv.hdr, ax, V + 1));
        float* t = x; x = y; y = t;
    }
    PL_LAUNCH(STAGE_SLICE_FWD, a.stream,
              k_slice<PD, V, true><<<a.lay.tiles, Cfg<PD>::P, 0, a.stream>>>(a.out, a.wout, geo, Lv, x));
    return cudaGetLastError();
}

template <int PD, int V>
cudaError_t backward_v(const CallArgs& a) {
    constexpr int CPB = pad_ch(V);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    const ScrView Sv = scr_view(a.scratch, a.lay);
    const int grid = a.sm_count * 8;
    cudaError_t e;
    if (a.lattice_state == 0) {
        e = build_lattice<PD, V>(a, geo, Lv, Sv, nullptr);
        if (e != cudaSuccess) return e;
    } else if (a.lattice_state == 2) {
        PL_LAUNCH(STAGE_ZERO, a.stream, k_zero_rows<<<grid, 256, 0, a.stream>>>(Lv.vb0, Lv.hdr, CPB));
    }
    PL_LAUNCH(STAGE_SPLAT_BWD, a.stream,
              k_splat_bwd<PD, V><<<a.lay.tiles, Cfg<PD>::P, 0, a.stream>>>(a.values, a.weight_in, geo, Lv, Lv.vb0));
    float* x = Lv.vb0;
    float* y = Lv.vb1;
    for (int s = 0; s <= PD; ++s) {   // axis order pd..0 (permutohedral.cu:647)
        PL_LAUNCH(STAGE_BLUR_BWD, a.stream, k_blur<CPB><<<grid, 256, 0, a.stream>>>(x, y, Lv.nbr, Lv.hdr, PD - s, V));
        float* t = x; x = y; y = t;
    }
    PL_LAUNCH(STAGE_SLICE_BWD, a.stream,
              k_slice<PD, V, false><<<a.lay.tiles, Cfg<PD>::P, 0, a.stream>>>(a.out, nullptr, geo, Lv, x));
    return cudaGetLastError();
}

#define PL_DISPATCH_V(FN, PDV, ARGS)                      \
    switch ((ARGS).lay.vd) {                              \
        case 1: return FN<PDV, 1>(ARGS);                  \
        case 2: return FN<PDV, 2>(ARGS);                  \
        case 3: return FN<PDV, 3>(ARGS);                  \
        case 4: return FN<PDV, 4>(ARGS);                  \
        case 5: return FN<PDV, 5>(ARGS);                  \
        case 6: return FN<PDV, 6>(ARGS);                  \
        case 7: return FN<PDV, 7>(ARGS);                  \
        case 8: return FN<PDV, 8>(ARGS);                  \
        default: return cudaErrorInvalidValue;            \
    }

template <int PD>
cudaError_t run_forward(const CallArgs& a) { PL_DISPATCH_V(forward_v, PD, a) }

template <int PD>
cudaError_t run_backward(const CallArgs& a) { PL_DISPATCH_V(backward_v, PD, a) }

template <int PD>
cudaError_t run_export_keys(const void* lattice, const void* scratch, const PlLayout& lay, int16_t* out,
                            int max_keys, cudaStream_t s) {
    const LatView Lv = lat_view(const_cast<void*>(lattice), lay);
    const ScrView Sv = scr_view(const_cast<void*>(scratch), lay);
    k_export_keys<PD><<<256, 256, 0, s>>>(Sv, Lv.hdr, out, max_keys);
    return cudaGetLastError();
}

}  // namespace pl
