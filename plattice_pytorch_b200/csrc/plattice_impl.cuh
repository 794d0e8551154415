// plattice_impl.cuh -- launch sequences of the forward and backward filter for
// one feature dimension PD (explicitly instantiated per PD in plattice_pd.cu,
// dispatched over pd at run time by plattice_capi.cu, over vd here).
#pragma once
#include <math.h>

#include <functional>
#include <utility>

#include "plattice_kernels.cuh"
#include "plattice_profile.h"
#include "plattice_runtime.h"

namespace pl {

// The kernel node of a captured call that writes the call's status word to
// its status-ring slot (the call's last kernel), and how to point it at the
// slot and sequence number of a later replay of the graph.
struct StatusNode {
    cudaGraphNode_t node = nullptr;
    std::function<cudaError_t(cudaGraphExec_t, unsigned long long*, unsigned)> retarget;
};

struct CallArgs {
    const float* features;
    const float* values;     // forward values, or backward upstream gradient
    const float* weight_in;  // backward: saved normaliser
    float* out;
    float* wout;             // forward: normaliser output
    void* lattice;
    void* scratch;           // build part of the scratch (lattice builds only)
    PlLayout lay;
    cudaStream_t stream;
    int sm_count;
    int lattice_state;       // backward: 0 rebuild, 1 reuse (rows zeroed by the forward), 2 reuse (re-zero)
    int cap_override_log2;
    int filter_min_log2;     // 0: the default (tables of 2^22 cells and more)
    int blur_flags;          // kBlurHalf (bfloat16 rows of large lattices), kBlurStream (tests)
    float* v0;               // lattice value rows of the call's blur (ping-pong; the splat
    float* v1;               // accumulates into v0) and their bookkeeping: the scratch's
    uint8_t* bstate;         // front part (a backward's v0: the lattice's vb0), or a
                             // kept-lattice call's workspace
    // feature gradient: dL/dout, the forward's out, and lattice rows / flags in the workspace
    const float* grad_in;
    const float* out_in;
    float* hbuf0;
    float* hbuf1;
    float* evec;
    int* flags;
    StatusTicket st;         // where the call's last kernel reports the status word
    StatusNode* status_node; // set while the call is being captured into a graph
};

inline LatView lat_view(void* base, const PlLayout& L) {
    char* b = static_cast<char*>(base);
    LatView v;
    v.hdr = reinterpret_cast<LatticeHeader*>(b);
    v.tile_off = reinterpret_cast<int*>(b + L.off_tile_off);
    v.tile_cnt = reinterpret_cast<int*>(b + L.off_tile_cnt);
    v.slot_lid = reinterpret_cast<uint16_t*>(b + L.off_slot_lid);
    v.slot_w = reinterpret_cast<float*>(b + L.off_slot_w);
    v.slot_order = reinterpret_cast<uint16_t*>(b + L.off_slot_order);
    v.slot_wsort = reinterpret_cast<float*>(b + L.off_slot_wsort);
    v.first_lid = reinterpret_cast<uint16_t*>(b + L.off_first_lid);
    v.staged_vid = reinterpret_cast<int*>(b + L.off_staged_vid);
    v.nbr = reinterpret_cast<int2*>(b + L.off_nbr);
    return v;
}

// `base`: the whole scratch buffer (front part + build part)
inline ScrView scr_view(void* base, const PlLayout& L) {
    char* b = static_cast<char*>(base);
    ScrView v;
    v.skeys = reinterpret_cast<uint4*>(b + L.off_skeys);
    v.table = reinterpret_cast<uint32_t*>(b + L.off_table);
    v.filter = reinterpret_cast<uint32_t*>(b + L.off_filter);
    v.owner = reinterpret_cast<int*>(b + L.off_owner);
    v.vid_of = reinterpret_cast<int*>(b + L.off_vid_of);
    v.vkeys = reinterpret_cast<uint4*>(b + L.off_vkeys);
    return v;
}

// The lattice's rows for the first backward.
inline float* lattice_vb0(const CallArgs& a) { return reinterpret_cast<float*>(static_cast<char*>(a.lattice) + a.lay.off_vb0); }

// The value rows of a call in the front part of a scratch buffer.
inline void rows_in_scratch(CallArgs& a, void* scratch) {
    char* b = static_cast<char*>(scratch);
    a.v0 = reinterpret_cast<float*>(b + a.lay.off_v0);
    a.v1 = reinterpret_cast<float*>(b + a.lay.off_v1);
    a.bstate = reinterpret_cast<uint8_t*>(b + a.lay.off_bstate);
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

// Grid of the per-tile kernels: one CTA per tile, (tiles_x, tiles_y, images).
inline dim3 tile_grid(const CallArgs& a) {
    return dim3((unsigned)a.lay.tiles_x, (unsigned)a.lay.tiles_y, (unsigned)a.lay.b);
}

inline Geo make_geo(const CallArgs& a) {
    Geo g;
    g.h = a.lay.h; g.w = a.lay.w; g.tiles_x = a.lay.tiles_x; g.tiles = a.lay.tiles;
    g.tiles_img = a.lay.tiles_img;
    g.n_img = a.lay.n_img;
    g.cap_max_log2 = a.lay.cap_max_log2;
    g.cap_override_log2 = a.cap_override_log2;
    g.filter_min_log2 = a.filter_min_log2 > 0 ? a.filter_min_log2 : 22;   // a 16 MB table and up
    g.idx_bits = 1;
    while (g.idx_bits < 32 && (1ll << g.idx_bits) <= a.lay.slots) ++g.idx_bits;   // 1 + index <= slots
    return g;
}

// Launch through cudaLaunchKernelEx (optionally cooperative), returning the
// launch error.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool coop,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = coop ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// opt in to more than 48 KB of dynamic shared memory, once per context
template <int PD>
cudaError_t tile_build_attr(int* v) {
    *v = 1;
    return cudaFuncSetAttribute(k_tile_build<PD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                tile_build_smem_bytes<PD>());
}

template <int PD>
cudaError_t prepare_tile_build() {
    int v = 0;
    return kernel_once(reinterpret_cast<const void*>(k_tile_build<PD>), tile_build_attr<PD>, &v);
}

// a grid of `want` CTAs, or fewer when `need` (at least 1) cover the work:
// small images then launch no CTAs that would exit at once
inline int capped_grid(long long want, long long need) {
    if (need < 1) need = 1;
    return (int)(want < need ? want : need);
}

// the blur kernel's dynamic shared memory and its co-resident CTAs per SM
template <int PD, int CP>
cudaError_t blur_attr(int* per_sm) {
    cudaError_t e = cudaFuncSetAttribute(k_blur_all<PD, CP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kBlurQueueBytes);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_blur_all<PD, CP>, kBlurThreads, kBlurQueueBytes);
    if (e != cudaSuccess) return e;
    return *per_sm < 1 ? cudaErrorLaunchOutOfResources : cudaSuccess;
}

// co-resident CTAs per SM of the insert
template <int PD>
cudaError_t insert_attr(int* per_sm) {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_insert<PD>, 256, 0);
    if (e != cudaSuccess) return e;
    return *per_sm < 1 ? cudaErrorLaunchOutOfResources : cudaSuccess;
}

// Build the lattice: tile dedup (which also zeroes the lattice value rows
// `zero` of cp floats each, and `zero_b` of cpb floats when set), table clear,
// global insert, vertex ids.  Blur neighbours follow, with the first splat.
template <int PD>
cudaError_t build_lattice(const CallArgs& a, const Geo& geo, const LatView& Lv, const ScrView& Sv, float* zero,
                          int cp, float* zero_b = nullptr, int cpb = 0) {
    using C = Cfg<PD>;
    const cudaStream_t s = a.stream;
    const int grid = a.sm_count * 8;
    cudaError_t e = prepare_tile_build<PD>();
    if (e != cudaSuccess) return e;
    PL_GROUP(STAGE_GROUP_BUILD, s, true);
    e = cudaMemsetAsync(Lv.hdr, 0, sizeof(LatticeHeader), s);
    if (e != cudaSuccess) return e;
    const EmbedConsts ec = embed_consts(PD);
    PL_LAUNCH(STAGE_TILE_BUILD, s,
              e = launch_k(k_tile_build<PD>, tile_grid(a), dim3(C::P), tile_build_smem_bytes<PD>(), s, false,
                             a.features, geo, ec, Lv, Sv, zero, cp, zero_b, cpb));
    if (e != cudaSuccess) return e;
    // no more CTAs than the largest table needs (2^cap_max_log2 cells, four a
    // thread); the insert no more than the staged keys (at most slots)
    PL_LAUNCH(STAGE_CLEAR, s,
              e = launch_k(k_clear, dim3(capped_grid(grid, ((1ll << a.lay.cap_max_log2) / 4 + 255) / 256)), dim3(256),
                           0, s, false, geo, Lv, Sv));
    if (e != cudaSuccess) return e;
    int per_sm = 0;   // the insert's co-resident CTAs per SM
    e = kernel_once(reinterpret_cast<const void*>(k_insert<PD>), insert_attr<PD>, &per_sm);
    if (e != cudaSuccess) return e;
    PL_LAUNCH(STAGE_INSERT, s,
              e = launch_k(k_insert<PD>, dim3(capped_grid(grid * 2, (a.lay.slots + 255) / 256)), dim3(256), 0, s, false,
                           geo, Lv, Sv, a.sm_count * per_sm));
    PL_GROUP(STAGE_GROUP_BUILD, s, false);
    return e;
}

// The splat right after a build, with the blur-neighbour lookups in the same
// launch.
template <int PD, int V, bool FWD>
cudaError_t splat_with_neighbors(const CallArgs& a, const Geo& geo, const LatView& Lv, const ScrView& Sv,
                                 const float* vals, const float* wt, float* rows, int stage) {
    cudaError_t e;
    if constexpr (Cfg<PD>::P == 256) {
        // lookup CTAs: as many threads as four 256-thread CTAs per SM, so that
        // the first wave leaves room for splat tiles beside them
        const int nbr_blocks = a.sm_count * 4 * kNbrThreads / Cfg<PD>::P;
        PL_LAUNCH(stage, a.stream,
                  e = launch_k(k_splat_nbr<PD, V, FWD>, dim3(nbr_blocks + a.lay.tiles), dim3(Cfg<PD>::P), 0,
                               a.stream, false, vals, wt, geo, Lv, Sv, rows, nbr_blocks));
    } else {
        // large feature dimensions: the lookups (most of the work) in their own
        // launch of 256-thread CTAs, then the splat, which resolves the vertex ids
        PL_LAUNCH(STAGE_NEIGHBORS, a.stream,
                  e = launch_k(k_neighbors<PD>, dim3(a.sm_count * 8), dim3(kNbrThreads), 0, a.stream, false, geo, Lv,
                               Sv));
        if (e != cudaSuccess) return e;
        PL_LAUNCH(stage, a.stream,
                  e = launch_k(k_splat<PD, V, FWD>, tile_grid(a), dim3(Cfg<PD>::P), 0, a.stream, false, vals, wt, geo,
                               Lv, Sv, 1, rows));
    }
    return e;
}

// Cooperative launch of the blur kernel on as many CTAs as are co-resident
// (at most kCoopPerSm per SM).
constexpr int kCoopPerSm = 1;

template <int PD, int CP>
cudaError_t launch_blur_all(const CallArgs& a, LatView Lv, float* b0, float* b1, int reverse,
                            int* final_flag = nullptr) {
    if (!final_flag) final_flag = &Lv.hdr->blur_final;
    int n = 0;
    cudaError_t e = kernel_once(reinterpret_cast<const void*>(k_blur_all<PD, CP>), blur_attr<PD, CP>, &n);
    if (e != cudaSuccess) return e;
    const int blocks = capped_grid((long long)a.sm_count * (n < kCoopPerSm ? n : kCoopPerSm),
                                   (a.lay.slots + kBlurThreads - 1) / kBlurThreads);
    PL_LAUNCH(reverse ? STAGE_BLUR_BWD : STAGE_BLUR_FWD, a.stream,
              e = launch_k(k_blur_all<PD, CP>, dim3(blocks), dim3(kBlurThreads), kBlurQueueBytes, a.stream, true, Lv,
                           b0, b1, a.bstate, reverse, final_flag, a.blur_flags));
    return e;
}

// co-resident CTAs per SM of the zero-then-splat kernel
template <int PD, int V, bool FWD>
cudaError_t splat_zeroed_attr(int* per_sm) {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_splat_zeroed<PD, V, FWD>, Cfg<PD>::P, 0);
    if (e != cudaSuccess) return e;
    return *per_sm < 1 ? cudaErrorLaunchOutOfResources : cudaSuccess;
}

// Splat into rows that must first be zeroed (a call on a kept lattice): one
// cooperative launch (zeroing, a grid barrier, the splat).
template <int PD, int V, bool FWD>
cudaError_t splat_zeroed(const CallArgs& a, const Geo& geo, const LatView& Lv, const float* vals, const float* wt,
                         float* rows, int stage) {
    constexpr int CP = FWD ? pad_ch(V + 1) : pad_ch(V);
    int per_sm = 0;
    cudaError_t e = kernel_once(reinterpret_cast<const void*>(k_splat_zeroed<PD, V, FWD>), splat_zeroed_attr<PD, V, FWD>,
                                &per_sm);
    if (e != cudaSuccess) return e;
    const int grid = a.sm_count * per_sm;
    PL_LAUNCH(stage, a.stream,
              e = launch_k(k_splat_zeroed<PD, V, FWD>, dim3(grid < a.lay.tiles ? grid : a.lay.tiles),
                           dim3(Cfg<PD>::P), 0, a.stream, true, vals, wt, geo, Lv, rows, CP));
    return e;
}

// the streamed slice's dynamic shared memory and its co-resident CTAs per SM
template <int PD, int V, bool FWD>
cudaError_t slice_attr(int* per_sm) {
    cudaError_t e = cudaFuncSetAttribute(k_slice_pipe<PD, V, FWD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         slice_pipe_smem_bytes<PD>());
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_slice_pipe<PD, V, FWD>, Cfg<PD>::P,
                                                      slice_pipe_smem_bytes<PD>());
    if (e != cudaSuccess) return e;
    return *per_sm < 1 ? cudaErrorLaunchOutOfResources : cudaSuccess;
}

// The slice (the call's last kernel: it reports the status word).  Tiles of
// 256 pixels (pd <= 6): persistent CTAs that stream the slot records, as many
// as are co-resident, at most one per tile; smaller tiles (whose CTAs would be
// too small to keep an SM busy that way): one CTA per tile.
template <int PD, int V, bool FWD>
cudaError_t launch_slice(const CallArgs& a, const Geo& geo, const LatView& Lv, float* out, float* wout,
                         const float* r0, const float* r1) {
    cudaError_t e;
    void (*kern)(float*, float*, Geo, LatView, const float*, const float*, unsigned long long*, unsigned);
    dim3 grid, block(Cfg<PD>::P);
    size_t smem = 0;
    if constexpr (kSlicePiped<PD>) {
        int per_sm = 0;
        e = kernel_once(reinterpret_cast<const void*>(k_slice_pipe<PD, V, FWD>), slice_attr<PD, V, FWD>, &per_sm);
        if (e != cudaSuccess) return e;
        const int want = a.sm_count * per_sm;
        kern = k_slice_pipe<PD, V, FWD>;
        grid = dim3(want < a.lay.tiles ? want : a.lay.tiles);
        smem = slice_pipe_smem_bytes<PD>();
    } else {
        kern = k_slice<PD, V, FWD>;
        grid = tile_grid(a);
    }
    PL_LAUNCH(FWD ? STAGE_SLICE_FWD : STAGE_SLICE_BWD, a.stream,
              e = launch_k(kern, grid, block, smem, a.stream, false, out, wout, geo, Lv, r0, r1, a.st.slot,
                           a.st.seq));
    if (e == cudaSuccess && a.status_node) {   // being captured: remember the node and its arguments
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        const cudaGraphNode_t* deps = nullptr;
        size_t nd = 0;
        e = cudaStreamGetCaptureInfo(a.stream, &cs, nullptr, nullptr, &deps, &nd);
        if (e != cudaSuccess) return e;
        if (cs == cudaStreamCaptureStatusActive && nd == 1) {
            const cudaGraphNode_t node = deps[0];
            a.status_node->node = node;
            a.status_node->retarget = [=](cudaGraphExec_t ex, unsigned long long* slot, unsigned seq) {
                float* o = out;
                float* wo = wout;
                Geo g = geo;
                LatView lv = Lv;
                const float* x0 = r0;
                const float* x1 = r1;
                unsigned long long* sl = slot;
                unsigned sq = seq;
                void* args[] = {&o, &wo, &g, &lv, &x0, &x1, &sl, &sq};
                cudaKernelNodeParams p = {};
                p.func = reinterpret_cast<void*>(kern);
                p.gridDim = grid;
                p.blockDim = block;
                p.sharedMemBytes = (unsigned)smem;
                p.kernelParams = args;
                return cudaGraphExecKernelNodeSetParams(ex, node, &p);
            };
        }
    }
    return e;
}

template <int PD, int V>
cudaError_t forward_v(const CallArgs& a) {
    constexpr int CPF = pad_ch(V + 1), CPB = pad_ch(V);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    const ScrView Sv = scr_view(a.scratch, a.lay);
    // zeroes the forward's rows and the lattice's rows for the first backward
    cudaError_t e = build_lattice<PD>(a, geo, Lv, Sv, a.v0, CPF, lattice_vb0(a), CPB);
    if (e != cudaSuccess) return e;
    PL_GROUP(STAGE_GROUP_FILTER_FWD, a.stream, true);
    // neighbour lookups (L2-latency-bound) alongside the splat (HBM-bound)
    e = splat_with_neighbors<PD, V, true>(a, geo, Lv, Sv, a.values, nullptr, a.v0, STAGE_SPLAT_FWD);
    if (e != cudaSuccess) return e;
    // blur in axis order 0..pd (permutohedral.cu:585)
    e = launch_blur_all<PD, CPF>(a, Lv, a.v0, a.v1, 0);
    if (e != cudaSuccess) return e;
    e = launch_slice<PD, V, true>(a, geo, Lv, a.out, a.wout, a.v0, a.v1);
    PL_GROUP(STAGE_GROUP_FILTER_FWD, a.stream, false);
    return e;
}

template <int PD, int V>
cudaError_t backward_v(const CallArgs& a) {
    constexpr int CPB = pad_ch(V);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    const ScrView Sv = a.scratch ? scr_view(a.scratch, a.lay) : ScrView{};
    cudaError_t e = cudaSuccess;
    if (a.lattice_state == 0) {   // rebuild (permutohedral.cu:615-635); the tile build zeroes the rows
        e = build_lattice<PD>(a, geo, Lv, Sv, a.v0, CPB);
        if (e != cudaSuccess) return e;
        PL_GROUP(STAGE_GROUP_FILTER_BWD, a.stream, true);
        e = splat_with_neighbors<PD, V, false>(a, geo, Lv, Sv, a.values, a.weight_in, a.v0, STAGE_SPLAT_BWD);
    } else if (a.lattice_state == 1) {   // rows zeroed by the forward's tile build
        PL_GROUP(STAGE_GROUP_FILTER_BWD, a.stream, true);
        PL_LAUNCH(STAGE_SPLAT_BWD, a.stream,
                  e = launch_k(k_splat<PD, V, false>, tile_grid(a), dim3(Cfg<PD>::P), 0, a.stream, false,
                               a.values, a.weight_in, geo, Lv, Sv, 0, a.v0));
    } else {   // used by an earlier backward: zero the rows and splat in one launch
        PL_GROUP(STAGE_GROUP_FILTER_BWD, a.stream, true);
        e = splat_zeroed<PD, V, false>(a, geo, Lv, a.values, a.weight_in, a.v0, STAGE_SPLAT_BWD);
    }
    if (e != cudaSuccess) return e;
    // blur in axis order pd..0 (permutohedral.cu:647)
    e = launch_blur_all<PD, CPB>(a, Lv, a.v0, a.v1, 1);
    if (e != cudaSuccess) return e;
    e = launch_slice<PD, V, false>(a, geo, Lv, a.out, nullptr, a.v0, a.v1);
    PL_GROUP(STAGE_GROUP_FILTER_BWD, a.stream, false);
    return e;
}

// Forward filter of new values on a kept lattice (built by a forward call on
// the same image): zero the value rows, splat, blur, slice.  No rebuild.
template <int PD, int V>
cudaError_t filter_v(const CallArgs& a) {
    constexpr int CPF = pad_ch(V + 1);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    cudaError_t e = splat_zeroed<PD, V, true>(a, geo, Lv, a.values, nullptr, a.v0, STAGE_SPLAT_FWD);
    if (e != cudaSuccess) return e;
    e = launch_blur_all<PD, CPF>(a, Lv, a.v0, a.v1, 0);
    if (e != cudaSuccess) return e;
    return launch_slice<PD, V, true>(a, geo, Lv, a.out, a.wout, a.v0, a.v1);
}

// Gradient of the forward filter with respect to the features, on a kept
// lattice: R = blur(splat(values)), H = blur_reverse(splat((G, -G.out) / Z)),
// then per pixel the chain rule through the weights and the elevation.
template <int PD, int V>
cudaError_t fgrad_v(const CallArgs& a) {
    constexpr int CPF = pad_ch(V + 1);
    const Geo geo = make_geo(a);
    const LatView Lv = lat_view(a.lattice, a.lay);
    const int grid = a.sm_count * 8;
    cudaError_t e;
    // R: the forward's lattice values
    e = splat_zeroed<PD, V, true>(a, geo, Lv, a.values, nullptr, a.v0, STAGE_SPLAT_FWD);
    if (e != cudaSuccess) return e;
    e = launch_blur_all<PD, CPF>(a, Lv, a.v0, a.v1, 0, a.flags);
    if (e != cudaSuccess) return e;
    // H: the lattice gradient, V+1 channels of (G, -G.out) weighted by 1/Z
    const size_t n = (size_t)a.lay.b * (size_t)a.lay.n_img;
    e = launch_k(k_fgrad_prep<V>, dim3(grid), dim3(256), 0, a.stream, false, a.evec, a.grad_in, a.out_in, n,
                 Lv.hdr);
    if (e != cudaSuccess) return e;
    e = splat_zeroed<PD, V + 1, false>(a, geo, Lv, a.evec, a.weight_in, a.hbuf0, STAGE_SPLAT_BWD);
    if (e != cudaSuccess) return e;
    e = launch_blur_all<PD, CPF>(a, Lv, a.hbuf0, a.hbuf1, 1, a.flags + 1);
    if (e != cudaSuccess) return e;
    return launch_k(k_fgrad<PD, V>, tile_grid(a), dim3(Cfg<PD>::P), 0, a.stream, false, a.out, a.features,
                    a.values, a.grad_in, a.out_in, a.weight_in, geo, embed_consts(PD), Lv, (const float*)a.v0,
                    (const float*)a.v1, (const float*)a.hbuf0, (const float*)a.hbuf1, (const int*)a.flags,
                    a.st.slot, a.st.seq);
}

// Everything the first call of (PD, V) does on a context besides the filter
// itself: kernel attributes, occupancy queries, and the loading of every
// kernel of the forward and backward (lazy module loading otherwise loads
// each on its first launch).
template <int PD, int V>
cudaError_t prepare_v(const CallArgs&) {
    constexpr int CPF = pad_ch(V + 1), CPB = pad_ch(V);
    cudaError_t e = prepare_tile_build<PD>();
    int n = 0;
    if (e == cudaSuccess) e = kernel_once(reinterpret_cast<const void*>(k_blur_all<PD, CPF>), blur_attr<PD, CPF>, &n);
    if (e == cudaSuccess) e = kernel_once(reinterpret_cast<const void*>(k_blur_all<PD, CPB>), blur_attr<PD, CPB>, &n);
    if (e == cudaSuccess) e = kernel_once(reinterpret_cast<const void*>(k_insert<PD>), insert_attr<PD>, &n);
    const void* fns[] = {reinterpret_cast<const void*>(k_tile_build<PD>), reinterpret_cast<const void*>(k_clear),
                         reinterpret_cast<const void*>(k_insert<PD>),
                         Cfg<PD>::P == 256 ? reinterpret_cast<const void*>(k_splat_nbr<PD, V, true>)
                                           : reinterpret_cast<const void*>(k_neighbors<PD>),
                         Cfg<PD>::P == 256 ? reinterpret_cast<const void*>(k_splat_nbr<PD, V, false>)
                                           : reinterpret_cast<const void*>(k_splat<PD, V, true>),
                         reinterpret_cast<const void*>(k_splat<PD, V, false>),
                         kSlicePiped<PD> ? reinterpret_cast<const void*>(k_slice_pipe<PD, V, true>)
                                         : reinterpret_cast<const void*>(k_slice<PD, V, true>),
                         kSlicePiped<PD> ? reinterpret_cast<const void*>(k_slice_pipe<PD, V, false>)
                                         : reinterpret_cast<const void*>(k_slice<PD, V, false>),
                         reinterpret_cast<const void*>(k_splat_zeroed<PD, V, true>),
                         reinterpret_cast<const void*>(k_splat_zeroed<PD, V, false>)};
    for (const void* f : fns) {
        cudaFuncAttributes fa;
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, f);
    }
    int n2 = 0;
    if (e == cudaSuccess && kSlicePiped<PD>)
        e = kernel_once(reinterpret_cast<const void*>(k_slice_pipe<PD, V, true>), slice_attr<PD, V, true>, &n2);
    if (e == cudaSuccess && kSlicePiped<PD>)
        e = kernel_once(reinterpret_cast<const void*>(k_slice_pipe<PD, V, false>), slice_attr<PD, V, false>, &n2);
    if (e == cudaSuccess)
        e = kernel_once(reinterpret_cast<const void*>(k_splat_zeroed<PD, V, true>), splat_zeroed_attr<PD, V, true>, &n2);
    if (e == cudaSuccess)
        e = kernel_once(reinterpret_cast<const void*>(k_splat_zeroed<PD, V, false>), splat_zeroed_attr<PD, V, false>,
                        &n2);
    return e;
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
cudaError_t run_filter(const CallArgs& a) { PL_DISPATCH_V(filter_v, PD, a) }

template <int PD>
cudaError_t run_feature_grad(const CallArgs& a) { PL_DISPATCH_V(fgrad_v, PD, a) }

template <int PD>
cudaError_t run_prepare(const CallArgs& a) { PL_DISPATCH_V(prepare_v, PD, a) }

template <int PD>
cudaError_t run_export_keys(const void* lattice, const void* scratch, const PlLayout& lay, int16_t* out,
                            int max_keys, cudaStream_t s) {
    const LatView Lv = lat_view(const_cast<void*>(lattice), lay);
    const ScrView Sv = scr_view(const_cast<void*>(scratch), lay);
    k_export_keys<PD><<<256, 256, 0, s>>>(Sv, Lv.hdr, out, max_keys);
    return cudaGetLastError();
}

}  // namespace pl
