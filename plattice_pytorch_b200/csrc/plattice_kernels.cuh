// plattice_kernels.cuh -- sm_100a kernels of the permutohedral-lattice filter.
//
// Pipeline of one forward call (all on one stream, no host synchronisation):
//   k_tile_build   per tile of P pixels: lattice embedding in registers, the
//                  tile's distinct vertex keys deduplicated in a shared-memory
//                  hash table, [v*w, w] pre-summed per distinct vertex in
//                  shared memory, unique keys + partial sums staged to HBM
//   k_clear        zero the part of the hash table and of the lattice value
//                  buffers that this call uses (sized from the staged count)
//   k_insert       global open-addressed insert of the staged keys, compact
//                  vertex ids allocated per CTA, partial sums reduced with
//                  vector red.global.add into the lattice values
//   k_neighbors    blur neighbours of every vertex resolved once per axis
//   k_blur         K passes of the [1 2 1]/4 stencil over the compact vertices
//   k_slice        barycentric gather back to the pixels and normalisation
// Backward reuses the lattice: k_splat_bwd, k_blur in reverse axis order,
// k_slice without normalisation.
//
// The float steps that decide the lattice keys (elevation, greedy rounding,
// rank, barycentric weights) reproduce the reference's operation order,
// permutohedral.cu:165-233, with the multiply-adds that its --use_fast_math
// build fuses written as explicit fused intrinsics, so that the vertex key set
// is bit-identical to the reference and independent of this file's own
// compiler flags.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "plattice_layout.h"

namespace pl {

// ---------------------------------------------------------------- constants

constexpr uint32_t kBusy = 0xFFFFFFFFu;   // global cell being written
constexpr int kSpinLimit = 1 << 20;       // bounded wait on a tile-local insert
constexpr int kRoundLimit = 1 << 16;      // bounded insert rounds per CTA chunk

template <int PD> struct Cfg {
    static constexpr int K = PD + 1;
    static constexpr int P = PD <= 6 ? 256 : (PD <= 10 ? 128 : 64);   // pixels per tile
    static constexpr int TW = 32, TH = P / 32;
    static constexpr int CW = (4 + 2 * PD + 15) / 16;   // 16-byte words per key record
    static constexpr int NW = 4 * CW;                    // 32-bit words per key record
    static constexpr int SLOTS = P * K;                  // (pixel, corner) slots per tile
    static constexpr int SC = SLOTS <= 512 ? 1024 : (SLOTS <= 1024 ? 2048 : (SLOTS <= 2048 ? 4096 : 8192));
};

__host__ __device__ constexpr int pad_ch(int c) { return c <= 2 ? c : ((c + 3) / 4) * 4; }

struct EmbedConsts {
    float sf[PL_MAX_PD];   // scale factors, permutohedral.cu:507-508 (computed on the host)
    float rk;              // 1/K rounded to float
    float kf;              // K as float
};

struct Geo {
    int h, w, tiles_x, tiles;
    int cap_max_log2, cap_override_log2;
};

struct LatView {
    LatticeHeader* hdr;
    int* tile_off;
    int* tile_cnt;
    uint16_t* slot_lid;
    float* slot_w;
    int* staged_vid;
    int2* nbr;
    float* vb0;
    float* vb1;
};

struct ScrView {
    uint4* skeys;
    float* svals;
    uint4* table;
    uint4* vkeys;
    float* vf0;
    float* vf1;
};

// ---------------------------------------------------------------- memory helpers

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
                 "f"(d) : "memory");
}
__device__ __forceinline__ void red_add_v2(float* p, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add_f32(float* p, float a) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

// red.global.add of CP consecutive floats (CP in {1, 2, 4, 8, 12}); p is CP*4-byte aligned
template <int CP>
__device__ __forceinline__ void red_add_row(float* p, const float* v) {
    if constexpr (CP == 1) {
        red_add_f32(p, v[0]);
    } else if constexpr (CP == 2) {
        red_add_v2(p, v[0], v[1]);
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4) red_add_v4(p + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
}

template <int CP>
__device__ __forceinline__ void load_row(const float* __restrict__ p, float (&v)[CP]) {
    if constexpr (CP == 1) {
        v[0] = __ldg(p);
    } else if constexpr (CP == 2) {
        float2 a = __ldg(reinterpret_cast<const float2*>(p));
        v[0] = a.x; v[1] = a.y;
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4) {
            float4 a = __ldg(reinterpret_cast<const float4*>(p + j));
            v[j] = a.x; v[j + 1] = a.y; v[j + 2] = a.z; v[j + 3] = a.w;
        }
    }
}

// store of CP consecutive floats with the widest aligned vector stores
template <int CP>
__device__ __forceinline__ void store_row(float* p, const float (&v)[CP]) {
    if constexpr (CP == 1) {
        p[0] = v[0];
    } else if constexpr (CP == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4)
            *reinterpret_cast<float4*>(p + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
}

// ---------------------------------------------------------------- hashing

__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
    h ^= h >> 16; h *= 0x85EBCA6Bu;
    h ^= h >> 13; h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

// hash of a key record's coordinate words (word 0 is the hash slot itself)
template <int NW>
__device__ __forceinline__ uint32_t key_hash(const uint32_t (&kw)[NW]) {
    uint32_t h = 0x9E3779B9u;
#pragma unroll
    for (int k = 1; k < NW; ++k) h = fmix32(h ^ kw[k]) + 0x7F4A7C15u * (uint32_t)k;
    return fmix32(h);
}

// ---------------------------------------------------------------- lattice embedding

// float -> int16 as the device conversion does it: truncate, saturate
__device__ __forceinline__ int f2s16(float x) {
    int r = __float2int_rz(x);
    return r < -32768 ? -32768 : (r > 32767 ? 32767 : r);
}

// Greedy remainder-0 point g, simplex rank and barycentric weights of one
// feature vector.  Operation order of permutohedral.cu:165-233; the
// multiply-adds are the fused ones of the reference build.
template <int PD>
__device__ __forceinline__ void embed(const float (&f)[PD], const EmbedConsts& ec, int (&g)[PD + 1],
                                      int (&rank)[PD + 1], float (&bary)[PD + 1]) {
    constexpr int K = PD + 1;
    float e[K];
    e[PD] = __fmul_rn(__fmul_rn((float)(-PD), f[PD - 1]), ec.sf[PD - 1]);
#pragma unroll
    for (int i = PD - 1; i > 0; --i) {
        const float a = __fmul_rn((float)i, f[i - 1]);
        const float c = __fmul_rn((float)(i + 2), f[i]);
        const float s = __fmaf_rn(-a, ec.sf[i - 1], e[i + 1]);
        e[i] = __fmaf_rn(c, ec.sf[i], s);
    }
    e[0] = __fmaf_rn(__fmul_rn(2.0f, f[0]), ec.sf[0], e[1]);

    // nearest multiple of K per coordinate; the running sum is int16
    int sum = 0;
#pragma unroll
    for (int i = 0; i < K; ++i) {
        const float v = __fmul_rn(e[i], ec.rk);
        const float up = __fmul_rn(ceilf(v), ec.kf);
        const float dn = __fmul_rn(floorf(v), ec.kf);
        g[i] = (__fsub_rn(up, e[i]) < __fsub_rn(e[i], dn)) ? f2s16(up) : f2s16(dn);
        sum = (int16_t)(sum + g[i]);
    }
    sum = (int16_t)(sum / K);

    // rank by counting, ties to the lower index
    float d[K];
#pragma unroll
    for (int i = 0; i < K; ++i) d[i] = __fsub_rn(e[i], (float)g[i]);
#pragma unroll
    for (int i = 0; i < K; ++i) {
        int r = 0;
#pragma unroll
        for (int j = 0; j < K; ++j) r += (d[i] < d[j] || (d[i] == d[j] && i > j)) ? 1 : 0;
        rank[i] = r;
    }

    // move the greedy point onto the hyperplane
    if (sum > 0) {
#pragma unroll
        for (int i = 0; i < K; ++i) {
            if (rank[i] >= K - sum) { g[i] -= K; rank[i] += sum - K; }
            else                    { rank[i] += sum; }
        }
    } else if (sum < 0) {
#pragma unroll
        for (int i = 0; i < K; ++i) {
            if (rank[i] < -sum) { g[i] += K; rank[i] += K + sum; }
            else                { rank[i] += sum; }
        }
    }

    // barycentric weights.  Position k receives +delta_i from the coordinate of
    // rank PD-k and -delta_i from the coordinate of rank PD+1-k, applied in
    // increasing i as fused multiply-adds starting from 0: the reference's
    // scatter, evaluated position by position so that it stays in registers.
#pragma unroll
    for (int i = 0; i < K; ++i) d[i] = __fsub_rn(e[i], (float)g[i]);
    float b[K + 1];
#pragma unroll
    for (int k = 0; k <= K; ++k) {
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < K; ++i) {
            if (k <= PD && rank[i] == PD - k) acc = __fmaf_rn(d[i], ec.rk, acc);
            if (k >= 1 && rank[i] == PD + 1 - k) acc = __fmaf_rn(-d[i], ec.rk, acc);
        }
        b[k] = acc;
    }
    b[0] = __fadd_rn(b[0], __fadd_rn(1.0f, b[K]));
#pragma unroll
    for (int k = 0; k < K; ++k) bary[k] = b[k];
}

// Key record of simplex corner c (permutohedral.cu:238-244): coordinate i is
// g[i] + c, minus K where rank[i] > PD - c, stored as int16 halfword i of
// words 1..; word 0 receives the hash.
template <int PD>
__device__ __forceinline__ void make_key(const int (&g)[PD + 1], const int (&rank)[PD + 1], int c,
                                         uint32_t (&kw)[Cfg<PD>::NW]) {
    constexpr int NW = Cfg<PD>::NW;
#pragma unroll
    for (int k = 0; k < NW; ++k) kw[k] = 0u;
#pragma unroll
    for (int i = 0; i < PD; ++i) {
        const int v = g[i] + c - ((rank[i] > PD - c) ? (PD + 1) : 0);
        kw[1 + i / 2] |= ((uint32_t)(uint16_t)(int16_t)v) << (16 * (i & 1));
    }
    kw[0] = key_hash<NW>(kw);
}

// ---------------------------------------------------------------- tile-local dedup

// Insert a key into the tile's shared-memory table; returns its local id.
// Cells hold -1 (empty), -2 (being written) or a local id.  The owner of a
// new key writes the record then publishes the id; other threads wait for
// the publication with a bounded spin.
template <int CW, int SC>
__device__ __forceinline__ int tile_insert(int* stab, uint4* ukeys, const uint32_t (&kw)[4 * CW],
                                           int* count, int* status) {
    uint32_t pos = (kw[0] >> 7) & (SC - 1);
    volatile int* vt = stab;
    for (int probe = 0; probe < SC; ++probe) {
        int cur = vt[pos];
        if (cur == -1) {
            cur = atomicCAS(&stab[pos], -1, -2);
            if (cur == -1) {
                const int lid = atomicAdd(count, 1);
#pragma unroll
                for (int w = 0; w < CW; ++w)
                    ukeys[lid * CW + w] = make_uint4(kw[4 * w], kw[4 * w + 1], kw[4 * w + 2], kw[4 * w + 3]);
                __threadfence_block();
                atomicExch(&stab[pos], lid);
                return lid;
            }
        }
        int spins = 0;
        while (cur == -2) {
            if (++spins > kSpinLimit) { atomicOr(status, PL_ST_SPIN); return 0; }
            cur = vt[pos];
        }
        __threadfence_block();
        const volatile uint4* rec = ukeys + cur * CW;
        bool eq = true;
#pragma unroll
        for (int w = 0; w < CW; ++w) {
            const uint32_t a = rec[w].x, b = rec[w].y, c = rec[w].z, d = rec[w].w;
            eq = eq && a == kw[4 * w] && b == kw[4 * w + 1] && c == kw[4 * w + 2] && d == kw[4 * w + 3];
        }
        if (eq) return cur;
        pos = (pos + 1) & (SC - 1);
    }
    atomicOr(status, PL_ST_SMEM_PROBE);
    return 0;
}

// ---------------------------------------------------------------- K1: tile build (+ forward splat)

template <int PD>
__host__ __device__ constexpr int tile_build_smem_bytes() {
    return Cfg<PD>::SLOTS * Cfg<PD>::CW * 16 + Cfg<PD>::SC * 4;
}

template <int PD, int V>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_tile_build(const float* __restrict__ feat, const float* __restrict__ vals, Geo geo, EmbedConsts ec,
             LatView L, ScrView S) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P, CW = C::CW, NW = C::NW, SLOTS = C::SLOTS, SC = C::SC;
    constexpr int CPF = pad_ch(V + 1);
    constexpr int REGION_FLOATS = tile_build_smem_bytes<PD>() / 4;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4* ukeys = reinterpret_cast<uint4*>(smem_raw);
    int* stab = reinterpret_cast<int*>(ukeys + SLOTS * CW);
    float* part = reinterpret_cast<float*>(smem_raw);   // reused once the keys are staged
    __shared__ int s_count, s_base;

    const int t = threadIdx.x;
    const int tile = blockIdx.x;
    const int x = (tile % geo.tiles_x) * C::TW + (t % C::TW);
    const int y = (tile / geo.tiles_x) * C::TH + (t / C::TW);
    const bool active = x < geo.w && y < geo.h;
    const size_t p = (size_t)y * geo.w + x;

    for (int i = t; i < SC; i += P) stab[i] = -1;
    if (t == 0) s_count = 0;

    float f[PD];
#pragma unroll
    for (int i = 0; i < PD; ++i) f[i] = active ? __ldg(feat + p * PD + i) : 0.0f;
    int g[K], rank[K];
    float bary[K];
    embed<PD>(f, ec, g, rank, bary);
    __syncthreads();

    int lid[K];
#pragma unroll
    for (int c = 0; c < K; ++c) {
        lid[c] = 0;
        if (active) {
            uint32_t kw[NW];
            make_key<PD>(g, rank, c, kw);
            lid[c] = tile_insert<CW, SC>(stab, ukeys, kw, &s_count, &L.hdr->status);
        }
    }
    __syncthreads();
    const int U = s_count;
    if (t == 0) {
        const int b = atomicAdd(&L.hdr->u_total, U);
        s_base = b;
        L.tile_off[tile] = b;
        L.tile_cnt[tile] = U;
    }
    __syncthreads();
    const int base = s_base;
    for (int i = t; i < U * CW; i += P) S.skeys[(size_t)base * CW + i] = ukeys[i];

    const size_t so = (size_t)tile * K * P + t;
#pragma unroll
    for (int c = 0; c < K; ++c) {
        L.slot_lid[so + (size_t)c * P] = (uint16_t)lid[c];
        L.slot_w[so + (size_t)c * P] = active ? bary[c] : 0.0f;
    }
    if (vals == nullptr) return;   // lattice rebuild only (block-uniform)

    float v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = active ? __ldg(vals + p * V + j) : 0.0f;
    __syncthreads();   // staged keys read out of shared memory before it is reused
    if (U * CPF <= REGION_FLOATS) {
        for (int i = t; i < U * CPF; i += P) part[i] = 0.0f;
        __syncthreads();
        if (active) {
#pragma unroll
            for (int c = 0; c < K; ++c) {
                float* pp = part + lid[c] * CPF;
#pragma unroll
                for (int j = 0; j < V; ++j) atomicAdd(pp + j, __fmul_rn(v[j], bary[c]));
                atomicAdd(pp + V, bary[c]);
            }
        }
        __syncthreads();
        float* out = S.svals + (size_t)base * CPF;
        for (int i = t; i < U * CPF; i += P) out[i] = part[i];
    } else {
        float* gp = S.svals + (size_t)base * CPF;
        for (int i = t; i < U * CPF; i += P) gp[i] = 0.0f;
        __syncthreads();
        if (active) {
#pragma unroll
            for (int c = 0; c < K; ++c) {
                float* pp = gp + lid[c] * CPF;
#pragma unroll
                for (int j = 0; j < V; ++j) atomicAdd(pp + j, __fmul_rn(v[j], bary[c]));
                atomicAdd(pp + V, bary[c]);
            }
        }
    }
}

// ---------------------------------------------------------------- K_clear

// Chooses the table capacity from the staged count (load <= 1/2), zeroes the
// cells in use and the first u_total rows of the lattice value buffers that
// are accumulated into (forward vf0 when cpf > 0, backward vb0).
static __global__ void k_clear(Geo geo, LatView L, ScrView S, int cw, int cpf, int cpb) {
    const int U = L.hdr->u_total;
    int lg = 6;
    while ((1ll << lg) < 2ll * U) ++lg;
    if (lg > geo.cap_max_log2) lg = geo.cap_max_log2;
    if (geo.cap_override_log2 > 0)
        lg = geo.cap_override_log2 < geo.cap_max_log2 ? geo.cap_override_log2 : geo.cap_max_log2;
    if (blockIdx.x == 0 && threadIdx.x == 0) L.hdr->cap_log2 = lg;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t cells = ((size_t)1 << lg) * cw;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (size_t i = tid; i < cells; i += stride) S.table[i] = z;
    if (cpf > 0) {
        float4* a = reinterpret_cast<float4*>(S.vf0);
        const size_t nf = (size_t)U * cpf;
        for (size_t i = tid; i < nf / 4; i += stride) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (size_t i = (nf / 4) * 4 + tid; i < nf; i += stride) S.vf0[i] = 0.0f;
    }
    {
        float4* a = reinterpret_cast<float4*>(L.vb0);
        const size_t nb = (size_t)U * cpb;
        for (size_t i = tid; i < nb / 4; i += stride) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (size_t i = (nb / 4) * 4 + tid; i < nb; i += stride) L.vb0[i] = 0.0f;
    }
}

// zero the first m rows of a lattice value buffer (a repeated backward)
static __global__ void k_zero_rows(float* buf, const LatticeHeader* hdr, int cp) {
    const size_t n = (size_t)hdr->m * cp;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) buf[i] = 0.0f;
}

// ---------------------------------------------------------------- global table lookups

template <int CW>
__device__ __forceinline__ bool cell_key_equal(const uint4* cell, const uint32_t (&kw)[4 * CW], uint4 c0) {
    bool eq = c0.y == kw[1] && c0.z == kw[2] && c0.w == kw[3];
#pragma unroll
    for (int w = 1; w < CW; ++w) {
        const uint4 c = __ldcg(cell + w);
        eq = eq && c.x == kw[4 * w] && c.y == kw[4 * w + 1] && c.z == kw[4 * w + 2] && c.w == kw[4 * w + 3];
    }
    return eq;
}

// read-only probe after the table is complete; returns the vertex id or -1
template <int CW>
__device__ __forceinline__ int table_find(const uint4* __restrict__ table, uint32_t mask,
                                          const uint32_t (&kw)[4 * CW], int* status) {
    uint32_t pos = kw[0] & mask;
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        const uint4* cell = table + (size_t)pos * CW;
        const uint4 c0 = __ldg(cell);
        if (c0.x == 0u) return -1;
        bool eq = c0.y == kw[1] && c0.z == kw[2] && c0.w == kw[3];
#pragma unroll
        for (int w = 1; w < CW; ++w) {
            const uint4 c = __ldg(cell + w);
            eq = eq && c.x == kw[4 * w] && c.y == kw[4 * w + 1] && c.z == kw[4 * w + 2] && c.w == kw[4 * w + 3];
        }
        if (eq && c0.x != kBusy) return (int)c0.x - 1;
        pos = (pos + 1) & mask;
    }
    atomicOr(status, PL_ST_TABLE_FULL);
    return -1;
}

// ---------------------------------------------------------------- K2: global insert

// One thread per staged key.  Each CTA works in rounds: every unresolved
// thread probes without waiting (a cell being written by another thread ends
// its probe for this round), winners of an empty cell get compact vertex ids
// from one atomicAdd per CTA, write the vertex record and publish the cell.
// Nobody spins, so every round ends and a published cell is seen next round.
template <int PD, int CPF>
__global__ void __launch_bounds__(256) k_insert(LatView L, ScrView S, int with_values) {
    constexpr int CW = Cfg<PD>::CW, NW = Cfg<PD>::NW;
    __shared__ int s_nwin, s_vbase;
    const int U = L.hdr->u_total;
    const uint32_t mask = (1u << L.hdr->cap_log2) - 1u;
    if (threadIdx.x == 0) s_nwin = 0;
    __syncthreads();
    for (int base = blockIdx.x * blockDim.x; base < U; base += gridDim.x * blockDim.x) {
        const int i = base + threadIdx.x;
        bool pending = i < U, won = false;
        uint32_t kw[NW];
#pragma unroll
        for (int k = 0; k < NW; ++k) kw[k] = 0u;
        if (pending) {
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const uint4 r = S.skeys[(size_t)i * CW + w];
                kw[4 * w] = r.x; kw[4 * w + 1] = r.y; kw[4 * w + 2] = r.z; kw[4 * w + 3] = r.w;
            }
        }
        uint32_t pos = kw[0] & mask, probes = 0;
        int vid = -1;
        for (int round = 0;; ++round) {
            if (pending && !won) {
                for (;;) {
                    uint4* cell = S.table + (size_t)pos * CW;
                    uint32_t* state = reinterpret_cast<uint32_t*>(cell);
                    uint32_t st = ld_acquire(state);
                    if (st == 0u) {
                        if (atomicCAS(state, 0u, kBusy) == 0u) {
                            uint32_t* cw32 = reinterpret_cast<uint32_t*>(cell);
#pragma unroll
                            for (int k = 1; k < NW; ++k) cw32[k] = kw[k];
                            won = true;
                            break;
                        }
                        st = ld_acquire(state);   // lost the race: see who won, with acquire
                        if (st == 0u) {           // cells never return to empty; stay bounded anyway
                            if (++probes > mask) {
                                atomicOr(&L.hdr->status, PL_ST_TABLE_FULL);
                                pending = false;
                                break;
                            }
                            continue;
                        }
                    }
                    if (st == kBusy) break;   // written right now: look again next round
                    const uint4 c0 = __ldcg(cell);
                    if (cell_key_equal<CW>(cell, kw, c0)) {
                        vid = (int)st - 1;
                        pending = false;
                        break;
                    }
                    pos = (pos + 1) & mask;
                    if (++probes > mask) {
                        atomicOr(&L.hdr->status, PL_ST_TABLE_FULL);
                        pending = false;
                        break;
                    }
                }
            }
            int local = 0;
            if (won) local = atomicAdd(&s_nwin, 1);
            __syncthreads();
            if (threadIdx.x == 0) {
                const int nw = s_nwin;
                s_vbase = nw ? atomicAdd(&L.hdr->m, nw) : 0;
                s_nwin = 0;
            }
            __syncthreads();
            if (won) {
                vid = s_vbase + local;
#pragma unroll
                for (int w = 0; w < CW; ++w)
                    S.vkeys[(size_t)vid * CW + w] = make_uint4(kw[4 * w], kw[4 * w + 1], kw[4 * w + 2], kw[4 * w + 3]);
                __threadfence();
                st_release(reinterpret_cast<uint32_t*>(S.table + (size_t)pos * CW), (uint32_t)vid + 1u);
                won = false;
                pending = false;
            }
            if (!__syncthreads_or(pending)) break;
            if (round >= kRoundLimit) {
                if (threadIdx.x == 0) atomicOr(&L.hdr->status, PL_ST_ROUNDS);
                break;
            }
        }
        if (i < U) {
            L.staged_vid[i] = vid;
            if (with_values && vid >= 0) {
                float r[CPF];
                const float* src = S.svals + (size_t)i * CPF;
#pragma unroll
                for (int j = 0; j < CPF; ++j) r[j] = __ldcg(src + j);
                red_add_row<CPF>(S.vf0 + (size_t)vid * CPF, r);
            }
        }
    }
}

// ---------------------------------------------------------------- K3: blur neighbours

// neighbour of key along axis c: every coordinate +1 (or -1), coordinate c
// (when c < PD) additionally -K (or +K); permutohedral.cu:368-375.
template <int PD>
__global__ void __launch_bounds__(256) k_neighbors(LatView L, ScrView S) {
    constexpr int K = PD + 1, CW = Cfg<PD>::CW, NW = Cfg<PD>::NW;
    const int M = L.hdr->m;
    const uint32_t mask = (1u << L.hdr->cap_log2) - 1u;
    const size_t total = (size_t)M * K;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int c = (int)(idx / M);
        const int v = (int)(idx - (size_t)c * M);
        uint32_t kp[NW], km[NW];
#pragma unroll
        for (int w = 0; w < CW; ++w) {
            const uint4 r = __ldg(S.vkeys + (size_t)v * CW + w);
            kp[4 * w] = r.x; kp[4 * w + 1] = r.y; kp[4 * w + 2] = r.z; kp[4 * w + 3] = r.w;
        }
#pragma unroll
        for (int k = 1; k < NW; ++k) {
            // +1 on the halfwords that hold coordinates, 0 on padding
            const int lo = 2 * (k - 1), hi = lo + 1;
            const uint32_t ones = (lo < PD ? 0x0001u : 0u) | (hi < PD ? 0x00010000u : 0u);
            uint32_t step = 0u;
            if (c < PD && (c >> 1) == k - 1) step = (uint32_t)K << (16 * (c & 1));
            const uint32_t w0 = kp[k];
            kp[k] = __vsub2(__vadd2(w0, ones), step);
            km[k] = __vadd2(__vsub2(w0, ones), step);
        }
        kp[0] = key_hash<NW>(kp);
        km[0] = key_hash<NW>(km);
        const int a = table_find<CW>(S.table, mask, kp, &L.hdr->status);
        const int b = table_find<CW>(S.table, mask, km, &L.hdr->status);
        L.nbr[(size_t)c * M + v] = make_int2(a, b);
    }
}

// ---------------------------------------------------------------- blur

// out[v] = (2 in[v] + in[n+] + in[n-]) / 4 along one axis; a missing neighbour
// adds nothing (permutohedral.cu:341-347).
template <int CP>
__global__ void __launch_bounds__(256) k_blur(const float* __restrict__ in, float* __restrict__ out,
                                              const int2* __restrict__ nbr, const LatticeHeader* hdr,
                                              int axis, int nch) {
    const int M = hdr->m;
    const int2* nb = nbr + (size_t)axis * M;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < (size_t)M; v += stride) {
        const int2 n = __ldg(nb + v);
        float me[CP], a[CP], b[CP];
        load_row<CP>(in + v * CP, me);
        if (n.x >= 0) load_row<CP>(in + (size_t)n.x * CP, a);
        if (n.y >= 0) load_row<CP>(in + (size_t)n.y * CP, b);
        float r[CP];
#pragma unroll
        for (int j = 0; j < CP; ++j) {
            float acc = __fmul_rn(2.0f, me[j]);
            if (n.x >= 0) acc = __fadd_rn(acc, a[j]);
            if (n.y >= 0) acc = __fadd_rn(acc, b[j]);
            r[j] = __fmul_rn(0.25f, acc);
        }
        store_row<CP>(out + v * CP, r);
    }
}

// ---------------------------------------------------------------- slice

// FWD: out = sum_i w_i val_i[0:V] / sum_i w_i val_i[V], weight_out = 1/sum;
// otherwise the unnormalised gather of V channels (permutohedral.cu:401-413,
// 487-496).
template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_slice(float* __restrict__ out, float* __restrict__ wout, Geo geo, LatView L, const float* __restrict__ lat) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P, SLOTS = C::SLOTS;
    constexpr int CP = FWD ? pad_ch(V + 1) : pad_ch(V);
    constexpr int NC = FWD ? V + 1 : V;
    __shared__ int svid[SLOTS];
    const int t = threadIdx.x, tile = blockIdx.x;
    const int cnt = L.tile_cnt[tile], off = L.tile_off[tile];
    for (int u = t; u < cnt; u += P) svid[u] = L.staged_vid[off + u];
    __syncthreads();
    const int x = (tile % geo.tiles_x) * C::TW + (t % C::TW);
    const int y = (tile / geo.tiles_x) * C::TH + (t / C::TW);
    if (x >= geo.w || y >= geo.h) return;
    const size_t p = (size_t)y * geo.w + x;
    const size_t so = (size_t)tile * K * P + t;
    float acc[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const int lid = L.slot_lid[so + (size_t)c * P];
        const float w = L.slot_w[so + (size_t)c * P];
        const int vid = svid[lid];
        if (vid < 0) continue;   // failed insert (reported in the status word)
        float r[CP];
        load_row<CP>(lat + (size_t)vid * CP, r);
#pragma unroll
        for (int j = 0; j < NC; ++j) acc[j] = __fmaf_rn(w, r[j], acc[j]);
    }
    if constexpr (FWD) {
        const float inv = 1.0f / acc[V];
#pragma unroll
        for (int j = 0; j < V; ++j) out[p * V + j] = acc[j] * inv;
        wout[p] = inv;
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) out[p * V + j] = acc[j];
    }
}

// ---------------------------------------------------------------- backward splat

// value (grad * weight_in) * w per slot (permutohedral.cu:437-445), summed per
// tile-unique vertex in shared memory, then one vector red per vertex.
template <int PD, int V>
__host__ __device__ constexpr int bsplat_part_floats() {
    return Cfg<PD>::SLOTS * pad_ch(V) <= 8192 ? Cfg<PD>::SLOTS * pad_ch(V) : 8192;
}

template <int PD, int V>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_splat_bwd(const float* __restrict__ grad, const float* __restrict__ wt, Geo geo, LatView L, float* vb) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P, SLOTS = C::SLOTS;
    constexpr int CP = pad_ch(V);
    constexpr int PF = bsplat_part_floats<PD, V>();
    __shared__ int svid[SLOTS];
    __shared__ __align__(16) float part[PF];
    const int t = threadIdx.x, tile = blockIdx.x;
    const int cnt = L.tile_cnt[tile], off = L.tile_off[tile];
    const bool in_smem = cnt * CP <= PF;
    for (int u = t; u < cnt; u += P) svid[u] = L.staged_vid[off + u];
    if (in_smem)
        for (int i = t; i < cnt * CP; i += P) part[i] = 0.0f;
    __syncthreads();
    const int x = (tile % geo.tiles_x) * C::TW + (t % C::TW);
    const int y = (tile / geo.tiles_x) * C::TH + (t / C::TW);
    if (x < geo.w && y < geo.h) {
        const size_t p = (size_t)y * geo.w + x;
        const float wp = __ldg(wt + p);
        float gw[V];
#pragma unroll
        for (int j = 0; j < V; ++j) gw[j] = __fmul_rn(__ldg(grad + p * V + j), wp);
        const size_t so = (size_t)tile * K * P + t;
#pragma unroll
        for (int c = 0; c < K; ++c) {
            const int lid = L.slot_lid[so + (size_t)c * P];
            const float w = L.slot_w[so + (size_t)c * P];
            if (in_smem) {
                float* pp = part + lid * CP;
#pragma unroll
                for (int j = 0; j < V; ++j) atomicAdd(pp + j, __fmul_rn(gw[j], w));
            } else if (svid[lid] >= 0) {
                float* gp = vb + (size_t)svid[lid] * CP;
#pragma unroll
                for (int j = 0; j < V; ++j) red_add_f32(gp + j, __fmul_rn(gw[j], w));
            }
        }
    }
    if (!in_smem) return;
    __syncthreads();
    for (int u = t; u < cnt; u += P) {
        if (svid[u] < 0) continue;
        float r[CP];
#pragma unroll
        for (int j = 0; j < CP; ++j) r[j] = part[u * CP + j];
        red_add_row<CP>(vb + (size_t)svid[u] * CP, r);
    }
}

// ---------------------------------------------------------------- key export (tests)

template <int PD>
__global__ void k_export_keys(const ScrView S, const LatticeHeader* hdr, int16_t* out, int max_keys) {
    constexpr int CW = Cfg<PD>::CW;
    const int M = hdr->m < max_keys ? hdr->m : max_keys;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < M; v += gridDim.x * blockDim.x) {
        const uint32_t* r = reinterpret_cast<const uint32_t*>(S.vkeys + (size_t)v * CW);
#pragma unroll
        for (int i = 0; i < PD; ++i) out[(size_t)v * PD + i] = (int16_t)(r[1 + i / 2] >> (16 * (i & 1)));
    }
}

}  // namespace pl
