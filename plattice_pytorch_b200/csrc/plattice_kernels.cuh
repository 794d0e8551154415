// plattice_kernels.cuh -- sm_100a kernels of the permutohedral-lattice filter.
//
// Pipeline of one forward call (no host synchronisation):
//   k_tile_build   per tile of P pixels: lattice embedding in registers; the
//                  tile's distinct vertex keys deduplicated in a shared-memory
//                  hash table (16-bit local ids); unique keys staged to HBM;
//                  the tile's slots counting-sorted by local id
//   k_clear        zero the part of the global hash table this call uses
//   k_insert       global open-addressed insert of the staged keys (tagged
//                  cells); compact vertex ids for the owners, one atomic per
//                  CTA chunk
//   k_splat_nbr    blur neighbours of every vertex by table lookup (the first
//                  CTAs) and the splat (the others): per tile, [v*w, w] summed
//                  over the sorted runs of equal vertex, one vector
//                  red.global.add per run piece.  Large pd: k_neighbors, then
//                  k_splat
//   k_blur_all     the pd+1 passes of the [1 2 1]/4 stencil over the compact
//                  vertex list: one cooperative launch with grid barriers
//                  between passes
//   k_slice_pipe   barycentric gather back to the pixels and normalisation;
//                  persistent CTAs that stream the tiles' slot records into
//                  shared memory (k_slice for tiles of fewer than 256 pixels)
// Backward reuses the lattice: k_splat of grad * weight, k_blur_all in
// reverse axis order, the slice without normalisation.
//
// The float steps that decide the lattice keys (elevation, greedy rounding,
// rank, barycentric weights) reproduce the reference's operation order,
// permutohedral.cu:165-233, with the multiply-adds that its --use_fast_math
// build fuses written as explicit fused intrinsics, so that the vertex key set
// is bit-identical to the reference and independent of this file's own
// compiler flags.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "plattice_layout.h"

namespace pl {

// ---------------------------------------------------------------- constants


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

// Blocks per SM a per-tile kernel asks the compiler for: full occupancy (32
// registers) for the small feature and value dimensions, where the kernels
// fit in them without spilling; the compiler's choice otherwise.
template <int PD, int V>
__host__ __device__ constexpr int slice_min_blocks() { return (PD <= 7 && V <= 4) ? 2048 / Cfg<PD>::P : 1; }

struct EmbedConsts {
    float sf[PL_MAX_PD];   // scale factors, permutohedral.cu:507-508 (computed on the host)
    float rk;              // 1/K rounded to float
    float kf;              // K as float
};

struct Geo {
    int h, w, tiles_x, tiles;   // tiles: of all images
    int tiles_img;              // tiles per image
    long long n_img;            // pixels per image
    int cap_max_log2, cap_override_log2;
    int idx_bits;   // bits that hold 1 + any staged index of the call (global table cells)
    int filter_min_log2;   // table size (log2 cells) from which lookups consult the miss filter
};

// Image, tile origin and first pixel of tile `tile` (tiles numbered image by
// image, row-major within an image).
struct TilePos {
    int img, x0, y0;
    long long pix0;   // index of pixel (x0, y0) in the [b][h][w] pixel array
};

// The tile of a CTA in a grid of (tiles_x, tiles_y, images) blocks: no
// divisions; *tile receives the linear tile index.
template <int TW, int TH>
__device__ __forceinline__ TilePos tile_pos_grid(const Geo& g, int* tile) {
    TilePos t;
    t.img = blockIdx.z;
    t.x0 = blockIdx.x * TW;
    t.y0 = blockIdx.y * TH;
    t.pix0 = (long long)t.img * g.n_img + (long long)t.y0 * g.w + t.x0;
    *tile = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
    return t;
}

template <int TW, int TH>
__device__ __forceinline__ TilePos tile_pos(const Geo& g, int tile) {
    TilePos t;
    t.img = tile / g.tiles_img;
    const int ti = tile - t.img * g.tiles_img;
    const int ty = ti / g.tiles_x;
    t.x0 = (ti - ty * g.tiles_x) * TW;
    t.y0 = ty * TH;
    t.pix0 = (long long)t.img * g.n_img + (long long)t.y0 * g.w + t.x0;
    return t;
}

// The tiles first, first + stride, first + 2 stride, ... of a persistent
// CTA: (image, tile row, tile column) advanced by mixed-radix addition, one
// division per CTA instead of two per tile.
struct TileWalk {
    int tx, ty, img;      // position of the current tile
    int dx, dy, dimg;     // the stride in the same radix
    int tiles_x, tiles_y;
    __device__ __forceinline__ TileWalk(const Geo& g, int first, int stride) {
        tiles_x = g.tiles_x;
        tiles_y = g.tiles_img / g.tiles_x;
        img = first / g.tiles_img;
        int r = first - img * g.tiles_img;
        ty = r / tiles_x;
        tx = r - ty * tiles_x;
        dimg = stride / g.tiles_img;
        r = stride - dimg * g.tiles_img;
        dy = r / tiles_x;
        dx = r - dy * tiles_x;
    }
    __device__ __forceinline__ void advance() {
        tx += dx;
        ty += dy;
        img += dimg;
        if (tx >= tiles_x) { tx -= tiles_x; ++ty; }
        if (ty >= tiles_y) { ty -= tiles_y; ++img; }
    }
    template <int TW, int TH>
    __device__ __forceinline__ TilePos pos(const Geo& g) const {
        TilePos t;
        t.img = img;
        t.x0 = tx * TW;
        t.y0 = ty * TH;
        t.pix0 = (long long)img * g.n_img + (long long)t.y0 * g.w + t.x0;
        return t;
    }
};

struct LatView {
    LatticeHeader* hdr;
    int* tile_off;
    int* tile_cnt;
    uint16_t* slot_lid;
    float* slot_w;
    uint16_t* slot_order;
    float* slot_wsort;
    uint16_t* first_lid;
    int* staged_vid;
    int2* nbr;
};

struct ScrView {
    uint4* skeys;
    uint32_t* table;
    uint32_t* filter;   // miss filter: one byte per table cell, used for large tables
    int* owner;     // [U] staged index of the owner of each staged key
    int* vid_of;    // [U] vertex id of each owner
    uint4* vkeys;
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

// load of CP consecutive floats through L2 only (data written in this launch)
template <int CP>
__device__ __forceinline__ void load_row_cg(const float* p, float (&v)[CP]) {
    if constexpr (CP == 1) {
        v[0] = __ldcg(p);
    } else if constexpr (CP == 2) {
        float2 a = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = a.x; v[1] = a.y;
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4) {
            float4 a = __ldcg(reinterpret_cast<const float4*>(p + j));
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

// Rows of CP bfloat16 values (the reduced-precision blur rows of large
// lattices): a bf16 value is the upper half of a float, so widening is exact;
// narrowing rounds to nearest even.  Rows of 4k values are 8k bytes, read and
// written as 8-byte words (their offsets are multiples of 8 bytes).
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf16_pack(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <int CP>
__device__ __forceinline__ void load_row_bf16(const uint16_t* p, float (&v)[CP]) {
    if constexpr (CP == 1) {
        v[0] = __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p)) << 16);
    } else if constexpr (CP == 2) {
        const uint32_t w = __ldcg(reinterpret_cast<const unsigned int*>(p));
        v[0] = bf16_lo(w); v[1] = bf16_hi(w);
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4) {
            const uint2 w = __ldcg(reinterpret_cast<const uint2*>(p + j));
            v[j] = bf16_lo(w.x); v[j + 1] = bf16_hi(w.x); v[j + 2] = bf16_lo(w.y); v[j + 3] = bf16_hi(w.y);
        }
    }
}

template <int CP>
__device__ __forceinline__ void store_row_bf16(uint16_t* p, const float (&v)[CP]) {
    if constexpr (CP == 1) {
        *p = (uint16_t)(bf16_pack(v[0], 0.0f) & 0xFFFFu);
    } else if constexpr (CP == 2) {
        *reinterpret_cast<uint32_t*>(p) = bf16_pack(v[0], v[1]);
    } else {
#pragma unroll
        for (int j = 0; j < CP; j += 4)
            *reinterpret_cast<uint2*>(p + j) = make_uint2(bf16_pack(v[j], v[j + 1]), bf16_pack(v[j + 2], v[j + 3]));
    }
}

// ---------------------------------------------------------------- packed int16 keys

// Two int16 key coordinates per 32-bit word.  Per-halfword wrap-around add in
// plain integer arithmetic: the low halfwords' carry is kept out of the high
// halfword by adding 15-bit parts and restoring the top bit with an XOR.
__device__ __forceinline__ uint32_t hw_add(uint32_t a, uint32_t b) {
    return ((a & 0x7FFF7FFFu) + (b & 0x7FFF7FFFu)) ^ ((a ^ b) & 0x80008000u);
}

__device__ __forceinline__ uint32_t pack_hw(int lo, int hi) {
    return (uint32_t)(uint16_t)lo | ((uint32_t)(uint16_t)hi << 16);
}

// ---------------------------------------------------------------- hashing

__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
    h ^= h >> 16; h *= 0x85EBCA6Bu;
    h ^= h >> 13; h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

// Key hash.  Its linear part is the sum of the int16 coordinates
// (sign-extended) times odd per-coordinate multipliers, mod 2^32, so that a
// step of the key by a vector d moves it by sum d_i * mul_i: a blur
// neighbour's hash is the vertex's plus a per-axis constant (the same idea as
// the reference's hash offsets, permutohedral.cu:50-53).  The stored hash is
// that sum after an avalanche (fmix32), for the table positions and tags.
__host__ __device__ constexpr uint32_t coord_mul(int i) {
    switch (i) {
        case 0: return 0x2AE75E2Fu;  case 1: return 0x9C2B9D9Fu;  case 2: return 0x4F876AA3u;
        case 3: return 0x02FF349Du;  case 4: return 0xBAEC4EF7u;  case 5: return 0xE06C85AFu;
        case 6: return 0x21F64545u;  case 7: return 0xE7158A81u;  case 8: return 0x819ED6B7u;
        case 9: return 0x3C95AD21u;  case 10: return 0x8BE9794Du; case 11: return 0x3C7BA9E3u;
        case 12: return 0x022DD18Du; case 13: return 0x4D317C69u; case 14: return 0x7965C0FFu;
        default: return 0x8ECA7365u;
    }
}

// Inverse of fmix32: the xor-shifts undone in reverse order, the odd
// multipliers replaced by their inverses mod 2^32 (Newton's iteration
// x <- x (2 - a x), exact after five steps from x = a for odd a).
__host__ __device__ constexpr uint32_t inv_odd(uint32_t a) {
    uint32_t x = a;
    for (int i = 0; i < 5; ++i) x *= 2u - a * x;
    return x;
}
static_assert(0x85EBCA6Bu * inv_odd(0x85EBCA6Bu) == 1u && 0xC2B2AE35u * inv_odd(0xC2B2AE35u) == 1u,
              "modular inverses of the avalanche multipliers");

__host__ __device__ __forceinline__ uint32_t fmix32_inv(uint32_t h) {
    h ^= h >> 16;
    h *= inv_odd(0xC2B2AE35u);
    h ^= (h >> 13) ^ (h >> 26);
    h *= inv_odd(0x85EBCA6Bu);
    h ^= h >> 16;
    return h;
}

// The stored hash of a key: the avalanche of its linear part plus the image's
// salt (image index times an odd constant).  Keys of different images with
// equal coordinates therefore differ in their hash word (fmix32 is a
// bijection and the salts differ mod 2^32), and every key comparison, which
// includes the hash word, keeps the images of a batch apart.  The linear part
// (with the salt) is recovered from the hash by the inverse avalanche, so a
// neighbour's hash follows from the vertex's stored hash alone.
constexpr uint32_t kHashSalt = 0x9E3779B9u;
constexpr uint32_t kImageMul = 0x61C88647u;   // odd
__device__ __forceinline__ uint32_t hash_of_lin(uint32_t lin) { return fmix32(lin ^ kHashSalt); }
__device__ __forceinline__ uint32_t lin_of_hash(uint32_t h) { return fmix32_inv(h) ^ kHashSalt; }
__device__ __forceinline__ uint32_t image_salt(int img) { return (uint32_t)img * kImageMul; }

// coordinate i (sign-extended int16) of a packed key record
__device__ __forceinline__ int key_coord(const uint32_t* kw, int i) {
    return (int)(int16_t)(uint16_t)(kw[1 + i / 2] >> (16 * (i & 1)));
}

template <int PD>
__device__ __forceinline__ uint32_t key_lin_words(const uint32_t* kw) {
    uint32_t lin = 0u;
#pragma unroll
    for (int i = 0; i < PD; ++i) lin += (uint32_t)key_coord(kw, i) * coord_mul(i);
    return lin;
}

// the change of the linear part for the blur step along axis c: every
// coordinate +1, and coordinate c -K when c < PD (permutohedral.cu:368-375)
__host__ __device__ constexpr uint32_t coord_mul_sum(int pd) { return pd <= 0 ? 0u : coord_mul(pd - 1) + coord_mul_sum(pd - 1); }

static __constant__ uint32_t c_coord_mul[16] = {coord_mul(0),  coord_mul(1),  coord_mul(2),  coord_mul(3),
                                                coord_mul(4),  coord_mul(5),  coord_mul(6),  coord_mul(7),
                                                coord_mul(8),  coord_mul(9),  coord_mul(10), coord_mul(11),
                                                coord_mul(12), coord_mul(13), coord_mul(14), coord_mul(15)};

// (axis c may be a run-time value: one constant-bank load)
template <int PD>
__device__ __forceinline__ uint32_t axis_lin_step(int c) {
    constexpr uint32_t all = coord_mul_sum(PD);
    return c < PD ? all - (uint32_t)(PD + 1) * c_coord_mul[c] : all;
}

// ---------------------------------------------------------------- lattice embedding

// float -> int16 as the device conversion does it: truncate, saturate, NaN -> 0
__device__ __forceinline__ int f2s16(float x) {
    short r;
    asm("cvt.rzi.s16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return (int)r;
}

// Greedy remainder-0 point g, simplex rank and barycentric weights of one
// feature vector.  Operation order of permutohedral.cu:165-233; the
// multiply-adds are the fused ones of the reference build.  `col` is this
// thread's column (stride P) of 2K ints of shared scratch.
template <int PD>
__device__ __forceinline__ void embed(const float (&f)[PD], const EmbedConsts& ec, int (&g)[PD + 1],
                                      int (&rank)[PD + 1], float (&bary)[PD + 1], int* col, int (&ir)[PD + 1]) {
    constexpr int P = Cfg<PD>::P;
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

    // nearest multiple of K per coordinate; the running sum is int16 (wrapped
    // once at the end: addition mod 2^16 does not depend on where it wraps)
    int sum = 0;
#pragma unroll
    for (int i = 0; i < K; ++i) {
        const float v = __fmul_rn(e[i], ec.rk);
        const float up = __fmul_rn(ceilf(v), ec.kf);
        const float dn = __fmul_rn(floorf(v), ec.kf);
        g[i] = f2s16((__fsub_rn(up, e[i]) < __fsub_rn(e[i], dn)) ? up : dn);   // one conversion
        sum += g[i];
    }
    sum = (int16_t)((int16_t)sum / K);
    // |sum| <= K/2 for finite features within the int16 key range; the clamp
    // only keeps NaN or saturated coordinates (no defined result) from moving
    // ranks outside [0, K)
    sum = sum > PD ? PD : (sum < -PD ? -PD : sum);

    // rank by counting, ties to the lower index: of each pair i < j, i
    // outranks j when d[i] < d[j], else j outranks i (one comparison per pair)
    float d[K];
#pragma unroll
    for (int i = 0; i < K; ++i) d[i] = __fsub_rn(e[i], (float)g[i]);
#pragma unroll
    for (int i = 0; i < K; ++i) rank[i] = 0;
#pragma unroll
    for (int i = 0; i < K; ++i) {
#pragma unroll
        for (int j = i + 1; j < K; ++j) {
            const int lt = d[i] < d[j] ? 1 : 0;
            rank[i] += lt;
            rank[j] += 1 - lt;
        }
    }

    // move the greedy point onto the hyperplane, without branches: for sum > 0
    // the coordinates of rank >= K - sum move by -K, for sum < 0 those of rank
    // < -sum (K-1-rank >= K + sum) move by +K, for sum == 0 none (threshold K);
    // every rank then shifts by sum plus the move
    {
        const bool flip = sum < 0;
        const int thr = K - (flip ? -sum : sum);
        const int step = flip ? K : -K;
#pragma unroll
        for (int i = 0; i < K; ++i) {
            const int mv = ((flip ? K - 1 - rank[i] : rank[i]) >= thr) ? step : 0;
            g[i] += mv;
            rank[i] += sum + mv;
        }
    }

    // barycentric weights.  Position k receives +delta_i from the coordinate of
    // rank PD-k and -delta_i from the coordinate of rank PD+1-k, applied in
    // increasing i as fused multiply-adds starting from 0 (the reference's
    // scatter).  The deltas and coordinate indices are put in rank order
    // through this thread's shared-memory column, then read position by
    // position.
#pragma unroll
    for (int i = 0; i < K; ++i) {
        col[rank[i] * P] = __float_as_int(__fsub_rn(e[i], (float)g[i]));
        col[(K + rank[i]) * P] = i;
    }
    float dr[K];
#pragma unroll
    for (int r = 0; r < K; ++r) {
        dr[r] = __int_as_float(col[r * P]);
        ir[r] = col[(K + r) * P];
    }
    float b[K + 1];
    b[0] = __fmaf_rn(dr[PD], ec.rk, 0.0f);
#pragma unroll
    for (int k = 1; k <= PD; ++k) {
        const float dp = dr[PD - k], dm = dr[PD + 1 - k];
        const bool plus_first = ir[PD - k] < ir[PD + 1 - k];
        const float first = plus_first ? dp : -dm;
        const float second = plus_first ? -dm : dp;
        b[k] = __fmaf_rn(second, ec.rk, __fmaf_rn(first, ec.rk, 0.0f));
    }
    b[K] = __fmaf_rn(-dr[0], ec.rk, 0.0f);
    b[0] = __fadd_rn(b[0], __fadd_rn(1.0f, b[K]));
#pragma unroll
    for (int k = 0; k < K; ++k) bary[k] = b[k];
}

// Key record of simplex corner c (permutohedral.cu:238-244): coordinate i is
// g[i] + c, minus K where rank[i] > PD - c, stored as int16 halfword i of
// words 1..; word 0 receives the hash.
template <int PD>
__device__ __forceinline__ void make_key(const int (&g)[PD + 1], const int (&rank)[PD + 1], int c, uint32_t salt,
                                         uint32_t (&kw)[Cfg<PD>::NW]) {
    constexpr int NW = Cfg<PD>::NW;
#pragma unroll
    for (int k = 0; k < NW; ++k) kw[k] = 0u;
#pragma unroll
    for (int i = 0; i < PD; ++i) {
        const int v = g[i] + c - ((rank[i] > PD - c) ? (PD + 1) : 0);
        kw[1 + i / 2] |= ((uint32_t)(uint16_t)(int16_t)v) << (16 * (i & 1));   // int16 wrap-around
    }
    kw[0] = hash_of_lin(key_lin_words<PD>(kw) + salt);
}

// ---------------------------------------------------------------- warp helpers

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------- block scan

// Exclusive prefix sum of a[0..n) in place by warp 0 alone (a few elements
// per lane), a[n] = the total.  The caller synchronises before (counts
// complete) and after (offsets visible).
__device__ __forceinline__ void warp0_scan_excl(int* a, int n) {
    const int lane = threadIdx.x;
    if (lane >= 32) return;
    const int per = (n + 31) / 32;
    const int b = lane * per, e = min(n, b + per);
    int sum = 0;
    for (int i = b; i < e; ++i) sum += a[i];
    int x = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(kFull, x, d);
        if (lane >= d) x += y;
    }
    int run = x - sum;
    for (int i = b; i < e; ++i) {
        const int v = a[i];
        a[i] = run;
        run += v;
    }
    if (lane == 31) a[n] = x;
}

// ---------------------------------------------------------------- K1: tile build

template <int PD>
__host__ __device__ constexpr int tile_build_smem_bytes() {
    return Cfg<PD>::SLOTS * Cfg<PD>::CW * 16 + Cfg<PD>::SC * 4 + Cfg<PD>::SLOTS * 2;
}

// Zero n floats from p by the P threads of a CTA (float4 stores when p is
// 16-byte aligned and n a multiple of 4).
template <int P>
__device__ __forceinline__ void zero_rows_block(float* p, int n, bool vec4) {
    if (vec4) {
        const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int i = threadIdx.x; 4 * i < n; i += P) reinterpret_cast<float4*>(p)[i] = z;
    } else {
        for (int i = threadIdx.x; i < n; i += P) p[i] = 0.0f;
    }
}

// CTAs of k_tile_build that fit on an SM by shared memory (228 KB, 1 KB of it
// reserved per CTA), at most 2048 threads: the register budget is set so that
// registers do not become the tighter limit.
template <int PD>
__host__ __device__ constexpr int tile_build_ctas_per_sm() {
    constexpr int by_smem = (228 * 1024) / (tile_build_smem_bytes<PD>() + 1024 + 64);
    constexpr int by_threads = 2048 / Cfg<PD>::P;
    return by_smem < 1 ? 1 : (by_smem < by_threads ? by_smem : by_threads);
}

// Per tile of P pixels (one thread per pixel):
//  1. lattice embedding in registers;
//  2. every slot (pixel, corner) writes its key record to shared memory; one
//     lane per distinct key of the warp (equal hash, then checked word by word
//     against the group leader) inserts the record's index into the tile hash
//     table with a CAS -- the first index to land in a cell owns the key, later
//     equal keys read the owner's record and take its index, so no cell is ever
//     half-written and nobody waits;
//  3. owners get compact local ids; the tile's unique keys are staged to HBM,
//     the per-slot (local id, weight) records written, and the tile's rows
//     [base, base + U) of the lattice value buffers zeroed (the union of all
//     tiles' rows covers every vertex id, since ids are < the staged count).
template <int PD>
__global__ void __launch_bounds__(Cfg<PD>::P, tile_build_ctas_per_sm<PD>())
k_tile_build(const float* __restrict__ feat, Geo geo, EmbedConsts ec, LatView L, ScrView S,
             float* zero_f, int cpf, float* zero_b, int cpb) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P, CW = C::CW, NW = C::NW, SLOTS = C::SLOTS, SC = C::SC;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4* ukeys = reinterpret_cast<uint4*>(smem_raw);                  // [SLOTS][CW]
    int* stab = reinterpret_cast<int*>(ukeys + SLOTS * CW);             // [SC]
    int16_t* cand_lid = reinterpret_cast<int16_t*>(stab + SC);          // [SLOTS]
    __shared__ int s_count, s_base;

    const int t = threadIdx.x, lane = t & 31;
    int tile;
    const TilePos tp = tile_pos_grid<C::TW, C::TH>(geo, &tile);
    const int x = tp.x0 + (t % C::TW);
    const int y = tp.y0 + (t / C::TW);
    const bool active = x < geo.w && y < geo.h;
    const size_t p = (size_t)(tp.pix0 + (long long)(t / C::TW) * geo.w + (t % C::TW));
    const uint32_t salt = image_salt(tp.img);

    if (t == 0) s_count = 0;

    float f[PD];
#pragma unroll
    for (int i = 0; i < PD; ++i) f[i] = active ? __ldg(feat + p * PD + i) : 0.0f;
    int g[K], rank[K], ir[K];
    float bary[K];
    static_assert(2 * K * P <= SC, "embed scratch must fit in the tile table");
    embed<PD>(f, ec, g, rank, bary, stab + t, ir);
    // the tile table: entries t + j*P are this thread's own scratch column
    for (int i = t; i < SC; i += P) stab[i] = -1;

    // 2a. candidate key records (visible to other lanes' CAS winners after the
    // barrier).  Corner 0 is the remainder-0 point g; corner c is corner c-1
    // plus one on every coordinate and minus K on the coordinate of rank
    // PD-c+1 (the corners of permutohedral.cu:238-244), so its words and the
    // linear part of its hash are updated, not rebuilt.  A point within 2K of
    // the int16 limits may wrap a coordinate: its keys are built from scratch.
    bool near_edge = false;
#pragma unroll
    for (int i = 0; i < PD; ++i) near_edge = near_edge || g[i] > 32767 - 2 * K || g[i] < -32768 + 2 * K;
    uint32_t kw[NW];
    uint32_t lin = salt;
#pragma unroll
    for (int k = 0; k < NW; ++k) kw[k] = 0u;
#pragma unroll
    for (int i = 0; i < PD; ++i) {
        kw[1 + i / 2] |= ((uint32_t)(uint16_t)(int16_t)g[i]) << (16 * (i & 1));
        lin += (uint32_t)g[i] * coord_mul(i);
    }
#pragma unroll
    for (int c = 0; c < K; ++c) {
        if (near_edge) {
            make_key<PD>(g, rank, c, salt, kw);
        } else {
            if (c > 0) {
                const int j = ir[PD + 1 - c];
#pragma unroll
                for (int k = 1; k <= 1 + (PD - 1) / 2; ++k) {   // the words that hold coordinates
                    const int lo = 2 * (k - 1), hi = lo + 1;
                    const int dlo = 1 - (j == lo ? K : 0);
                    const int dhi = hi < PD ? 1 - (j == hi ? K : 0) : 0;
                    kw[k] = hw_add(kw[k], pack_hw(dlo, dhi));
                }
                // (coordinate PD is implied by the others and not part of the key)
                lin += coord_mul_sum(PD) - (j < PD ? (uint32_t)K * c_coord_mul[j] : 0u);
            }
            kw[0] = hash_of_lin(lin);
        }
        if (active) {
#pragma unroll
            for (int w = 0; w < CW; ++w)
                ukeys[(t * K + c) * CW + w] = make_uint4(kw[4 * w], kw[4 * w + 1], kw[4 * w + 2], kw[4 * w + 3]);
        }
    }
    __syncthreads();   // table initialised, records written

    // 2b. one CAS per distinct key of the warp; the cell stores the owning candidate
    const unsigned amask = __ballot_sync(kFull, active);
    int mine[K];
    unsigned hgrp[K];   // lanes with my key (valid where bit c of huse is set)
    unsigned huse = 0u;  // warp-uniform: bit c set when no lane met a hash collision at corner c
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const int cand = t * K + c;
        uint32_t kw[NW];   // my record, read back (an inactive lane's is never used)
#pragma unroll
        for (int w = 0; w < CW; ++w) {
            const uint4 r = ukeys[cand * CW + w];
            kw[4 * w] = r.x; kw[4 * w + 1] = r.y; kw[4 * w + 2] = r.z; kw[4 * w + 3] = r.w;
        }
        const unsigned grp = __match_any_sync(kFull, kw[0]) & amask;
        const int leader = active ? __ffs(grp) - 1 : lane;
        bool same = true;
#pragma unroll
        for (int k = 1; k < NW; ++k) same = (__shfl_sync(kFull, kw[k], leader) == kw[k]) && same;
        int res = cand;
        if (active && (lane == leader || !same)) {
            uint32_t pos = (kw[0] >> 7) & (SC - 1);
            int probe = 0;
            for (; probe < SC; ++probe) {
                const int cur = atomicCAS(&stab[pos], -1, cand);
                if (cur == -1) break;
                const uint4* rec = ukeys + cur * CW;
                bool eq = true;
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const uint4 r = rec[w];
                    eq = eq && r.x == kw[4 * w] && r.y == kw[4 * w + 1] && r.z == kw[4 * w + 2] && r.w == kw[4 * w + 3];
                }
                if (eq) {
                    res = cur;
                    break;
                }
                pos = (pos + 1) & (SC - 1);
            }
            if (probe == SC) atomicOr(&L.hdr->status, PL_ST_SMEM_PROBE);   // unreachable: table is 2x the slots
        }
        const int lres = __shfl_sync(kFull, res, leader);
        mine[c] = (active && same) ? lres : res;
        hgrp[c] = grp;
        if (__ballot_sync(kFull, active && !same) == 0u) huse |= 1u << c;
    }
    __syncthreads();

    // 3. compact local ids for owners, staging, slot records, value rows
    {   // one shared atomic per warp for all its owners
        unsigned om[K];
        int n = 0;
#pragma unroll
        for (int c = 0; c < K; ++c) {
            om[c] = __ballot_sync(kFull, active && mine[c] == t * K + c);
            n += __popc(om[c]);
        }
        int wb = 0;
        if (lane == 0 && n) wb = atomicAdd(&s_count, n);
        wb = __shfl_sync(kFull, wb, 0);
        const unsigned lt = (1u << lane) - 1u;
#pragma unroll
        for (int c = 0; c < K; ++c) {
            if ((om[c] >> lane) & 1u) cand_lid[t * K + c] = (int16_t)(wb + __popc(om[c] & lt));
            wb += __popc(om[c]);
        }
    }
    __syncthreads();
    const int U = s_count;
    // the tile hash table is dead from here on: reuse it for the counting sort
    int* cnt = stab;                                                     // [U + 1]
    uint16_t* ord = reinterpret_cast<uint16_t*>(stab + ((SLOTS + 4) & ~3));   // [SLOTS], 16-byte aligned
    for (int i = t; i <= U; i += P) cnt[i] = 0;
    if (t == 0) {
        const int b = atomicAdd(&L.hdr->u_total, U);
        s_base = b;
        L.tile_off[tile] = b;
        L.tile_cnt[tile] = U;
    }
    __syncthreads();
    const int base = s_base;
    const size_t so = (size_t)tile * K * P + t;
    int lid[K];
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const int l = active ? cand_lid[mine[c]] : 0;
        lid[c] = l;
        if (active && mine[c] == t * K + c) {
#pragma unroll
            for (int w = 0; w < CW; ++w)
                S.skeys[(size_t)(base + l) * CW + w] = ukeys[(t * K + c) * CW + w];
        }
        L.slot_lid[so + (size_t)c * P] = (uint16_t)l;
        L.slot_w[so + (size_t)c * P] = active ? bary[c] : 0.0f;
    }

    // 4. counting sort of the tile's slots by local id (integer shared
    // atomics, one per distinct id of the warp), for the splat kernels
    int rk[K];
#pragma unroll
    for (int c = 0; c < K; ++c) {
        // the branch is warp-uniform: every lane calls the match or none does
        const unsigned grp = ((huse >> c) & 1u) ? hgrp[c]
                                                : __match_any_sync(kFull, active ? lid[c] : (1 << 20) + lane);
        const int leader = active ? __ffs(grp) - 1 : lane;
        int b = 0;
        if (active && lane == leader) b = atomicAdd(&cnt[lid[c]], __popc(grp));
        b = __shfl_sync(kFull, b, leader);
        rk[c] = b + __popc(grp & ((1u << lane) - 1u));
    }
    __syncthreads();
    warp0_scan_excl(cnt, U);   // cnt[u] = first sorted position of id u, cnt[U] = total
    __syncthreads();
    float* wsort = reinterpret_cast<float*>(ukeys);      // key records are staged: reuse their space
    int16_t* slid = cand_lid;                             // dead since the local ids were read
    if (active) {
#pragma unroll
        for (int c = 0; c < K; ++c) {
            const int pos = cnt[lid[c]] + rk[c];
            ord[pos] = (uint16_t)((t << 1) | (rk[c] == 0 ? 1 : 0));   // pixel, run start
            wsort[pos] = bary[c];
            slid[pos] = (int16_t)lid[c];
        }
    }
    __syncthreads();
    const int total = cnt[U];
    if (t * K < total) L.first_lid[(size_t)tile * P + t] = (uint16_t)slid[t * K];
    uint16_t* gord = L.slot_order + (size_t)tile * SLOTS;
    float* gws = L.slot_wsort + (size_t)tile * SLOTS;
    // 16-byte copies; the tile's regions are 16-byte aligned and a multiple of
    // 16 bytes long, so the tail copies stay inside them
    for (int i = t; 16 * i < 2 * total; i += P)
        reinterpret_cast<uint4*>(gord)[i] = reinterpret_cast<const uint4*>(ord)[i];
    for (int i = t; 16 * i < 4 * total; i += P)
        reinterpret_cast<float4*>(gws)[i] = reinterpret_cast<const float4*>(wsort)[i];
    zero_rows_block<P>(zero_f + (size_t)base * cpf, U * cpf, cpf % 4 == 0);
    if (zero_b) zero_rows_block<P>(zero_b + (size_t)base * cpb, U * cpb, cpb % 4 == 0);
}

// ---------------------------------------------------------------- K_clear

// Chooses the table capacity from the staged count (load <= 1/2) and zeroes
// the cells in use (cell format: TableFmt).
static __global__ void k_clear(Geo geo, LatView L, ScrView S) {
    const int U = L.hdr->u_total;
    int lg = 6;
    while ((1ll << lg) < 2ll * U) ++lg;
    if (lg > geo.cap_max_log2) lg = geo.cap_max_log2;
    if (geo.cap_override_log2 > 0)
        lg = geo.cap_override_log2 < geo.cap_max_log2 ? geo.cap_override_log2 : geo.cap_max_log2;
    if (blockIdx.x == 0 && threadIdx.x == 0) L.hdr->cap_log2 = lg;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t n4 = ((size_t)1 << lg) / 4;
    uint4* t4 = reinterpret_cast<uint4*>(S.table);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) t4[i] = z;
    if (lg >= geo.filter_min_log2) {   // the miss filter: one byte per cell
        uint4* f4 = reinterpret_cast<uint4*>(S.filter);
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4 / 4; i += stride) f4[i] = z;
    }
}

// ---------------------------------------------------------------- global table

template <int CW>
__device__ __forceinline__ void load_key(const uint4* rec, uint32_t (&kw)[4 * CW]) {
#pragma unroll
    for (int w = 0; w < CW; ++w) {
        const uint4 r = __ldg(rec + w);
        kw[4 * w] = r.x; kw[4 * w + 1] = r.y; kw[4 * w + 2] = r.z; kw[4 * w + 3] = r.w;
    }
}

// 16-byte key compares against a staged record (word 0 is the hash: compared too)
template <int CW>
__device__ __forceinline__ bool key_equal(const uint4* rec, const uint32_t (&kw)[4 * CW]) {
    bool eq = true;
#pragma unroll
    for (int w = 0; w < CW; ++w) {
        const uint4 r = __ldg(rec + w);
        eq = eq && r.x == kw[4 * w] && r.y == kw[4 * w + 1] && r.z == kw[4 * w + 2] && r.w == kw[4 * w + 3];
    }
    return eq;
}

// Cell format of the global table.  A cell is 0 (empty) or holds, in its low
// idx_bits, 1 + the staged index of the key that owns it, and above them the
// same bits of that key's hash (a tag): a probe passes over the cells of
// other keys on a tag mismatch without reading their records, so a lookup of
// an absent key usually costs the cells it walks and nothing else.  idx_bits
// is the width of the call's largest staged index + 1; the tag is what is left
// of the 32 bits (possibly nothing, which only costs key compares).
struct TableFmt {
    uint32_t idx_mask;
};

__device__ __forceinline__ TableFmt table_fmt(const Geo& g) {
    TableFmt f;
    f.idx_mask = g.idx_bits >= 32 ? 0xFFFFFFFFu : ((1u << g.idx_bits) - 1u);
    return f;
}

__device__ __forceinline__ uint32_t cell_tag(uint32_t hash, TableFmt f) { return hash & ~f.idx_mask; }

// Miss filter of a large table: a bit array of 8 bits per cell, one bit per
// vertex key, chosen by the key's home cell (the low bits of its hash) and the
// top three hash bits.  A clear bit proves a key absent without touching the
// table, whose cells are random HBM reads once it outgrows L2, while the
// filter (a quarter of the table's size) stays in L2.  With one bit per key
// and 8 bits per cell at a load of at most one key per two cells, at most
// 1 - e^(-1/16) (6%) of absent keys still reach the table; a present key
// always does (no false negatives: its owner set the bit before lookups run).
__device__ __forceinline__ uint32_t filter_word(uint32_t hash, uint32_t mask) { return (hash & mask) >> 2; }
__device__ __forceinline__ uint32_t filter_bit(uint32_t hash) { return 1u << (((hash & 3u) << 3) | (hash >> 29)); }

// The key of the blur neighbour of `key` along axis c, direction sgn (+1/-1),
// with int16 wrap-around per coordinate; word 0 receives `hash`.
template <int PD>
__device__ __forceinline__ void neighbour_key(const uint32_t (&key)[Cfg<PD>::NW], int c, int sgn, uint32_t hash,
                                              uint32_t (&kw)[Cfg<PD>::NW]) {
    constexpr int K = PD + 1, NW = Cfg<PD>::NW;
#pragma unroll
    for (int k = 0; k < NW; ++k) kw[k] = key[k];   // padding words stay as they are (0)
#pragma unroll
    for (int k = 1; k <= 1 + (PD - 1) / 2; ++k) {  // the words that hold coordinates
        const int lo = 2 * (k - 1), hi = lo + 1;
        const int dlo = lo < PD ? 1 - (c == lo ? K : 0) : 0;
        const int dhi = hi < PD ? 1 - (c == hi ? K : 0) : 0;
        kw[k] = hw_add(key[k], pack_hw(sgn * dlo, sgn * dhi));
    }
    kw[0] = hash;
}

// Continue a probe for the neighbour (c, sgn) of `key`, whose hash is h and
// whose cell at pos has been read as `cell`: the vertex id of the neighbour,
// or -1 when it is not a lattice vertex.  Its key words are formed only when a
// cell's tag matches.  Read-only use, after the table is complete.
template <int PD>
__device__ __forceinline__ int neighbour_find(const uint32_t* __restrict__ table, uint32_t mask, TableFmt f,
                                              const uint4* __restrict__ skeys, const int* __restrict__ vid_of,
                                              const uint32_t (&key)[Cfg<PD>::NW], int c, int sgn, uint32_t h,
                                              uint32_t pos, uint32_t cell, int* status) {
    constexpr int CW = Cfg<PD>::CW, NW = Cfg<PD>::NW;
    const uint32_t tag = cell_tag(h, f);
    for (uint32_t probe = 0; probe <= mask; ++probe) {
        if (cell == 0u) return -1;
        if ((cell & ~f.idx_mask) == tag) {
            const int o = (int)(cell & f.idx_mask) - 1;
            uint32_t kw[NW];
            neighbour_key<PD>(key, c, sgn, h, kw);
            if (key_equal<CW>(skeys + (size_t)o * CW, kw)) return __ldg(vid_of + o);
        }
        pos = (pos + 1) & mask;
        cell = __ldg(table + pos);
    }
    atomicOr(status, PL_ST_TABLE_FULL);
    return -1;
}

// ---------------------------------------------------------------- K2: global insert

// KPT staged keys per thread and chunk.  The staged key records are complete
// before this kernel starts, so a cell can name its owner the moment the
// owner's CAS lands: a CAS of (tag | 1 + my staged index) into an empty cell
// makes me the owner; a full cell with my tag names an owner whose record is
// compared word by word.  No cell is ever half-written and nobody waits.  The
// first CAS of each of a thread's keys is issued before any result is used
// (most keys settle there); collisions continue probing one key at a time.
// The owners of each CTA's chunk then take consecutive vertex ids (one atomic
// per CTA and chunk) and write their key to the vertex key array; cells keep
// the staged index, and lookups map it to the vertex id through vid_of.
constexpr int kInsertKpt = 4;

//
// The launch is oversubscribed (more CTAs than are co-resident).  When the
// co-resident CTAs (`resident`) can hold every key with two per thread, only
// they work, each key in flight at once (one wave); otherwise every CTA takes
// chunks of one key per thread, or of KPT keys per thread when the keys
// outnumber the grid's threads KPT to one (many short-lived CTAs, so that a
// CTA waiting on a long probe leaves its SM to others).
template <int PD>
__global__ void __launch_bounds__(256) k_insert(Geo geo, LatView L, ScrView S, int resident) {
    constexpr int CW = Cfg<PD>::CW, NW = Cfg<PD>::NW, KPT = kInsertKpt;
    __shared__ int s_wcnt[8], s_base;
    const int U = L.hdr->u_total;
    const uint32_t mask = (1u << L.hdr->cap_log2) - 1u;
    const bool use_filter = L.hdr->cap_log2 >= geo.filter_min_log2;
    const TableFmt f = table_fmt(geo);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int res = resident < (int)gridDim.x ? resident : (int)gridDim.x;
    const bool one_wave = U <= 2 * res * (int)blockDim.x;
    const int ctas = one_wave ? res : (int)gridDim.x;
    if ((int)blockIdx.x >= ctas) return;
    const int kpt = one_wave ? (U > res * (int)blockDim.x ? 2 : 1)
                             : (U >= (int)gridDim.x * (int)blockDim.x * KPT ? KPT : 1);
    const int chunk = blockDim.x * kpt;
    for (int i0 = blockIdx.x * chunk; i0 < U; i0 += ctas * chunk) {   // block-uniform
        uint32_t h[KPT], c0[KPT];
        int owner[KPT];
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = i0 + threadIdx.x + j * blockDim.x;
            owner[j] = -1;
            c0[j] = 0u;
            h[j] = 0u;
            if (j < kpt && i < U) {
                h[j] = __ldg(reinterpret_cast<const uint32_t*>(S.skeys + (size_t)i * CW));   // word 0: the hash
                c0[j] = atomicCAS(S.table + (h[j] & mask), 0u, cell_tag(h[j], f) | (uint32_t)(i + 1));
            }
        }
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = i0 + threadIdx.x + j * blockDim.x;
            if (j >= kpt || i >= U) continue;
            if (c0[j] == 0u) {
                owner[j] = i;
            } else {
                uint32_t kw[NW];
                load_key<CW>(S.skeys + (size_t)i * CW, kw);
                const uint32_t tag = cell_tag(h[j], f);
                uint32_t pos = h[j] & mask;
                uint32_t c = c0[j];
                for (uint32_t probe = 0; probe <= mask; ++probe) {
                    if (probe > 0) {
                        c = atomicCAS(S.table + pos, 0u, tag | (uint32_t)(i + 1));
                        if (c == 0u) {
                            owner[j] = i;
                            break;
                        }
                    }
                    if ((c & ~f.idx_mask) == tag) {
                        const int o = (int)(c & f.idx_mask) - 1;
                        if (key_equal<CW>(S.skeys + (size_t)o * CW, kw)) {
                            owner[j] = o;
                            break;
                        }
                    }
                    pos = (pos + 1) & mask;
                }
                if (owner[j] < 0) atomicOr(&L.hdr->status, PL_ST_TABLE_FULL);
            }
            if (owner[j] == i && use_filter) atomicOr(S.filter + filter_word(h[j], mask), filter_bit(h[j]));
            S.owner[i] = owner[j];
        }
        unsigned m[KPT];
        int wtot = 0;
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = i0 + threadIdx.x + j * blockDim.x;
            m[j] = __ballot_sync(kFull, j < kpt && i < U && owner[j] == i);
            wtot += __popc(m[j]);
        }
        if (lane == 0) s_wcnt[wid] = wtot;
        __syncthreads();
        if (threadIdx.x == 0) {
            int tot = 0;
            for (int k = 0; k < 8; ++k) {
                const int c = s_wcnt[k];
                s_wcnt[k] = tot;
                tot += c;
            }
            s_base = tot ? atomicAdd(&L.hdr->m, tot) : 0;
        }
        __syncthreads();
        int vbase = s_base + s_wcnt[wid];
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            if ((m[j] >> lane) & 1u) {
                const int i = i0 + threadIdx.x + j * blockDim.x;
                const int vid = vbase + __popc(m[j] & ((1u << lane) - 1u));
                S.vid_of[i] = vid;
#pragma unroll
                for (int w = 0; w < CW; ++w) S.vkeys[(size_t)vid * CW + w] = __ldg(S.skeys + (size_t)i * CW + w);
            }
            vbase += __popc(m[j]);
        }
        __syncthreads();   // s_wcnt / s_base reused by the next chunk
    }
}

// The two blur neighbours of vertex v (key words `key`, linear part `lin`)
// along axis c: for axis c < PD the step is every coordinate +1 (or -1) and
// coordinate c -K (or +K), for c == PD every coordinate +1 (or -1)
// (permutohedral.cu:368-375).  Both cells are read, then probed and compared;
// the pair is stored streamed (evict-first).  A key within K of the int16
// limits may wrap a coordinate (`edge`), so its neighbours' linear parts are
// recomputed from their words.
template <int PD>
__device__ __forceinline__ void neighbour_pair(const ScrView& S, const LatView& L, uint32_t mask, TableFmt f,
                                               bool use_filter, const uint32_t (&key)[Cfg<PD>::NW], uint32_t lin,
                                               bool edge, int v, int M, int c, bool try_a = true,
                                               bool try_b = true) {
    constexpr int NW = Cfg<PD>::NW;
    uint32_t hp, hm;
    if (!edge) {
        const uint32_t d = axis_lin_step<PD>(c);
        hp = hash_of_lin(lin + d);
        hm = hash_of_lin(lin - d);
    } else {   // linear parts from the words, plus the vertex's image salt
        const uint32_t salt = lin - key_lin_words<PD>(key);
        uint32_t kw[NW];
        neighbour_key<PD>(key, c, 1, 0u, kw);
        hp = hash_of_lin(key_lin_words<PD>(kw) + salt);
        neighbour_key<PD>(key, c, -1, 0u, kw);
        hm = hash_of_lin(key_lin_words<PD>(kw) + salt);
    }
    const uint32_t pa = hp & mask, pb = hm & mask;
    // a cell reads as empty when the key is already known to be absent or the filter rules it out
    bool ina = try_a, inb = try_b;
    if (use_filter) {
        ina = ina && (__ldg(S.filter + filter_word(hp, mask)) & filter_bit(hp)) != 0u;
        inb = inb && (__ldg(S.filter + filter_word(hm, mask)) & filter_bit(hm)) != 0u;
    }
    const uint32_t ca = ina ? __ldg(S.table + pa) : 0u, cb = inb ? __ldg(S.table + pb) : 0u;
    const int na = neighbour_find<PD>(S.table, mask, f, S.skeys, S.vid_of, key, c, 1, hp, pa, ca, &L.hdr->status);
    const int nb = neighbour_find<PD>(S.table, mask, f, S.skeys, S.vid_of, key, c, -1, hm, pb, cb, &L.hdr->status);
    __stcs(L.nbr + (size_t)c * M + v, make_int2(na, nb));
}

template <int PD>
__device__ __forceinline__ void load_vertex_key(const ScrView& S, int v, uint32_t (&key)[Cfg<PD>::NW], uint32_t& lin,
                                                bool& edge) {
    constexpr int K = PD + 1, CW = Cfg<PD>::CW;
#pragma unroll
    for (int w = 0; w < CW; ++w) {   // streamed (evict-first): the table stays in L2
        const uint4 r = __ldcs(S.vkeys + (size_t)v * CW + w);
        key[4 * w] = r.x; key[4 * w + 1] = r.y; key[4 * w + 2] = r.z; key[4 * w + 3] = r.w;
    }
    lin = lin_of_hash(key[0]);   // linear part plus the image's salt
    edge = false;
#pragma unroll
    for (int i = 0; i < PD; ++i) {
        const int x = key_coord(key, i);
        edge = edge || x > 32767 - K || x < -32768 + K;
    }
}

constexpr int kNbrThreads = 256;

// Blur neighbours of every vertex.  The vertex keys and the neighbour pairs
// are streamed with evict-first hints, so that the hash table, which every
// lookup probes at random, stays resident in L2.
//
// Dense lattices (no miss filter: tables below 2^22 cells): a thread takes one
// vertex and a group of axes (all of them when there are enough vertices to
// occupy the grid), loads the vertex key once and issues the two lookups of an
// axis together.
//
// Sparse lattices (large tables, most neighbours absent): a thread takes one
// vertex and settles, in a first sweep, every axis whose two lookups the
// filter or an empty home cell rule out, with a few instructions each.  The
// remaining (vertex, axis) pairs of the warp go to a queue in shared memory
// (with the vertices' keys) and the warp's lanes take them one each, so that
// the full probe and key compare run with every lane busy.
// Per-warp shared memory of the sparse path's queue.
template <int PD>
struct NbrWarpSmem {
    uint32_t key[Cfg<PD>::NW][32];
    uint32_t lin[32];
    unsigned long long side[32];   // bits 2c, 2c+1: the + / - lookup of axis c may hit
    uint16_t q[32 * (PD + 1)];     // (lane << 5) | axis
};

// The neighbour lookups of all vertices by the threads gtid = 0..nthreads-1
// of a grid (whole warps); `wsm` is this warp's queue memory.
template <int PD>
__device__ __forceinline__ void neighbors_grid(const Geo& geo, const LatView& L, const ScrView& S, int gtid,
                                               int nthreads, NbrWarpSmem<PD>* wsm) {
    constexpr int K = PD + 1, NW = Cfg<PD>::NW;
    const int M = L.hdr->m;
    if (M <= 0) return;
    const uint32_t mask = (1u << L.hdr->cap_log2) - 1u;
    const bool use_filter = L.hdr->cap_log2 >= geo.filter_min_log2;
    const TableFmt f = table_fmt(geo);
    int G = (nthreads + M - 1) / M;   // axis groups
    G = G < 1 ? 1 : (G > K ? K : G);
    if (!(use_filter && G == 1)) {   // dense (uniform over the grid)
        const size_t total = (size_t)M * G;
        for (size_t idx = gtid; idx < total; idx += nthreads) {
            const int g = (int)(idx / M);
            const int v = (int)(idx - (size_t)g * M);
            uint32_t key[NW], lin;
            bool edge;
            load_vertex_key<PD>(S, v, key, lin, edge);
            for (int c = g; c < K; c += G) neighbour_pair<PD>(S, L, mask, f, use_filter, key, lin, edge, v, M, c);
        }
        return;
    }
    const int lane = gtid & 31;
    for (int wb = gtid - lane; wb < M; wb += nthreads) {   // warp-uniform
        const int v = wb + lane;
        uint32_t pend = 0u;   // my axes still to look up, one bit each
        unsigned long long side = ~0ull;
        if (v < M) {
            uint32_t key[NW], lin;
            bool edge;
            load_vertex_key<PD>(S, v, key, lin, edge);
            if (edge) {
                pend = (1u << K) - 1u;   // (the queue below recomputes edge hashes from the words)
            } else {
                side = 0ull;
#pragma unroll 4
                for (int c = 0; c < K; ++c) {
                    const uint32_t d = axis_lin_step<PD>(c);
                    const uint32_t hp = hash_of_lin(lin + d), hm = hash_of_lin(lin - d);
                    const bool ina = (__ldg(S.filter + filter_word(hp, mask)) & filter_bit(hp)) != 0u;
                    const bool inb = (__ldg(S.filter + filter_word(hm, mask)) & filter_bit(hm)) != 0u;
                    const uint32_t ca = ina ? __ldg(S.table + (hp & mask)) : 0u;
                    const uint32_t cb = inb ? __ldg(S.table + (hm & mask)) : 0u;
                    if ((ca | cb) != 0u) {
                        pend |= 1u << c;
                        side |= (unsigned long long)((ca != 0u ? 1u : 0u) | (cb != 0u ? 2u : 0u)) << (2 * c);
                    } else {
                        __stcs(L.nbr + (size_t)c * M + v, make_int2(-1, -1));
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < NW; ++k) wsm->key[k][lane] = key[k];
            wsm->lin[lane] = lin;
            wsm->side[lane] = side;
        }
        // my queue entries after those of the lanes below me
        const int cnt = __popc(pend);
        int pre = cnt;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(kFull, pre, d);
            if (lane >= d) pre += o;
        }
        const int qtotal = __shfl_sync(kFull, pre, 31);
        pre -= cnt;
        for (uint32_t m = pend; m != 0u; m &= m - 1u) wsm->q[pre++] = (uint16_t)((lane << 5) | (__ffs(m) - 1));
        __syncwarp();
        for (int j = lane; j < qtotal; j += 32) {
            const int e = wsm->q[j];
            const int src = e >> 5, c = e & 31;
            uint32_t key[NW];
#pragma unroll
            for (int k = 0; k < NW; ++k) key[k] = wsm->key[k][src];
            bool edge = false;
#pragma unroll
            for (int i = 0; i < PD; ++i) {
                const int x = key_coord(key, i);
                edge = edge || x > 32767 - K || x < -32768 + K;
            }
            // a lookup the first sweep ruled out (filter bit clear or home cell
            // empty) reads nothing; the other reads its home cell again
            const unsigned sd = (unsigned)(wsm->side[src] >> (2 * c)) & 3u;
            neighbour_pair<PD>(S, L, mask, f, false, key, wsm->lin[src], edge, wb + src, M, c, (sd & 1u) != 0u,
                               (sd & 2u) != 0u);
        }
        __syncwarp();   // the queue is refilled by the next step
    }
}

template <int PD>
__global__ void __launch_bounds__(kNbrThreads, PD <= 6 ? 8 : 4) k_neighbors(Geo geo, LatView L, ScrView S) {
    __shared__ NbrWarpSmem<PD> wsm[kNbrThreads / 32];
    neighbors_grid<PD>(geo, L, S, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x,
                       &wsm[threadIdx.x >> 5]);
}

// ---------------------------------------------------------------- grid barrier

// Grid barrier over the CTAs of a cooperative launch (all co-resident): one
// acquire-release add per CTA on a counter that only grows during the launch
// (it is zero when the launch starts), then acquire polls until all CTAs of
// this phase have arrived.  The CTA whose add completes the phase learns it
// from the add's result and does not poll (one L2 round trip less on the
// barrier's critical path).  The wait is bounded: a CTA that polls
// kBarrierSpin times records PL_ST_SPIN and continues, so a failure shows in
// the status word instead of a hang.
constexpr int kBarrierSpin = 1 << 22;

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// (`counter`: the lattice's bar_count unless the kernel has its own)
__device__ __forceinline__ void grid_barrier(LatticeHeader* hdr, unsigned& phase, unsigned* counter = nullptr) {
    __syncthreads();
    ++phase;
    if (threadIdx.x == 0) {
        unsigned* const cnt = counter ? counter : &hdr->bar_count;
        const unsigned target = phase * gridDim.x;
        const unsigned arrived = atom_add_acq_rel(cnt, 1u) + 1u;
        int spins = 0;
        while (arrived < target && ld_acquire(cnt) < target) {
            if (++spins > kBarrierSpin) {
                atomicOr(&hdr->status, PL_ST_SPIN);
                break;
            }
            if (spins > 4096) __nanosleep(32);
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------- splat

// FWD: [v*w, w] per slot (permutohedral.cu:286-293); otherwise
// (grad * weight_in) * w (permutohedral.cu:437-445).
//
// The tile's slots were counting-sorted by local vertex when the lattice was
// built: every local vertex owns a contiguous run of the sorted order, runs
// are in local-id order, and each sorted entry carries its pixel and a
// run-start flag.  Thread t sums the K sorted positions [t*K, t*K + K),
// starting from the local id recorded for position t*K and stepping to the
// next id at every run start, and adds each piece of a run that falls in its
// positions to the lattice with one vector red.global.add; the pieces of a
// run that crosses lanes are first merged by a segmented warp scan, so that
// about one red per run and warp remains.  Balanced work per thread, no
// search; no shared-memory float atomics.
template <int CP, int NC>
__device__ __forceinline__ void red_run(float* lat, int vid, const float (&s)[NC]) {
    float r[CP];
#pragma unroll
    for (int j = 0; j < CP; ++j) r[j] = j < NC ? s[j] : 0.0f;
    red_add_row<CP>(lat + (size_t)vid * CP, r);
}

// Shared memory of one tile worker of the splat: the tile's vertex ids and
// the per-pixel value rows.
template <int PD, int NC>
struct SplatSmem {
    int svid[Cfg<PD>::SLOTS];
    float4 pv[Cfg<PD>::P * ((NC + 3) / 4)];
};

// Synchronisation of the P threads that work on one tile: the whole CTA
// (one tile per CTA) or a named barrier of a tile worker inside a larger CTA.
struct CtaSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
struct WorkerSync {
    int id, n;   // barrier id (1..15) and thread count
    __device__ __forceinline__ void operator()() const {
        asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
    }
};

template <int PD, int V, bool FWD, typename Sync>
__device__ __forceinline__ void splat_tile(int tile, const TilePos& tp, int t, const float* __restrict__ vals,
                                           const float* __restrict__ wt, const Geo& geo, const LatView& L,
                                           const ScrView& S, int resolve, float* lat,
                                           SplatSmem<PD, FWD ? V + 1 : V>& sm, Sync sync) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P, SLOTS = C::SLOTS;
    constexpr int CP = FWD ? pad_ch(V + 1) : pad_ch(V);
    constexpr int NC = FWD ? V + 1 : V;
    constexpr int NV4 = (NC + 3) / 4;            // float4 per pixel value row
    int* svid = sm.svid;
    float4* pv = sm.pv;
    const int x0 = tp.x0, y0 = tp.y0;
    const int nx = min(C::TW, geo.w - x0), ny = min(C::TH, geo.h - y0);
    const int total = nx * ny * K;
    // my K sorted positions: entries and weights straight into registers
    const int q0 = t * K;
    const int nq = max(0, min(K, total - q0));
    int code[K];
    float wq[K];
    {
        const uint16_t* go = L.slot_order + (size_t)tile * SLOTS + q0;
        const float* gw = L.slot_wsort + (size_t)tile * SLOTS + q0;
        if constexpr (K % 2 == 0) {
            // K even: the K entries are K/2 aligned 32-bit words, the weights K/2 float2
#pragma unroll
            for (int k = 0; k < K; k += 2) {
                uint32_t two = 0u;
                float2 ww = make_float2(0.0f, 0.0f);
                if (k < nq) {
                    two = __ldg(reinterpret_cast<const uint32_t*>(go + k));
                    ww = __ldg(reinterpret_cast<const float2*>(gw + k));
                }
                code[k] = (int)(two & 0xffffu);
                code[k + 1] = (int)(two >> 16);
                wq[k] = ww.x;
                wq[k + 1] = ww.y;
            }
        } else {
#pragma unroll
            for (int k = 0; k < K; ++k) {
                code[k] = k < nq ? (int)__ldg(go + k) : 0;
                wq[k] = k < nq ? __ldg(gw + k) : 0.0f;
            }
        }
    }
    const int first = nq > 0 ? (int)L.first_lid[(size_t)tile * P + t] : 0;
    {   // this pixel's values
        const int x = x0 + (t % C::TW), y = y0 + (t / C::TW);
        const bool active = x < geo.w && y < geo.h;
        const size_t p = (size_t)(tp.pix0 + (long long)(t / C::TW) * geo.w + (t % C::TW));
        float wp = 1.0f;
        if constexpr (!FWD) wp = active ? __ldg(wt + p) : 0.0f;
        float r[4 * NV4];
#pragma unroll
        for (int j = 0; j < 4 * NV4; ++j) r[j] = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const float v = active ? __ldg(vals + p * V + j) : 0.0f;
            r[j] = FWD ? v : __fmul_rn(v, wp);
        }
        if constexpr (FWD) r[V] = 1.0f;
#pragma unroll
        for (int k = 0; k < NV4; ++k) pv[t * NV4 + k] = make_float4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
    }
    // vertex ids of the tile's local vertices; the call right after a build
    // resolves them through the owners and stores them for the kernels that
    // follow
    const int cnt = L.tile_cnt[tile], off = L.tile_off[tile];
    for (int u = t; u < cnt; u += P) {
        int vid;
        if (resolve) {
            const int o = S.owner[off + u];
            vid = o >= 0 ? S.vid_of[o] : -1;
            L.staged_vid[off + u] = vid;
        } else {
            vid = L.staged_vid[off + u];
        }
        svid[u] = vid;
    }
    sync();
    // my pieces: the first (it may continue the previous lane's run), complete
    // runs in between (added at once), and the last (it may continue into the
    // next lane); the first and last are the same piece when no run starts
    // after my first position
    int l = first;
    bool multi = false;
    float cur[NC], head[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) cur[j] = head[j] = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        if (k < nq) {
            if (k > 0 && (code[k] & 1)) {   // a run starts: the piece before it is complete
                if (!multi) {
#pragma unroll
                    for (int j = 0; j < NC; ++j) head[j] = cur[j];
                    multi = true;
                } else if (svid[l] >= 0) {
                    red_run<CP, NC>(lat, svid[l], cur);
                }
                ++l;
#pragma unroll
                for (int j = 0; j < NC; ++j) cur[j] = 0.0f;
            }
            const int px = code[k] >> 1;
            const float w = wq[k];
            float r[4 * NV4];
#pragma unroll
            for (int m = 0; m < NV4; ++m) {
                const float4 a = pv[px * NV4 + m];
                r[4 * m] = a.x; r[4 * m + 1] = a.y; r[4 * m + 2] = a.z; r[4 * m + 3] = a.w;
            }
#pragma unroll
            for (int j = 0; j < NC; ++j) cur[j] = (FWD && j == V) ? __fadd_rn(cur[j], w) : __fmaf_rn(r[j], w, cur[j]);
        }
    }
    // merge the pieces of a run that crosses lanes: a segmented inclusive sum
    // of the last pieces, segments starting at every lane whose last piece
    // starts inside it or whose first position starts a run
    const int lane = t & 31;
    const bool cont = lane > 0 && nq > 0 && !(code[0] & 1);   // my first piece continues lane-1's run
    const unsigned below = 0xffffffffu >> (31 - lane);
    const unsigned heads = __ballot_sync(kFull, multi || !cont);
    const int start = 31 - __clz(heads & below);
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
        for (int j = 0; j < NC; ++j) {
            const float o = __shfl_up_sync(kFull, cur[j], d);
            if (lane - d >= start) cur[j] = __fadd_rn(cur[j], o);
        }
    }
    float prev[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) prev[j] = __shfl_up_sync(kFull, cur[j], 1);
    const bool next_cont = __shfl_down_sync(kFull, cont ? 1 : 0, 1) != 0;
    if (nq > 0) {
        if (multi) {   // my first piece closes a run: add what the lanes before me carried
            if (cont) {
#pragma unroll
                for (int j = 0; j < NC; ++j) head[j] = __fadd_rn(head[j], prev[j]);
            }
            if (svid[first] >= 0) red_run<CP, NC>(lat, svid[first], head);
        }
        if ((lane == 31 || !next_cont) && svid[l] >= 0) red_run<CP, NC>(lat, svid[l], cur);
    }
    sync();   // svid / pv are reused by the worker's next tile
}

template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_splat(const float* __restrict__ vals, const float* __restrict__ wt, Geo geo, LatView L, ScrView S,
        int resolve, float* lat) {
    __shared__ SplatSmem<PD, FWD ? V + 1 : V> sm;
    int tile;
    const TilePos tp = tile_pos_grid<Cfg<PD>::TW, Cfg<PD>::TH>(geo, &tile);
    splat_tile<PD, V, FWD>(tile, tp, threadIdx.x, vals, wt, geo, L, S, resolve, lat, sm, CtaSync{});
}

// The splat right after a lattice build, together with the blur-neighbour
// lookups of the new lattice in the same launch: the first `nbr_blocks` blocks
// look up neighbours (grid-stride over the vertices), the others splat one
// tile each and resolve the tile's vertex ids.  Blocks are dispatched in index
// order, so the latency-bound lookups start first and the bandwidth-bound
// tiles fill the SMs around them.
template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P, slice_min_blocks<PD, V>())
k_splat_nbr(const float* __restrict__ vals, const float* __restrict__ wt, Geo geo, LatView L, ScrView S, float* lat,
            int nbr_blocks) {
    __shared__ union {
        SplatSmem<PD, FWD ? V + 1 : V> sp;
        NbrWarpSmem<PD> nb[Cfg<PD>::P / 32];
    } sm;
    if ((int)blockIdx.x < nbr_blocks)
        neighbors_grid<PD>(geo, L, S, blockIdx.x * blockDim.x + threadIdx.x, nbr_blocks * blockDim.x,
                           &sm.nb[threadIdx.x >> 5]);
    else {
        const int tile = blockIdx.x - nbr_blocks;
        splat_tile<PD, V, FWD>(tile, tile_pos<Cfg<PD>::TW, Cfg<PD>::TH>(geo, tile), threadIdx.x, vals, wt, geo, L, S,
                               1, lat, sm.sp, CtaSync{});
    }
}

// The splat of a call on a kept lattice, whose value rows must start at zero:
// one cooperative launch that zeroes the first m rows (cp floats each, float4
// stores), waits at one grid barrier, then takes the tiles in turn -- in place
// of a separate zeroing kernel, whose launch costs more than its stores.  Its
// barrier counts on bar_zero, which the blur that follows leaves alone; the
// kernel after that blur (the slice), or that blur's own exit, zeroes it, so
// this kernel ends without an exit protocol.
template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_splat_zeroed(const float* __restrict__ vals, const float* __restrict__ wt, Geo geo, LatView L, float* lat,
               int cp) {
    __shared__ SplatSmem<PD, FWD ? V + 1 : V> sm;
    unsigned phase = 0;
    {
        const size_t n = (size_t)L.hdr->m * cp;
        const size_t stride = (size_t)gridDim.x * blockDim.x;
        const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        float4* b4 = reinterpret_cast<float4*>(lat);
        const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (size_t i = i0; i < n / 4; i += stride) b4[i] = z;
        for (size_t i = (n & ~(size_t)3) + i0; i < n; i += stride) lat[i] = 0.0f;
    }
    grid_barrier(L.hdr, phase, &L.hdr->bar_zero);
    for (int tile = blockIdx.x; tile < geo.tiles; tile += gridDim.x)
        splat_tile<PD, V, FWD>(tile, tile_pos<Cfg<PD>::TW, Cfg<PD>::TH>(geo, tile), threadIdx.x, vals, wt, geo, L,
                               ScrView{}, 0, lat, sm, CtaSync{});
}

// ---------------------------------------------------------------- bulk copies

// Bulk asynchronous copies global -> shared memory (cp.async.bulk, no
// multicast), completed on an mbarrier of the CTA with a transaction count.
// Addresses 16-byte aligned, sizes multiples of 16 bytes.
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of `parity` to complete: false (and the status
// bit PL_ST_SPIN recorded) when it has not completed after kMbarSpin tries.
constexpr int kMbarSpin = 1 << 20;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, LatticeHeader* hdr) {
    for (int i = 0; i < kMbarSpin; ++i)
        if (mbar_test(bar, parity)) return true;
    atomicOr(&hdr->status, PL_ST_SPIN);
    return false;
}

// ---------------------------------------------------------------- blur

// r *= 2^-e (exact: a power of two, far from the float range limits here)
template <int CP>
__device__ __forceinline__ void scale_pow2(float (&r)[CP], int e) {
    if (e == 0) return;
    const float f = __int_as_float((127 - e) << 23);
#pragma unroll
    for (int j = 0; j < CP; ++j) r[j] = __fmul_rn(r[j], f);
}

// One [1 2 1]/4 stencil step of a row along one axis; a missing neighbour
// (index -1) contributes nothing (permutohedral.cu:341-347).
template <int CP>
__device__ __forceinline__ void blur_row(const float (&me)[CP], const float (&a)[CP], const float (&b)[CP], int2 n,
                                         float (&r)[CP]) {
#pragma unroll
    for (int j = 0; j < CP; ++j) {
        float acc = __fmul_rn(2.0f, me[j]);
        if (n.x >= 0) acc = __fadd_rn(acc, a[j]);
        if (n.y >= 0) acc = __fadd_rn(acc, b[j]);
        r[j] = __fmul_rn(0.25f, acc);
    }
}

// The K blur passes, axis order 0..PD or PD..0 (reverse), from buf0 over the
// pair buf0/buf1; *final_flag (normally hdr->blur_final) is set to the buffer
// (0 or 1) that holds the result.
// One cooperative launch: grid barriers separate the steps; every read of
// data written inside this launch goes to L2 (ld.global.cg), never to a
// stale L1 line.
//
// At most R vertices per thread (R = 2 for rows of up to 2 channels, else 1): a thread keeps the same
// vertices throughout, their rows in registers, and runs the passes in pairs.
// For passes s, s+1 it evaluates pass s at its vertex v and at v's two
// neighbours along the axis of pass s+1 (each from the rows pass s reads
// there, with the float operations the owner of that neighbour uses, so the
// values are bit-identical), then pass s+1 at v: one barrier per pair.  The
// neighbour indices of a step, those two hops away included, are requested
// before the preceding barrier.  Larger lattices stream every row through one
// pass per step.
constexpr int kBlurThreads = 1024;

struct BlurIdx {
    int2 s;        // neighbours along the step's first axis
    int2 t;        // neighbours along its second axis (pairs only)
    int2 ta, tb;   // first-axis neighbours of t.x and of t.y
};

// (through L2: in the fused filter kernel the table was written in the same launch)
__device__ __forceinline__ int2 nbr_at(const int2* nbr, int M, int axis, int v) {
    return v >= 0 ? __ldcg(nbr + (size_t)axis * M + v) : make_int2(-1, -1);
}

__device__ __forceinline__ BlurIdx blur_idx(const int2* nbr, int M, int v, int ax_s, int ax_t) {
    BlurIdx I;
    I.s = nbr_at(nbr, M, ax_s, v);
    I.t = ax_t >= 0 ? nbr_at(nbr, M, ax_t, v) : make_int2(-1, -1);
    I.ta = nbr_at(nbr, M, ax_s, I.t.x);
    I.tb = nbr_at(nbr, M, ax_s, I.t.y);
    return I;
}

// pass s evaluated at vertex u (u >= 0) whose first-axis neighbours are n, on
// W channels of rows of stride CP (x points at the first of the W channels)
template <int W, int CP>
__device__ __forceinline__ void blur_at(const float* x, int u, int2 n, float (&r)[W]) {
    float me[W], a[W], b[W];
    load_row_cg<W>(x + (size_t)u * CP, me);
    if (n.x >= 0) load_row_cg<W>(x + (size_t)n.x * CP, a);
    if (n.y >= 0) load_row_cg<W>(x + (size_t)n.y * CP, b);
    blur_row<W>(me, a, b, n, r);
}

// Where a vertex's current row of a streaming blur lives, and how many
// halvings are still to be applied to it: one state byte per vertex and pass
// parity, location in bits 6-7, pending halvings (at most K) in bits 0-5.
// Locations: 0 = buf0 (float, where the splat left it), 1 = buf1 (float),
// 2 / 3 = the two bfloat16 row arrays that share buf1's memory in the
// reduced-precision mode.  A row is only ever rewritten into another location
// than the one the pass reads it from.
constexpr int kLocBuf0 = 0, kLocBuf1 = 1, kLocH0 = 2, kLocH1 = 3;

template <int CP, bool HALF>
__device__ __forceinline__ void load_loc(int loc, int v, const float* buf0, const float* buf1, const uint16_t* h0,
                                         const uint16_t* h1, float (&r)[CP]) {
    if (!HALF || loc < kLocH0) load_row_cg<CP>((loc == kLocBuf0 ? buf0 : buf1) + (size_t)v * CP, r);
    else                       load_row_bf16<CP>((loc == kLocH0 ? h0 : h1) + (size_t)v * CP, r);
}

template <int CP, bool HALF>
__device__ __forceinline__ void store_loc(int loc, int v, float* buf0, float* buf1, uint16_t* h0, uint16_t* h1,
                                          const float (&r)[CP]) {
    if (!HALF) store_row<CP>((loc == kLocBuf0 ? buf0 : buf1) + (size_t)v * CP, r);
    else       store_row_bf16<CP>((loc == kLocH0 ? h0 : h1) + (size_t)v * CP, r);
}

// Larger lattices stream every row, one pass per step.  A vertex without a
// neighbour along the pass's axis only halves (0.25 * (2 x) = x / 2, exact in
// float): its row is left where it is and the halving is recorded in its
// state byte; the rows that are read are scaled by their pending powers of
// two first, which is exact too, so the values are those of the plain
// sequence of passes.  The indices and states of VPT vertices per lane are
// requested together; the vertices of the warp's step that have neighbours go
// through a per-warp queue in shared memory, one per lane, so that the row
// work runs with every lane busy however sparse the axis is.  Each vertex
// keeps its owner thread in every pass (isolated vertices) or its warp
// (queued ones); the final gather, after a barrier, puts every row, scaled,
// into buf0 as floats.  With HALF, the rows a pass
// writes are stored as bfloat16 (half the row bytes; the arithmetic stays
// float), in two arrays of M rows laid out in buf1.  (A separate function, so
// that its registers do not weigh on the resident path.)
constexpr int kBlurVpt = 4;   // vertices per lane whose indices and states are requested together
constexpr int kBlurQueueBytes = kBlurThreads * kBlurVpt * 16;   // dynamic shared memory of k_blur_all

template <int PD, int CP, bool HALF>
__device__ __noinline__ void blur_streaming(const int2* nbr, uint8_t* bstate, LatticeHeader* hdr, float* buf0,
                                            float* buf1, int reverse, int* final_flag, int M, int tid, int stride,
                                            uint4* blur_queue, unsigned& phase) {
    constexpr int K = PD + 1;
    constexpr int VPT = kBlurVpt;
    const int lane = threadIdx.x & 31;
    uint4* const q = blur_queue + (threadIdx.x >> 5) * (32 * VPT);   // per warp: its step's vertices with neighbours
    const int wbase = tid - lane;   // the warp's first vertex of a step: the loop below is warp-uniform
    uint8_t* const st0 = bstate;
    uint8_t* const st1 = bstate + M;
    uint16_t* const h0 = reinterpret_cast<uint16_t*>(buf1);
    uint16_t* const h1 = h0 + (size_t)M * CP;
#pragma unroll 1
    for (int s = 0; s < K; ++s) {
        const int ax = reverse ? K - 1 - s : s;
        const int2* nb = nbr + (size_t)ax * M;
        const uint8_t* sc = (s & 1) ? st1 : st0;
        uint8_t* sn = (s & 1) ? st0 : st1;
        for (int w0 = wbase; w0 < M; w0 += stride * VPT) {
            int2 n[VPT];
            int cv[VPT], ca[VPT], cb[VPT];
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int v = w0 + lane + k * stride;
                n[k] = v < M ? __ldcg(nb + v) : make_int2(-1, -1);
                cv[k] = (s == 0 || v >= M) ? 0 : (int)__ldcg(sc + v);
            }
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                ca[k] = (s == 0 || n[k].x < 0) ? 0 : (int)__ldcg(sc + n[k].x);
                cb[k] = (s == 0 || n[k].y < 0) ? 0 : (int)__ldcg(sc + n[k].y);
            }
            // isolated vertices only count a halving; the others are queued, so
            // that the lanes of the warp take them one each below
            int total = 0;
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int v = w0 + lane + k * stride;
                const bool busy = n[k].x >= 0 || n[k].y >= 0;   // false beyond M
                const unsigned m = __ballot_sync(kFull, busy);
                if (busy) {
                    q[total + __popc(m & ((1u << lane) - 1u))] =
                        make_uint4((uint32_t)v, (uint32_t)n[k].x, (uint32_t)n[k].y,
                                   (uint32_t)cv[k] | ((uint32_t)ca[k] << 8) | ((uint32_t)cb[k] << 16));
                } else if (v < M) {
                    sn[v] = (uint8_t)((cv[k] & ~63) | ((cv[k] & 63) + 1));
                }
                total += __popc(m);
            }
            __syncwarp();
            for (int j = lane; j < total; j += 32) {
                const uint4 e = q[j];
                const int v = (int)e.x;
                const int2 nv = make_int2((int)e.y, (int)e.z);
                const int c0 = (int)(e.w & 255u), c1 = (int)((e.w >> 8) & 255u), c2 = (int)(e.w >> 16);
                const int lv = c0 >> 6;
                float me[CP], a[CP], b[CP], r[CP];
                load_loc<CP, HALF>(lv, v, buf0, buf1, h0, h1, me);
                if (nv.x >= 0) load_loc<CP, HALF>(c1 >> 6, nv.x, buf0, buf1, h0, h1, a);
                if (nv.y >= 0) load_loc<CP, HALF>(c2 >> 6, nv.y, buf0, buf1, h0, h1, b);
                scale_pow2<CP>(me, c0 & 63);
                if (nv.x >= 0) scale_pow2<CP>(a, c1 & 63);
                if (nv.y >= 0) scale_pow2<CP>(b, c2 & 63);
                blur_row<CP>(me, a, b, nv, r);
                const int nl = HALF ? (lv == kLocH0 ? kLocH1 : kLocH0) : (lv ^ 1);
                store_loc<CP, HALF>(nl, v, buf0, buf1, h0, h1, r);
                sn[v] = (uint8_t)(nl << 6);
            }
            __syncwarp();   // the queue is refilled by the next step
        }
        // after the last pass too: the gather below rewrites buf0 rows that
        // neighbours may still be reading in that pass
        grid_barrier(hdr, phase);
    }
    const uint8_t* sf = (K & 1) ? st1 : st0;
    for (int v = tid; v < M; v += stride) {   // my own vertices
        const int c = (int)sf[v];
        if (c == 0) continue;
        float r[CP];
        load_loc<CP, HALF>(c >> 6, v, buf0, buf1, h0, h1, r);
        scale_pow2<CP>(r, c & 63);
        store_row<CP>(buf0 + (size_t)v * CP, r);
    }
    if (tid == 0 && final_flag) *final_flag = 0;
}

constexpr int kBlurHalf = 1;     // flags of k_blur_all: bfloat16 rows in the streaming passes
constexpr int kBlurStream = 2;   // the streaming passes whatever the lattice's size (tests)

// The resident blur: every vertex's row stays in a register of one thread
// for the K passes, passes in fused pairs (one grid barrier per pair).  CTA b
// of G owns the contiguous vertices [M b / G, M (b+1) / G) (balanced over the
// SMs), R per thread.  Requires M <= G * blockDim * R.  Returns the buffer
// that holds the result.
template <int PD, int CP>
__device__ __forceinline__ float* blur_resident(const LatView& L, float* buf0, float* buf1, int reverse, int M,
                                                unsigned& phase) {
    constexpr int K = PD + 1;
    constexpr int R = CP <= 2 ? 2 : 1;        // vertices per thread kept in registers
    constexpr int W = CP < 4 ? CP : 4;         // channels per group (the stencil is per channel)
    const int G = gridDim.x;
    const int vb = (int)((long long)M * blockIdx.x / G), ve = (int)((long long)M * (blockIdx.x + 1) / G);
    float* x = buf0;
    float* y = buf1;
    auto axis = [&](int k) { return k >= K ? -1 : (reverse ? K - 1 - k : k); };
    float me[R][CP];
    BlurIdx idx[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int v = vb + threadIdx.x + r * blockDim.x;
        if (v < ve) load_row_cg<CP>(x + (size_t)v * CP, me[r]);
        idx[r] = blur_idx(L.nbr, M, v < ve ? v : -1, axis(0), axis(1));
    }
#pragma unroll 1
    for (int k = 0; k < K; k += 2) {
        const bool pair = k + 1 < K;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int v = vb + threadIdx.x + r * blockDim.x;
            if (v >= ve) continue;
            const BlurIdx& I = idx[r];
#pragma unroll
            for (int c0 = 0; c0 < CP; c0 += W) {
                const float* xc = x + c0;
                float mine[W], a[W], b[W], o[W];
#pragma unroll
                for (int j = 0; j < W; ++j) mine[j] = me[r][c0 + j];
                if (I.s.x >= 0) load_row_cg<W>(xc + (size_t)I.s.x * CP, a);
                if (I.s.y >= 0) load_row_cg<W>(xc + (size_t)I.s.y * CP, b);
                blur_row<W>(mine, a, b, I.s, o);
                if (pair) {
                    float pa[W], pb[W], q[W];
                    if (I.t.x >= 0) blur_at<W, CP>(xc, I.t.x, I.ta, pa);
                    if (I.t.y >= 0) blur_at<W, CP>(xc, I.t.y, I.tb, pb);
                    blur_row<W>(o, pa, pb, I.t, q);
#pragma unroll
                    for (int j = 0; j < W; ++j) o[j] = q[j];
                }
                store_row<W>(y + (size_t)v * CP + c0, o);
#pragma unroll
                for (int j = 0; j < W; ++j) me[r][c0 + j] = o[j];
            }
        }
        float* t = x; x = y; y = t;
        if (k + 2 < K) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int v = vb + threadIdx.x + r * blockDim.x;
                idx[r] = blur_idx(L.nbr, M, v < ve ? v : -1, axis(k + 2), axis(k + 3));
            }
            grid_barrier(L.hdr, phase);
        }
    }
    return x;
}

template <int CP>
__device__ __forceinline__ bool blur_fits_resident(int M, int threads) {
    return M <= threads * (CP <= 2 ? 2 : 1);
}

template <int PD, int CP>
__global__ void __launch_bounds__(kBlurThreads) k_blur_all(LatView L, float* buf0, float* buf1, uint8_t* bstate,
                                                             int reverse, int* final_flag, int flags) {
    extern __shared__ uint4 blur_queue[];
    const int M = L.hdr->m;
    const int stride = gridDim.x * blockDim.x;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned phase = 0;
    if (blur_fits_resident<CP>(M, stride) && !(flags & kBlurStream)) {
        float* res = blur_resident<PD, CP>(L, buf0, buf1, reverse, M, phase);
        if (tid == 0) *final_flag = (res == buf1) ? 1 : 0;
    } else if (flags & kBlurHalf) {
        blur_streaming<PD, CP, true>(L.nbr, bstate, L.hdr, buf0, buf1, reverse, final_flag, M, tid, stride,
                                     blur_queue, phase);
    } else {
        blur_streaming<PD, CP, false>(L.nbr, bstate, L.hdr, buf0, buf1, reverse, final_flag, M, tid, stride,
                                      blur_queue, phase);
    }
    // The barrier counters must be zero when the next cooperative kernel on
    // this lattice starts.  The kernel that follows a blur in stream order
    // (the slice, or the feature-gradient kernels) zeroes them when it starts
    // (reset_barrier), after every CTA of the blur has finished; so the blur
    // ends without an exit protocol (a fence and counter atomics per CTA).
}

// Zeroes the grid-barrier counters of the lattice (one thread): called at the
// start of the kernel that follows a blur, whose CTAs (and those of the
// zero-then-splat kernel before it) have all finished.
__device__ __forceinline__ void reset_barrier(LatticeHeader* hdr) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        hdr->bar_count = 0u;
        hdr->bar_gen = 0u;
        hdr->bar_zero = 0u;
    }
}

// ---------------------------------------------------------------- status

// The last kernel of a call copies the lattice's status word, with the
// call's sequence number, to the call's slot of the host-mapped status ring
// (one thread; every earlier kernel of the call has finished, stream order).
__device__ __forceinline__ void report_status(unsigned long long* slot, unsigned seq, const LatticeHeader* hdr) {
    if (slot && blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned st = (unsigned)*reinterpret_cast<const volatile int*>(&hdr->status);
        *reinterpret_cast<volatile unsigned long long*>(slot) = ((unsigned long long)seq << 32) | st;
    }
}

// ---------------------------------------------------------------- slice

// FWD: out = sum_i w_i val_i[0:V] / sum_i w_i val_i[V], weight_out = 1/sum;
// otherwise the unnormalised gather of V channels (permutohedral.cu:401-413,
// 487-496).  One thread per pixel; the tile's vertex ids staged in shared
// memory.

// One thread per pixel.  The K slot records are loaded first, then the K
// vertex ids through L1 (the tile's few hundred staged ids are shared by its
// 256 pixels), then the K rows: no shared-memory stage and no barrier, so
// every warp proceeds on its own.
template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P, slice_min_blocks<PD, V>())
k_slice(float* __restrict__ out, float* __restrict__ wout, Geo geo, LatView L, const float* __restrict__ lat0,
        const float* __restrict__ lat1, unsigned long long* st_slot, unsigned st_seq) {
    using C = Cfg<PD>;
    constexpr int K = C::K, P = C::P;
    constexpr int CP = FWD ? pad_ch(V + 1) : pad_ch(V);
    constexpr int NC = FWD ? V + 1 : V;
    report_status(st_slot, st_seq, L.hdr);
    reset_barrier(L.hdr);
    const float* __restrict__ lat = L.hdr->blur_final ? lat1 : lat0;
    const int t = threadIdx.x;
    int tile;
    const TilePos tp = tile_pos_grid<C::TW, C::TH>(geo, &tile);
    const bool act = tp.x0 + (t % C::TW) < geo.w && tp.y0 + (t / C::TW) < geo.h;
    const size_t p = (size_t)(tp.pix0 + (long long)(t / C::TW) * geo.w + (t % C::TW));
    int vid[K];
    float w[K];
    const size_t so = (size_t)tile * K * P + t;
#pragma unroll
    for (int c = 0; c < K; ++c) {
        vid[c] = act ? (int)L.slot_lid[so + (size_t)c * P] : 0;
        w[c] = act ? L.slot_w[so + (size_t)c * P] : 0.0f;
    }
    const int off = act ? L.tile_off[tile] : 0;
#pragma unroll
    for (int c = 0; c < K; ++c) vid[c] = act ? __ldg(L.staged_vid + off + vid[c]) : -1;
    float acc[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int c = 0; c < K; ++c) {
        if (vid[c] < 0) continue;   // inactive pixel, or failed insert (reported in the status word)
        float rw[CP];
        load_row<CP>(lat + (size_t)vid[c] * CP, rw);
#pragma unroll
        for (int j = 0; j < NC; ++j) acc[j] = __fmaf_rn(w[c], rw[j], acc[j]);
    }
    if (act) {
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
}

// ---------------------------------------------------------------- slice, streamed

// The slice as persistent CTAs that stream the per-slot records of their
// tiles into shared memory ahead of use.  Each CTA takes tiles blockIdx.x,
// blockIdx.x + gridDim.x, ...; kSliceStages tiles ahead, thread 0 issues
// bulk copies of the tile's local ids, weights and the tile's vertex ids
// (staged_vid[tile_off .. tile_off + tile_cnt), widened to 16-byte bounds)
// into a ring of stages.  The HBM stream of the records thus overlaps the
// L2 gathers of the rows, and no thread holds registers for loads in flight.
// Same arithmetic as k_slice (permutohedral.cu:401-413, 487-496).
constexpr int kSliceStages = 3;
template <int PD>
constexpr bool kSlicePiped = Cfg<PD>::P == 256;

template <int PD>
struct SliceStage {
    static constexpr int SLOTS = Cfg<PD>::SLOTS;
    static constexpr int LID_B = SLOTS * 2;            // multiple of 128 (P >= 64)
    static constexpr int W_B = SLOTS * 4;
    static constexpr int VID_N = SLOTS + 32;           // room for the 16-byte widening
    static constexpr int BYTES = LID_B + W_B + VID_N * 4;
};

template <int PD>
__host__ __device__ constexpr int slice_pipe_smem_bytes() {
    return kSliceStages * SliceStage<PD>::BYTES;
}

template <int PD, int V, bool FWD>
__global__ void __launch_bounds__(Cfg<PD>::P, 1024 / Cfg<PD>::P)
k_slice_pipe(float* __restrict__ out, float* __restrict__ wout, Geo geo, LatView L, const float* __restrict__ lat0,
             const float* __restrict__ lat1, unsigned long long* st_slot, unsigned st_seq) {
    using C = Cfg<PD>;
    using SS = SliceStage<PD>;
    constexpr int K = C::K, P = C::P, SLOTS = C::SLOTS, ST = kSliceStages;
    constexpr int CP = FWD ? pad_ch(V + 1) : pad_ch(V);
    constexpr int NC = FWD ? V + 1 : V;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ uint64_t full[ST];
    __shared__ int vshift[ST];
    report_status(st_slot, st_seq, L.hdr);
    reset_barrier(L.hdr);
    const float* __restrict__ lat = L.hdr->blur_final ? lat1 : lat0;
    const int t = threadIdx.x;
    const int first = blockIdx.x, stride = gridDim.x;
    const int mine = first < geo.tiles ? (geo.tiles - 1 - first) / stride + 1 : 0;

    // thread 0: copy tile i of this CTA (tile_off `off`, tile_cnt `cnt`) into stage i % ST
    auto issue = [&](int i, int off, int cnt) {
        const int s = i % ST;
        const int tile = first + i * stride;
        unsigned char* st = smem_raw + s * SS::BYTES;
        const int v0 = off & ~3, v1 = (off + cnt + 3) & ~3;   // staged_vid widened to 16-byte bounds
        const unsigned vbytes = (unsigned)(v1 - v0) * 4u;
        vshift[s] = off - v0;
        mbar_expect_tx(&full[s], (unsigned)(SS::LID_B + SS::W_B) + vbytes);
        bulk_g2s(st, L.slot_lid + (size_t)tile * SLOTS, SS::LID_B, &full[s]);
        bulk_g2s(st + SS::LID_B, L.slot_w + (size_t)tile * SLOTS, SS::W_B, &full[s]);
        if (vbytes) bulk_g2s(st + SS::LID_B + SS::W_B, L.staged_vid + v0, vbytes, &full[s]);
    };
    int nx_off = 0, nx_cnt = 0;   // thread 0: tile_off / tile_cnt of the next tile to issue
    if (t == 0) {
        for (int s = 0; s < ST; ++s) mbar_init(&full[s], 1);
        mbar_init_fence();
        int offs[ST], cnts[ST];
#pragma unroll
        for (int i = 0; i < ST; ++i) {
            offs[i] = i < mine ? L.tile_off[first + i * stride] : 0;
            cnts[i] = i < mine ? L.tile_cnt[first + i * stride] : 0;
        }
        if (ST < mine) {
            nx_off = L.tile_off[first + ST * stride];
            nx_cnt = L.tile_cnt[first + ST * stride];
        }
#pragma unroll
        for (int i = 0; i < ST; ++i)
            if (i < mine) issue(i, offs[i], cnts[i]);
    }
    __syncthreads();   // barriers initialised, first stages issued

    TileWalk walk(geo, first, stride);
    int i = 0;
    for (; i < mine; ++i) {
        const int s = i % ST;
        const bool got = mbar_wait(&full[s], (unsigned)((i / ST) & 1), L.hdr);
        // every thread has its stage, and every thread is done with tile i-1
        if (!__syncthreads_and(got)) break;
        if (t == 0 && i >= 1 && i - 1 + ST < mine) {   // refill the stage of tile i-1
            issue(i - 1 + ST, nx_off, nx_cnt);
            if (i + ST < mine) {
                nx_off = L.tile_off[first + (i + ST) * stride];
                nx_cnt = L.tile_cnt[first + (i + ST) * stride];
            }
        }
        const unsigned char* st = smem_raw + s * SS::BYTES;
        const uint16_t* slid = reinterpret_cast<const uint16_t*>(st);
        const float* sw = reinterpret_cast<const float*>(st + SS::LID_B);
        const int* svid = reinterpret_cast<const int*>(st + SS::LID_B + SS::W_B) + vshift[s];
        const TilePos tp = walk.pos<C::TW, C::TH>(geo);
        walk.advance();
        const bool act = tp.x0 + (t % C::TW) < geo.w && tp.y0 + (t / C::TW) < geo.h;
        const size_t p = (size_t)(tp.pix0 + (long long)(t / C::TW) * geo.w + (t % C::TW));
        // an inactive pixel, or a corner whose insert failed (reported in the
        // status word), reads row 0 with weight 0
        int vid[K];
        float w[K];
#pragma unroll
        for (int c = 0; c < K; ++c) {
            const int v = act ? svid[slid[c * P + t]] : -1;
            w[c] = v >= 0 ? sw[c * P + t] : 0.0f;
            vid[c] = v >= 0 ? v : 0;
        }
        // all K rows requested before the first is used (one L2 round trip per tile)
        float rw[K][CP];
#pragma unroll
        for (int c = 0; c < K; ++c) load_row<CP>(lat + (size_t)vid[c] * CP, rw[c]);
        float acc[NC];
#pragma unroll
        for (int j = 0; j < NC; ++j) acc[j] = 0.0f;
#pragma unroll
        for (int c = 0; c < K; ++c) {
#pragma unroll
            for (int j = 0; j < NC; ++j) acc[j] = __fmaf_rn(w[c], rw[c][j], acc[j]);
        }
        if (act) {
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
    }
    // A wait that gave up (recorded as PL_ST_SPIN): the copies still in
    // flight -- tiles i up to the last one issued -- land before the CTA exits (bounded).
    if (i < mine && t == 0) {
        const int last = i == 0 ? ST - 1 : i + ST - 2;   // the last tile issued
        for (int j = i; j < mine && j <= last; ++j)
            for (int r = 0; r < kMbarSpin && !mbar_test(&full[j % ST], (unsigned)((j / ST) & 1)); ++r) {
            }
    }
}

// ---------------------------------------------------------------- feature gradient

// The features enter the filter only through the barycentric weights (the
// vertex assignment is piecewise constant).  With R = the blurred forward
// lattice values, Z_p = 1 / weight_p, G_p = dL/dout_p and H = B^T S'(d),
// d_p = (G_p, -(G_p . out_p)) / Z_p:
//   dL/dw_pc = (G_p . R[v][0:V] - (G_p . out_p) R[v][V]) / Z_p + H[v] . (val_p, 1),
//   dL/de_i  = (dL/dw_{PD-rank_i} - dL/dw_{(PD+1-rank_i) mod K}) / K,
// (the derivative of permutohedral.cu:224-233), and dL/df through the
// elevation recurrence of permutohedral.cu:166-173.  The reference has no
// feature gradient (plattice.py:19 returns None).

// e_p = (G_p, -(G_p . out_p)): the V+1 channels splatted (times 1/Z_p) for H
template <int V>
static __global__ void k_fgrad_prep(float* __restrict__ ev, const float* __restrict__ grad,
                                    const float* __restrict__ out, size_t n, LatticeHeader* hdr) {
    reset_barrier(hdr);   // (it follows a blur)
    for (size_t p = (size_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (size_t)gridDim.x * blockDim.x) {
        float dot = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const float gj = __ldg(grad + p * V + j);
            dot = __fmaf_rn(gj, __ldg(out + p * V + j), dot);
            ev[p * (V + 1) + j] = gj;
        }
        ev[p * (V + 1) + V] = -dot;
    }
}

template <int PD, int V>
__global__ void __launch_bounds__(Cfg<PD>::P)
k_fgrad(float* __restrict__ gfeat, const float* __restrict__ feat, const float* __restrict__ vals,
        const float* __restrict__ grad, const float* __restrict__ outp, const float* __restrict__ winv, Geo geo,
        EmbedConsts ec, LatView L, const float* R0, const float* R1, const float* H0, const float* H1,
        const int* flags, unsigned long long* st_slot, unsigned st_seq) {
    using C = Cfg<PD>;
    report_status(st_slot, st_seq, L.hdr);
    reset_barrier(L.hdr);   // (it follows a blur)
    constexpr int K = C::K, P = C::P, SLOTS = C::SLOTS;
    constexpr int CP = pad_ch(V + 1);
    __shared__ int svid[SLOTS];
    __shared__ int scol[2 * K * P];   // embed scratch, then dL/dw by corner; column t per thread
    const float* __restrict__ R = flags[0] ? R1 : R0;
    const float* __restrict__ H = flags[1] ? H1 : H0;
    const int t = threadIdx.x;
    int tile;
    const TilePos tp = tile_pos_grid<C::TW, C::TH>(geo, &tile);
    const int x = tp.x0 + (t % C::TW);
    const int y = tp.y0 + (t / C::TW);
    const bool act = x < geo.w && y < geo.h;
    const size_t p = (size_t)(tp.pix0 + (long long)(t / C::TW) * geo.w + (t % C::TW));
    const size_t so = (size_t)tile * K * P + t;
    int lid[K];
    float w[K];
#pragma unroll
    for (int c = 0; c < K; ++c) {
        lid[c] = act ? (int)L.slot_lid[so + (size_t)c * P] : 0;
        w[c] = act ? L.slot_w[so + (size_t)c * P] : 0.0f;
    }
    const int cnt = L.tile_cnt[tile], off = L.tile_off[tile];
    for (int u = t; u < cnt; u += P) svid[u] = L.staged_vid[off + u];
    float f[PD];
#pragma unroll
    for (int i = 0; i < PD; ++i) f[i] = act ? __ldg(feat + p * PD + i) : 0.0f;
    int g[K], rank[K];
    float bary[K];
    int ir[K];
    embed<PD>(f, ec, g, rank, bary, scol + t, ir);
    __syncthreads();
    if (!act) return;
    float G[V], vv[V];
    float gdot = 0.0f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        G[j] = __ldg(grad + p * V + j);
        vv[j] = __ldg(vals + p * V + j);
        gdot = __fmaf_rn(G[j], __ldg(outp + p * V + j), gdot);
    }
    const float zinv = __ldg(winv + p);
    float* dwc = reinterpret_cast<float*>(scol) + t;   // dL/dw of corner c at dwc[c * P]
#pragma unroll
    for (int c = 0; c < K; ++c) {
        const int vid = svid[lid[c]];
        float dw = 0.0f;
        if (vid >= 0) {
            float r[CP], hh[CP];
            load_row<CP>(R + (size_t)vid * CP, r);
            load_row<CP>(H + (size_t)vid * CP, hh);
            float sl = 0.0f, sp = hh[V];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                sl = __fmaf_rn(G[j], r[j], sl);
                sp = __fmaf_rn(hh[j], vv[j], sp);
            }
            sl = __fmaf_rn(-gdot, r[V], sl);
            dw = __fmaf_rn(sl, zinv, sp);
        }
        dwc[c * P] = dw;
    }
    float de[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
        const int r = rank[i];
        de[i] = (dwc[(PD - r) * P] - dwc[(r == 0 ? 0 : PD + 1 - r) * P]) * ec.rk;
    }
    float gf[PD];
#pragma unroll
    for (int i = 0; i < PD; ++i) gf[i] = 0.0f;
    float carry = 0.0f;
#pragma unroll
    for (int i = 0; i <= PD; ++i) {
        carry += de[i];
        if (i == 0) {
            gf[0] = __fmaf_rn(2.0f * ec.sf[0], carry, gf[0]);
        } else if (i < PD) {
            gf[i - 1] = __fmaf_rn(-(float)i * ec.sf[i - 1], carry, gf[i - 1]);
            gf[i] = __fmaf_rn((float)(i + 2) * ec.sf[i], carry, gf[i]);
        } else {
            gf[PD - 1] = __fmaf_rn(-(float)PD * ec.sf[PD - 1], carry, gf[PD - 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < PD; ++i) gfeat[p * PD + i] = gf[i];
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
