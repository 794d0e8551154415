// plattice_layout.h -- host+device description of the lattice and scratch
// buffers used by the sm_100a permutohedral-lattice filter.
//
// Geometry.  A call filters b images of h x w pixels (b = 1 for the
// single-image entry points).  Each image is cut into tiles of P pixels (32
// wide, P/32 high); the tiles of all images are numbered image by image.  One
// CTA owns one tile in every per-pixel kernel, so each tile's distinct lattice
// vertices (at most P*K, K = pd+1) can be deduplicated in shared memory and
// addressed by a 16-bit local id.  The b images share one lattice: the key
// hash mixes in the image index, so equal coordinates in two images are two
// different vertices (see hash_of_key in plattice_kernels.cuh), and every
// stage runs once over all images.
//
// Lattice blob (kept from forward to backward; everything before vb0 is
// independent of vd):
//   hdr            LatticeHeader (status word, vertex count m, staged count)
//   tile_off/cnt   per tile: offset and length of its unique-vertex list
//   slot_lid       [tile][K][P] uint16   local id of each (pixel, simplex corner)
//   slot_w         [tile][K][P] float    barycentric weight of the same slot
//   slot_order     [tile][K*P]  uint16   the tile's slots sorted by local id:
//                                        (pixel << 1) | 1 where a local id's
//                                        run of slots starts
//   slot_wsort     [tile][K*P]  float    the weights in that sorted order
//   first_lid      [tile][P]    uint16   local id at sorted position t*K (the
//                                        first position of splat thread t)
//   staged_vid     [U]          int32    global vertex id of each staged key
//   nbr            [K][m]       int2     blur neighbours (+, -) per axis, -1 absent
//   vb0            [m][CPb]     float    the first backward's splat target: zeroed
//                                        by the forward's tile build, so that a
//                                        backward right after its forward needs
//                                        no zeroing pass (CPb = pad(vd))
// Scratch blob: a front part that every call uses -- the lattice value rows
// of its blur and their bookkeeping -- and a build part that only a call
// which builds the lattice uses:
//   v1             [m][CPf]     float    lattice values, the ping-pong partner of
//                                        v0 (forward) or of vb0 (backward)
//   bstate         [2][slots]   uint8    blur bookkeeping of large lattices: per
//                                        vertex, the buffer holding its row and
//                                        its pending halvings (ping-pong)
//   v0             [m][CPf]     float    the forward's splat target (CPf = pad(vd+1))
// (a backward on a kept lattice needs only v1 and bstate: reuse_bytes)
//   -- build part --
//   staged_keys    [U][CW]      uint4    each tile's unique keys (word 0: hash)
//   table          [cap]        uint32   open-addressed hash table: 0 empty, else
//                                        1 + staged index of the owning key in the
//                                        low bits, hash bits above (a tag)
//   filter         [cap]        uint8    miss filter of large tables
//   owner          [U]          int32    staged index of the owner of each staged key
//   vid_of         [U]          int32    vertex id of each owner
//   vkeys          [m][CW]      uint4    key of every vertex
// U, m <= slots = tiles*K*P: buffers are sized for that bound, but every kernel
// reads the live counts from the header and touches only what is used.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define PL_MAX_PD 16
#define PL_MAX_VD 8

// status bits (LatticeHeader::status)
#define PL_ST_SMEM_PROBE 1   /* tile-local table exhausted (cannot happen: sized 2x) */
#define PL_ST_TABLE_FULL 2   /* global hash table probe limit reached */
#define PL_ST_SPIN 4         /* a bounded wait (grid barrier) gave up */
#define PL_ST_ROUNDS 8       /* global insert did not settle within the round limit */

typedef struct {
    int status;
    int m;           /* distinct vertices */
    int u_total;     /* staged (tile-unique) keys */
    int cap_log2;    /* hash table capacity in use (log2 of cells) */
    int n, pd, vd, tiles;
    unsigned bar_count, bar_gen;   /* grid barrier of the cooperative blur kernel; bar_gen spare (zero) */
    int blur_final;  /* which value buffer (0/1) holds the last blur's result */
    unsigned bar_zero;   /* grid barrier of the zero-then-splat kernel */
    int pad[52];     /* header is 256 bytes */
} LatticeHeader;

typedef char pl_header_is_256_bytes[(sizeof(LatticeHeader) == 256) ? 1 : -1];

static inline int pl_tile_pixels(int pd) { return pd <= 6 ? 256 : (pd <= 10 ? 128 : 64); }
static inline int pl_key_words(int pd) { return (4 + 2 * pd + 15) / 16; }   /* 16-byte words */
static inline int pl_pad_ch(int c) { return c <= 2 ? c : ((c + 3) / 4) * 4; }
static inline size_t pl_align(size_t x) { return (x + 255) & ~(size_t)255; }

typedef struct {
    int b, h, w, pd, vd, K, P, TH, tiles_x, tiles_y, tiles_img, tiles;
    int CW, CPf, CPb;
    long long n_img;      /* pixels per image */
    long long slots;      /* tiles*K*P: bound on staged keys and on vertices */
    int cap_max_log2;     /* table cells allocated = 2^cap_max_log2 >= 2*slots */
    size_t off_tile_off, off_tile_cnt, off_slot_lid, off_slot_w, off_slot_order, off_slot_wsort, off_first_lid,
        off_staged_vid, off_nbr, off_vb0, lattice_bytes;
    size_t off_v0, off_v1, off_bstate, reuse_bytes, rows_bytes;   /* scratch front part */
    size_t off_skeys, off_table, off_filter, off_owner, off_vid_of, off_vkeys, scratch_bytes;
} PlLayout;

static inline void pl_layout_batch(PlLayout* L, int b, int h, int w, int pd, int vd) {
    L->b = b; L->h = h; L->w = w; L->pd = pd; L->vd = vd; L->K = pd + 1;
    L->P = pl_tile_pixels(pd);
    L->TH = L->P / 32;
    L->tiles_x = (w + 31) / 32;
    L->tiles_y = (h + L->TH - 1) / L->TH;
    L->tiles_img = L->tiles_x * L->tiles_y;
    L->tiles = L->tiles_img * b;
    L->n_img = (long long)h * w;
    L->CW = pl_key_words(pd);
    L->CPf = pl_pad_ch(vd + 1);
    L->CPb = pl_pad_ch(vd);
    L->slots = (long long)L->tiles * L->K * L->P;
    int lg = 6;
    while ((1ll << lg) < 2 * L->slots) lg++;
    L->cap_max_log2 = lg;
    const size_t S = (size_t)L->slots, T = (size_t)L->tiles;
    size_t o = pl_align(sizeof(LatticeHeader));
    L->off_tile_off = o;   o = pl_align(o + T * 4);
    L->off_tile_cnt = o;   o = pl_align(o + T * 4);
    L->off_slot_lid = o;   o = pl_align(o + S * 2);
    L->off_slot_w = o;     o = pl_align(o + S * 4);
    L->off_slot_order = o; o = pl_align(o + S * 2);
    L->off_slot_wsort = o; o = pl_align(o + S * 4);
    L->off_first_lid = o;  o = pl_align(o + T * (size_t)L->P * 2);
    L->off_staged_vid = o; o = pl_align(o + S * 4);
    L->off_nbr = o;        o = pl_align(o + S * L->K * 8);
    L->off_vb0 = o;        o = pl_align(o + S * L->CPb * 4);
    L->lattice_bytes = o;
    o = 0;
    L->off_v1 = o;         o = pl_align(o + S * L->CPf * 4);
    L->off_bstate = o;     o = pl_align(o + 2 * S);
    L->reuse_bytes = o;
    L->off_v0 = o;         o = pl_align(o + S * L->CPf * 4);
    L->rows_bytes = o;
    L->off_skeys = o;      o = pl_align(o + S * L->CW * 16);
    L->off_table = o;      o = pl_align(o + ((size_t)1 << lg) * 4);
    L->off_filter = o;     o = pl_align(o + ((size_t)1 << lg));
    L->off_owner = o;      o = pl_align(o + S * 4);
    L->off_vid_of = o;     o = pl_align(o + S * 4);
    L->off_vkeys = o;      o = pl_align(o + S * L->CW * 16);
    L->scratch_bytes = o;
}

static inline void pl_layout(PlLayout* L, int h, int w, int pd, int vd) { pl_layout_batch(L, 1, h, w, pd, vd); }
