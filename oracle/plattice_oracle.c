/*
 * plattice_oracle.c -- CPU oracle for the permutohedral-lattice filter.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
 * this file: it is the checker that the CUDA path is compared against (tests,
 * the smoke check and the CPU-baseline leg of the benchmark).
 *
 * It restates, sequentially and in plain C, the algorithm of the reference
 * CUDA filter (OliveMY/plattice_pytorch, permutohedral.cu):
 *   - lattice constants           permutohedral.cu:502-517
 *   - elevation onto H_d          permutohedral.cu:165-173
 *   - greedy nearest zero point   permutohedral.cu:175-186
 *   - rank by counting            permutohedral.cu:188-198
 *   - rank / greedy fix-up        permutohedral.cu:200-221
 *   - barycentric weights         permutohedral.cu:223-233
 *   - the K vertex keys           permutohedral.cu:236-250
 *   - splat [v*w, w]              permutohedral.cu:286-293, 316-318
 *   - blur neighbours             permutohedral.cu:364-381
 *   - [1 2 1]/4 blur per axis     permutohedral.cu:341-347, axis order 585 (fwd) / 647 (bwd)
 *   - normalised slice            permutohedral.cu:401-413
 *   - backward splat / slice      permutohedral.cu:437-445, 487-496
 * The hash table is this file's own (sequential open addressing); only the
 * resulting vertex key set matters, not the table layout.
 *
 * A few float steps of the reference are left to the CUDA compiler's FMA
 * contraction under --use_fast_math.  Which contraction the reference build
 * actually used is an empirical fact; the `variant` bit mask selects between
 * the candidates and is pinned against golden vectors produced by the
 * reference build itself (tests/golden).
 *
 * Also here: the gradient of the forward filter with respect to the features
 * (the reference returns none, plattice.py:19), derived from the forward above:
 * the features enter only through the barycentric weights (the vertex
 * assignment is piecewise constant), so with R = blurred lattice values,
 * Z_p = the normaliser, G_p = dL/dout_p and H = B^T S'(G/Z, -(G.out)/Z):
 *   dL/dw_pc = (G_p . R[v][0:V] - (G_p . out_p) R[v][V]) / Z_p + H[v] . (val_p, 1),
 *   dL/de_i(r) = (dL/dw_{pd-r} - dL/dw_{(pd+1-r) mod K}) / K   (i(r): coordinate of rank r),
 * and dL/df through the elevation recurrence of permutohedral.cu:165-173.
 * Also here: a brute-force dense Gaussian filter out_p = sum_q g_pq v_q /
 * sum_q g_pq with g_pq = exp(-|f_p - f_q|^2 / 2), the generalisation to any
 * features of the reference test's brute_force_bilateral
 * (tests/test_plattice.py:58-77, whose features are (x/ss, y/ss, rgb/sr)),
 * and its value-gradient (the transpose with the normaliser held fixed).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PO_MAX_PD 16

/* variant bits: which float steps are fused multiply-adds */
#define PO_ELEV_FMA_SUB 1  /* e[i+1] - (i*f[i-1])*sf[i-1]  ->  fma(-(i*f), sf, e) */
#define PO_ELEV_FMA_ADD 2  /* s + ((i+2)*f[i])*sf[i]        ->  fma((i+2)*f, sf, s) */
#define PO_BARY_FMA     4  /* b[x] +/- (e-g)*(1/K)          ->  fma(+/-(e-g), 1/K, b[x]) */
#define PO_SLICE_FMA    8  /* acc + w*val                   ->  fma(w, val, acc) */

/* status codes */
#define PO_OK 0
#define PO_EINVAL 1
#define PO_ENOMEM 2

/* ------------------------------------------------------------------------ */
/* lattice constants: permutohedral.cu:502-517 (scale factors; the reference  */
/* computes them on the host in float)                                        */

static void po_scale_factors(int pd, float* sf) {
    for (int i = 0; i < pd; i++) {
        float var = (1.0f / 6.0f) + 0.5f;
        sf[i] = (float)(pd + 1) * sqrtf(var / (float)((i + 1) * (i + 2)));
    }
}

/* float -> int16 as the device conversion does it: truncate toward zero,
 * saturate to the int16 range */
static int po_f2s16(float x) {
    if (!(x == x)) return 0;
    if (x >= 32767.0f) return 32767;
    if (x <= -32768.0f) return -32768;
    return (int)(int16_t)(int)x;
}

/* Per-pixel lattice embedding: K = pd+1 vertex keys (pd int16 coordinates
 * each, the (pd+1)-th is implied by the zero sum) and K barycentric weights.
 * permutohedral.cu:165-250 */
static void po_embed(const float* f, int pd, const float* sf, int var,
                     int16_t* keys /* [K][pd] */, float* w /* [K] */, int* rank_out /* [K] or NULL */) {
    const int K = pd + 1;
    float e[PO_MAX_PD + 1];
    int g[PO_MAX_PD + 1];
    int rank[PO_MAX_PD + 1];
    float b[PO_MAX_PD + 2];

    /* elevation (permutohedral.cu:166-173) */
    e[pd] = ((float)(-pd) * f[pd - 1]) * sf[pd - 1];
    for (int i = pd - 1; i > 0; i--) {
        float a = (float)i * f[i - 1];
        float c = (float)(i + 2) * f[i];
        float s;
        if (var & PO_ELEV_FMA_SUB) s = fmaf(-a, sf[i - 1], e[i + 1]);
        else                       s = e[i + 1] - a * sf[i - 1];
        if (var & PO_ELEV_FMA_ADD) e[i] = fmaf(c, sf[i], s);
        else                       e[i] = s + c * sf[i];
    }
    {
        float a0 = 2.0f * f[0];
        if (var & PO_ELEV_FMA_ADD) e[0] = fmaf(a0, sf[0], e[1]);
        else                       e[0] = e[1] + a0 * sf[0];
    }

    /* greedy rounding to the nearest multiple of K (permutohedral.cu:176-186);
     * the running sum is an int16 in the reference */
    const float rk = 1.0f / (float)K;
    int16_t sum = 0;
    for (int i = 0; i <= pd; i++) {
        float v = e[i] * rk;
        float up = ceilf(v) * (float)K;
        float dn = floorf(v) * (float)K;
        g[i] = (up - e[i] < e[i] - dn) ? po_f2s16(up) : po_f2s16(dn);
        sum = (int16_t)(sum + g[i]);
    }
    sum = (int16_t)(sum / K);

    /* rank by counting, ties broken by index (permutohedral.cu:189-198) */
    for (int i = 0; i <= pd; i++) {
        int r = 0;
        float di = e[i] - (float)g[i];
        for (int j = 0; j <= pd; j++) {
            float dj = e[j] - (float)g[j];
            if (di < dj || (di == dj && i > j)) r++;
        }
        rank[i] = r;
    }

    /* fix-up when the greedy point is off the hyperplane (permutohedral.cu:201-221) */
    if (sum > 0) {
        for (int i = 0; i <= pd; i++) {
            if (rank[i] >= K - sum) { g[i] -= K; rank[i] += sum - K; }
            else                    { rank[i] += sum; }
        }
    } else if (sum < 0) {
        for (int i = 0; i <= pd; i++) {
            if (rank[i] < -sum) { g[i] += K; rank[i] += K + sum; }
            else                { rank[i] += sum; }
        }
    }

    /* barycentric coordinates (permutohedral.cu:224-233) */
    for (int i = 0; i <= pd + 1; i++) b[i] = 0.0f;
    for (int i = 0; i <= pd; i++) {
        float d = e[i] - (float)g[i];
        int lo = pd - rank[i], hi = pd + 1 - rank[i];
        if (var & PO_BARY_FMA) {
            b[lo] = fmaf(d, rk, b[lo]);
            b[hi] = fmaf(-d, rk, b[hi]);
        } else {
            float delta = d * rk;
            b[lo] += delta;
            b[hi] -= delta;
        }
    }
    b[0] += 1.0f + b[pd + 1];

    /* vertex keys of the enclosing simplex (permutohedral.cu:238-250) */
    for (int c = 0; c <= pd; c++) {
        for (int i = 0; i < pd; i++) {
            int k = (int16_t)(g[i] + c);
            if (rank[i] > pd - c) k = (int16_t)(k - K);
            keys[c * pd + i] = (int16_t)k;
        }
        w[c] = b[c];
    }
    if (rank_out)
        for (int i = 0; i <= pd; i++) rank_out[i] = rank[i];
}

/* ------------------------------------------------------------------------ */
/* sequential hash set of int16 keys                                        */

typedef struct {
    int pd;
    uint64_t mask;
    int32_t* cells;   /* vertex id + 1, 0 = empty */
    int16_t* vkeys;   /* [cap_vertices][pd] */
    long nv;
} po_table;

static uint64_t po_hash(const int16_t* k, int pd) {
    uint64_t h = 0x9E3779B97F4A7C15ull;
    for (int i = 0; i < pd; i++) {
        h ^= (uint64_t)(uint16_t)k[i];
        h *= 0xFF51AFD7ED558CCDull;
        h ^= h >> 29;
    }
    h ^= h >> 32;
    h *= 0xC4CEB9FE1A85EC53ull;
    h ^= h >> 29;
    return h;
}

static int po_table_init(po_table* t, int pd, long max_vertices) {
    uint64_t cap = 16;
    while (cap < (uint64_t)(2 * max_vertices)) cap <<= 1;
    t->pd = pd;
    t->mask = cap - 1;
    t->cells = (int32_t*)calloc(cap, sizeof(int32_t));
    t->vkeys = (int16_t*)malloc((size_t)max_vertices * pd * sizeof(int16_t) + 2);
    t->nv = 0;
    if (!t->cells || !t->vkeys) { free(t->cells); free(t->vkeys); return PO_ENOMEM; }
    return PO_OK;
}

static void po_table_free(po_table* t) { free(t->cells); free(t->vkeys); }

/* insert == 1: insert when absent; returns vertex id, or -1 when absent */
static long po_table_find(po_table* t, const int16_t* key, int insert) {
    const int pd = t->pd;
    uint64_t h = po_hash(key, pd) & t->mask;
    for (;;) {
        int32_t c = t->cells[h];
        if (c == 0) {
            if (!insert) return -1;
            long v = t->nv++;
            memcpy(t->vkeys + (size_t)v * pd, key, pd * sizeof(int16_t));
            t->cells[h] = (int32_t)(v + 1);
            return v;
        }
        if (memcmp(t->vkeys + (size_t)(c - 1) * pd, key, pd * sizeof(int16_t)) == 0) return c - 1;
        h = (h + 1) & t->mask;
    }
}

/* ------------------------------------------------------------------------ */
/* lattice: per-slot vertex ids and weights, vertex keys, blur neighbours    */

typedef struct {
    long n;
    int pd;
    long m;
    int32_t* slot_vid;   /* [n*K] */
    float* slot_w;       /* [n*K] */
    int32_t* nbr;        /* [m][K][2]  (+, -) per axis, -1 = absent */
    po_table tab;
} po_lattice;

static void po_lattice_free(po_lattice* L) {
    free(L->slot_vid); free(L->slot_w); free(L->nbr); po_table_free(&L->tab);
}

static int po_lattice_build(po_lattice* L, const float* feat, long n, int pd, int var) {
    const int K = pd + 1;
    float sf[PO_MAX_PD];
    int16_t keys[(PO_MAX_PD + 1) * PO_MAX_PD];
    float w[PO_MAX_PD + 1];
    memset(L, 0, sizeof(*L));
    L->n = n; L->pd = pd;
    po_scale_factors(pd, sf);
    L->slot_vid = (int32_t*)malloc((size_t)n * K * sizeof(int32_t) + 4);
    L->slot_w = (float*)malloc((size_t)n * K * sizeof(float) + 4);
    if (!L->slot_vid || !L->slot_w) return PO_ENOMEM;
    if (po_table_init(&L->tab, pd, n * K + 1) != PO_OK) return PO_ENOMEM;
    for (long p = 0; p < n; p++) {
        po_embed(feat + (size_t)p * pd, pd, sf, var, keys, w, NULL);
        for (int c = 0; c < K; c++) {
            L->slot_vid[p * K + c] = (int32_t)po_table_find(&L->tab, keys + c * pd, 1);
            L->slot_w[p * K + c] = w[c];
        }
    }
    L->m = L->tab.nv;
    /* blur neighbours: for axis c < pd the step is (1,..,1) - K e_c, for
     * c == pd it is (1,..,1); permutohedral.cu:364-381 */
    L->nbr = (int32_t*)malloc((size_t)L->m * K * 2 * sizeof(int32_t) + 4);
    if (!L->nbr) return PO_ENOMEM;
    int16_t np[PO_MAX_PD], nm[PO_MAX_PD];
    for (long v = 0; v < L->m; v++) {
        const int16_t* k = L->tab.vkeys + (size_t)v * pd;
        for (int c = 0; c < K; c++) {
            for (int i = 0; i < pd; i++) {
                np[i] = (int16_t)(k[i] + 1);
                nm[i] = (int16_t)(k[i] - 1);
            }
            if (c < pd) {
                np[c] = (int16_t)(np[c] - K);
                nm[c] = (int16_t)(nm[c] + K);
            }
            L->nbr[(v * K + c) * 2 + 0] = (int32_t)po_table_find(&L->tab, np, 0);
            L->nbr[(v * K + c) * 2 + 1] = (int32_t)po_table_find(&L->tab, nm, 0);
        }
    }
    return PO_OK;
}

/* one [1 2 1]/4 pass along axis c over C channels; a missing neighbour adds
 * nothing (permutohedral.cu:341-347) */
static void po_blur_axis(const po_lattice* L, int c, int C, const float* in, float* out) {
    const int K = L->pd + 1;
    for (long v = 0; v < L->m; v++) {
        int32_t a = L->nbr[(v * K + c) * 2 + 0];
        int32_t b = L->nbr[(v * K + c) * 2 + 1];
        for (int j = 0; j < C; j++) {
            float acc = 2.0f * in[v * C + j];
            if (a >= 0) acc += in[(long)a * C + j];
            if (b >= 0) acc += in[(long)b * C + j];
            out[v * C + j] = 0.25f * acc;
        }
    }
}

/* blur all axes: forward order 0..pd, backward pd..0; returns the buffer that
 * holds the result */
static float* po_blur(const po_lattice* L, int C, float* x, float* y, int reverse) {
    const int K = L->pd + 1;
    for (int s = 0; s < K; s++) {
        int c = reverse ? (K - 1 - s) : s;
        po_blur_axis(L, c, C, x, y);
        float* t = x; x = y; y = t;
    }
    return x;
}

static float po_madd(float acc, float w, float v, int var) {
    return (var & PO_SLICE_FMA) ? fmaf(w, v, acc) : acc + w * v;
}

/* ------------------------------------------------------------------------ */
/* public entry points (ctypes)                                             */

/* Per-slot keys [n][K][pd] and weights [n][K]; no hashing. */
int po_embed_all(const float* feat, long n, int pd, int var, int16_t* keys, float* w) {
    if (pd < 1 || pd > PO_MAX_PD || n < 0) return PO_EINVAL;
    const int K = pd + 1;
    float sf[PO_MAX_PD];
    po_scale_factors(pd, sf);
    for (long p = 0; p < n; p++)
        po_embed(feat + (size_t)p * pd, pd, sf, var, keys + (size_t)p * K * pd, w + (size_t)p * K, NULL);
    return PO_OK;
}

void po_scale_factors_out(int pd, float* sf) { po_scale_factors(pd, sf); }

/* Vertex key set: writes up to max_keys keys [m][pd] into vkeys (may be NULL),
 * per-slot vertex ids (may be NULL) and returns m (or -status on error). */
long po_vertex_keys(const float* feat, long n, int pd, int var,
                    int16_t* vkeys, long max_keys, int32_t* slot_vid) {
    if (pd < 1 || pd > PO_MAX_PD || n < 0) return -PO_EINVAL;
    po_lattice L;
    if (po_lattice_build(&L, feat, n, pd, var) != PO_OK) { po_lattice_free(&L); return -PO_ENOMEM; }
    long m = L.m;
    if (vkeys) {
        long k = m < max_keys ? m : max_keys;
        memcpy(vkeys, L.tab.vkeys, (size_t)k * pd * sizeof(int16_t));
    }
    if (slot_vid) memcpy(slot_vid, L.slot_vid, (size_t)n * (pd + 1) * sizeof(int32_t));
    po_lattice_free(&L);
    return m;
}

/* Forward filter: out [n][vd], weight_out [n] (the reciprocal normaliser).
 * Splat sums are accumulated in double and rounded once, the blur and the
 * slice follow the reference's float steps.  Returns m, or -status. */
long po_forward(const float* feat, const float* vals, long n, int pd, int vd, int var,
                float* out, float* weight_out) {
    if (pd < 1 || pd > PO_MAX_PD || vd < 1 || vd > 8 || n < 0) return -PO_EINVAL;
    const int K = pd + 1, C = vd + 1;
    po_lattice L;
    if (po_lattice_build(&L, feat, n, pd, var) != PO_OK) { po_lattice_free(&L); return -PO_ENOMEM; }
    double* acc = (double*)calloc((size_t)L.m * C + 1, sizeof(double));
    float* x = (float*)malloc(((size_t)L.m * C + 1) * sizeof(float));
    float* y = (float*)malloc(((size_t)L.m * C + 1) * sizeof(float));
    if (!acc || !x || !y) { free(acc); free(x); free(y); po_lattice_free(&L); return -PO_ENOMEM; }
    for (long p = 0; p < n; p++)
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            float w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) acc[v * C + j] += (double)(vals[p * vd + j] * w);
            acc[v * C + vd] += (double)w;
        }
    for (long i = 0; i < L.m * C; i++) x[i] = (float)acc[i];
    float* r = po_blur(&L, C, x, y, 0);
    for (long p = 0; p < n; p++) {
        float a[8] = {0};
        float ws = 0.0f;
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            float w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) a[j] = po_madd(a[j], w, r[v * C + j], var);
            ws = po_madd(ws, w, r[v * C + vd], var);
        }
        float inv = 1.0f / ws;
        for (int j = 0; j < vd; j++) out[p * vd + j] = a[j] * inv;
        weight_out[p] = inv;
    }
    long m = L.m;
    free(acc); free(x); free(y); po_lattice_free(&L);
    return m;
}

/* Backward (value gradient): grad_out [n][vd] from grad [n][vd] and the saved
 * normaliser weight_in [n]; blur axes in reverse order.  Returns m, or -status. */
long po_backward(const float* feat, const float* grad, const float* weight_in, long n,
                 int pd, int vd, int var, float* grad_out) {
    if (pd < 1 || pd > PO_MAX_PD || vd < 1 || vd > 8 || n < 0) return -PO_EINVAL;
    const int K = pd + 1, C = vd;
    po_lattice L;
    if (po_lattice_build(&L, feat, n, pd, var) != PO_OK) { po_lattice_free(&L); return -PO_ENOMEM; }
    double* acc = (double*)calloc((size_t)L.m * C + 1, sizeof(double));
    float* x = (float*)malloc(((size_t)L.m * C + 1) * sizeof(float));
    float* y = (float*)malloc(((size_t)L.m * C + 1) * sizeof(float));
    if (!acc || !x || !y) { free(acc); free(x); free(y); po_lattice_free(&L); return -PO_ENOMEM; }
    for (long p = 0; p < n; p++)
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            float w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++)
                acc[v * C + j] += (double)((grad[p * vd + j] * weight_in[p]) * w);
        }
    for (long i = 0; i < L.m * C; i++) x[i] = (float)acc[i];
    float* r = po_blur(&L, C, x, y, 1);
    for (long p = 0; p < n; p++) {
        float a[8] = {0};
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            float w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) a[j] = po_madd(a[j], w, r[v * C + j], var);
        }
        for (int j = 0; j < vd; j++) grad_out[p * vd + j] = a[j];
    }
    long m = L.m;
    free(acc); free(x); free(y); po_lattice_free(&L);
    return m;
}

/* one [1 2 1]/4 pass in double (the gradient's lattice sweeps) */
static double* po_blur_d(const po_lattice* L, int C, double* x, double* y, int reverse) {
    const int K = L->pd + 1;
    for (int s = 0; s < K; s++) {
        const int c = reverse ? (K - 1 - s) : s;
        for (long v = 0; v < L->m; v++) {
            const int32_t a = L->nbr[(v * K + c) * 2 + 0], b = L->nbr[(v * K + c) * 2 + 1];
            for (int j = 0; j < C; j++) {
                double acc = 2.0 * x[v * C + j];
                if (a >= 0) acc += x[(long)a * C + j];
                if (b >= 0) acc += x[(long)b * C + j];
                y[v * C + j] = 0.25 * acc;
            }
        }
        double* t = x; x = y; y = t;
    }
    return x;
}

/* Feature gradient dL/df [n][pd] of L = sum_p grad_p . out_p, out = the
 * forward filter of (features, values).  Lattice sweeps in double; the
 * forward lattice values as po_forward computes them.  Returns m or -status. */
long po_feature_grad(const float* feat, const float* vals, const float* grad, long n, int pd, int vd, int var,
                     float* grad_feat) {
    if (pd < 1 || pd > PO_MAX_PD || vd < 1 || vd > 8 || n < 0) return -PO_EINVAL;
    const int K = pd + 1, C = vd + 1;
    po_lattice L;
    if (po_lattice_build(&L, feat, n, pd, var) != PO_OK) { po_lattice_free(&L); return -PO_ENOMEM; }
    const size_t mc = (size_t)L.m * C + 1;
    double* acc = (double*)calloc(mc, sizeof(double));
    float* x = (float*)malloc(mc * sizeof(float));
    float* y = (float*)malloc(mc * sizeof(float));
    double* hx = (double*)calloc(mc, sizeof(double));
    double* hy = (double*)malloc(mc * sizeof(double));
    double* zp = (double*)malloc(((size_t)n + 1) * sizeof(double));
    double* go = (double*)malloc(((size_t)n + 1) * sizeof(double));   /* G_p . out_p */
    if (!acc || !x || !y || !hx || !hy || !zp || !go) {
        free(acc); free(x); free(y); free(hx); free(hy); free(zp); free(go); po_lattice_free(&L);
        return -PO_ENOMEM;
    }
    /* forward lattice values R, as po_forward */
    for (long p = 0; p < n; p++)
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            float w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) acc[v * C + j] += (double)(vals[p * vd + j] * w);
            acc[v * C + vd] += (double)w;
        }
    for (size_t i = 0; i + 1 < mc; i++) x[i] = (float)acc[i];
    const float* R = po_blur(&L, C, x, y, 0);
    /* per pixel: Z, out, G.out; splat of d_p = (G/Z, -(G.out)/Z) */
    for (long p = 0; p < n; p++) {
        double a[8] = {0}, z = 0.0;
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            double w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) a[j] += w * R[v * C + j];
            z += w * R[v * C + vd];
        }
        double gdot = 0.0;
        for (int j = 0; j < vd; j++) gdot += (double)grad[p * vd + j] * (a[j] / z);
        zp[p] = z;
        go[p] = gdot;
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            double w = L.slot_w[p * K + c];
            for (int j = 0; j < vd; j++) hx[v * C + j] += w * (double)grad[p * vd + j] / z;
            hx[v * C + vd] -= w * gdot / z;
        }
    }
    const double* H = po_blur_d(&L, C, hx, hy, 1);
    /* per pixel: dL/dw, then dL/de by rank, then dL/df through the elevation */
    float sf[PO_MAX_PD];
    po_scale_factors(pd, sf);
    int16_t keys[(PO_MAX_PD + 1) * PO_MAX_PD];
    float wt[PO_MAX_PD + 1];
    int rank[PO_MAX_PD + 1], coord_of_rank[PO_MAX_PD + 1];
    for (long p = 0; p < n; p++) {
        po_embed(feat + (size_t)p * pd, pd, sf, var, keys, wt, rank);
        for (int i = 0; i < K; i++) coord_of_rank[rank[i]] = i;
        double dw[PO_MAX_PD + 1];
        for (int c = 0; c < K; c++) {
            long v = L.slot_vid[p * K + c];
            double sl = 0.0, sp = H[v * C + vd];
            for (int j = 0; j < vd; j++) {
                sl += (double)grad[p * vd + j] * R[v * C + j];
                sp += H[v * C + j] * (double)vals[p * vd + j];
            }
            sl = (sl - go[p] * R[v * C + vd]) / zp[p];
            dw[c] = sl + sp;
        }
        double de[PO_MAX_PD + 1];
        for (int r = 0; r < K; r++)
            de[coord_of_rank[r]] = (dw[pd - r] - dw[(pd + 1 - r) % K]) / (double)K;
        /* elevation: e[pd] = -pd f[pd-1] sf[pd-1]; e[i] = e[i+1] - i f[i-1] sf[i-1]
         * + (i+2) f[i] sf[i]; e[0] = e[1] + 2 f[0] sf[0] (permutohedral.cu:166-173) */
        double gf[PO_MAX_PD] = {0};
        double carry = 0.0;   /* dL/de[i] accumulated down the recurrence */
        for (int i = 0; i <= pd; i++) {
            carry += de[i];
            if (i == 0) {
                gf[0] += 2.0 * sf[0] * carry;
            } else if (i < pd) {
                gf[i - 1] -= (double)i * sf[i - 1] * carry;
                gf[i] += (double)(i + 2) * sf[i] * carry;
            } else {
                gf[pd - 1] -= (double)pd * sf[pd - 1] * carry;
            }
        }
        for (int i = 0; i < pd; i++) grad_feat[(size_t)p * pd + i] = (float)gf[i];
    }
    long m = L.m;
    free(acc); free(x); free(y); free(hx); free(hy); free(zp); free(go); po_lattice_free(&L);
    return m;
}

/* ------------------------------------------------------------------------ */
/* brute-force dense Gaussian (O(n^2)), multi-threaded over output pixels    */

typedef struct {
    const float* feat; const float* vals; const float* wt;
    long n; int pd; int vd; long p0; long p1; double* out; int mode;
} po_bf_job;

/* mode 0: forward, out[p] = sum_q g_pq v_q / sum_q g_pq  (rows p in [p0,p1))
 * mode 1: value gradient with fixed normaliser wt: out[q] = sum_p g_pq wt_p v_p */
static void* po_bf_worker(void* arg) {
    po_bf_job* J = (po_bf_job*)arg;
    const int pd = J->pd, vd = J->vd;
    for (long p = J->p0; p < J->p1; p++) {
        const float* fp = J->feat + (size_t)p * pd;
        double acc[8] = {0};
        double ws = 0.0;
        for (long q = 0; q < J->n; q++) {
            const float* fq = J->feat + (size_t)q * pd;
            double d2 = 0.0;
            for (int i = 0; i < pd; i++) { double d = (double)fp[i] - (double)fq[i]; d2 += d * d; }
            double g = exp(-0.5 * d2);
            if (J->mode == 1) g *= (double)J->wt[q];
            ws += g;
            for (int j = 0; j < vd; j++) acc[j] += g * (double)J->vals[(size_t)q * vd + j];
        }
        for (int j = 0; j < vd; j++)
            J->out[(size_t)(p - J->p0) * vd + j] = (J->mode == 0) ? acc[j] / ws : acc[j];
    }
    return NULL;
}

/* Output rows [p0, p1) into out[(p1-p0)][vd], spread over nthreads threads. */
int po_brute_gaussian(const float* feat, const float* vals, const float* wt, long n, int pd,
                      int vd, long p0, long p1, int mode, int nthreads, double* out) {
    if (pd < 1 || vd < 1 || vd > 8 || p0 < 0 || p1 > n || p0 > p1) return PO_EINVAL;
    if (mode == 1 && !wt) return PO_EINVAL;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    po_bf_job jobs[256];
    long total = p1 - p0;
    for (int t = 0; t < nthreads; t++) {
        long a = p0 + total * t / nthreads, b = p0 + total * (t + 1) / nthreads;
        jobs[t] = (po_bf_job){feat, vals, wt, n, pd, vd, a, b, out + (size_t)(a - p0) * vd, mode};
        jobs[t].out = out + (size_t)(a - p0) * vd;
        if (pthread_create(&th[t], NULL, po_bf_worker, &jobs[t]) != 0) { po_bf_worker(&jobs[t]); th[t] = 0; }
    }
    for (int t = 0; t < nthreads; t++) if (th[t]) pthread_join(th[t], NULL);
    return PO_OK;
}
