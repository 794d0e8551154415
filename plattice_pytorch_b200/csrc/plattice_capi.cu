// plattice_capi.cu -- the C ABI declared in include/plattice.h: argument
// checks, buffer sizing, run-time pd dispatch to the per-pd instantiations.
#include <cuda_runtime.h>
#include <limits.h>
#include <stdio.h>

#include <stdlib.h>
#include <string.h>

#include <initializer_list>
#include <mutex>
#include <vector>

#include "../../include/plattice.h"
#include "plattice_impl.cuh"
#include "plattice_runtime.h"

namespace pl {
#define PL_DECLARE_PD(N)                                                                    \
    extern template cudaError_t run_forward<N>(const CallArgs&);                             \
    extern template cudaError_t run_backward<N>(const CallArgs&);                            \
    extern template cudaError_t run_filter<N>(const CallArgs&);                              \
    extern template cudaError_t run_feature_grad<N>(const CallArgs&);                        \
    extern template cudaError_t run_prepare<N>(const CallArgs&);                             \
    extern template cudaError_t run_export_keys<N>(const void*, const void*, const PlLayout&, \
                                                   int16_t*, int, cudaStream_t);
PL_DECLARE_PD(1) PL_DECLARE_PD(2) PL_DECLARE_PD(3) PL_DECLARE_PD(4)
PL_DECLARE_PD(5) PL_DECLARE_PD(6) PL_DECLARE_PD(7) PL_DECLARE_PD(8)
PL_DECLARE_PD(9) PL_DECLARE_PD(10) PL_DECLARE_PD(11) PL_DECLARE_PD(12)
PL_DECLARE_PD(13) PL_DECLARE_PD(14) PL_DECLARE_PD(15) PL_DECLARE_PD(16)
}  // namespace pl

static int g_cap_override_log2 = 0;
static int g_filter_min_log2 = 0;
static int g_blur_half = 0;     // bfloat16 rows in the streaming blur passes
static int g_blur_stream = 0;   // test support: streaming blur passes for every lattice

static int blur_flags() { return (g_blur_half ? pl::kBlurHalf : 0) | (g_blur_stream ? pl::kBlurStream : 0); }

// ---------------------------------------------------------------- profiling

namespace {
struct ProfRec {
    int stage;
    cudaEvent_t begin, end;
};
std::mutex g_prof_mu;
int g_prof_mode = 0;
std::vector<cudaEvent_t> g_prof_pool;
std::vector<ProfRec> g_prof_done;
ProfRec g_prof_open[pl::STAGE_COUNT];

cudaEvent_t prof_event() {
    if (!g_prof_pool.empty()) {
        cudaEvent_t e = g_prof_pool.back();
        g_prof_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}
}  // namespace

namespace pl {
int prof_mode() { return g_prof_mode; }

void prof_mark(int stage, cudaStream_t s, bool begin) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_mode || stage < 0 || stage >= STAGE_COUNT) return;
    cudaEvent_t e = prof_event();
    if (!e) return;
    cudaEventRecord(e, s);
    if (begin) {
        g_prof_open[stage].stage = stage;
        g_prof_open[stage].begin = e;
    } else {
        ProfRec r = g_prof_open[stage];
        r.end = e;
        if (r.begin) g_prof_done.push_back(r);
        g_prof_open[stage].begin = nullptr;
    }
}
}  // namespace pl

#define PL_PD_SWITCH(PD, CALL)          \
    switch (PD) {                       \
        case 1: return CALL(1);         \
        case 2: return CALL(2);         \
        case 3: return CALL(3);         \
        case 4: return CALL(4);         \
        case 5: return CALL(5);         \
        case 6: return CALL(6);         \
        case 7: return CALL(7);         \
        case 8: return CALL(8);         \
        case 9: return CALL(9);         \
        case 10: return CALL(10);       \
        case 11: return CALL(11);       \
        case 12: return CALL(12);       \
        case 13: return CALL(13);       \
        case 14: return CALL(14);       \
        case 15: return CALL(15);       \
        case 16: return CALL(16);       \
        default: return cudaErrorInvalidValue; \
    }

static cudaError_t dispatch_forward(const pl::CallArgs& a) {
#define PL_FWD(N) pl::run_forward<N>(a)
    PL_PD_SWITCH(a.lay.pd, PL_FWD)
#undef PL_FWD
}

static cudaError_t dispatch_filter(const pl::CallArgs& a) {
#define PL_FIL(N) pl::run_filter<N>(a)
    PL_PD_SWITCH(a.lay.pd, PL_FIL)
#undef PL_FIL
}

static cudaError_t dispatch_feature_grad(const pl::CallArgs& a) {
#define PL_FG(N) pl::run_feature_grad<N>(a)
    PL_PD_SWITCH(a.lay.pd, PL_FG)
#undef PL_FG
}

static cudaError_t dispatch_backward(const pl::CallArgs& a) {
#define PL_BWD(N) pl::run_backward<N>(a)
    PL_PD_SWITCH(a.lay.pd, PL_BWD)
#undef PL_BWD
}

static cudaError_t dispatch_keys(const void* lat, const void* scr, const PlLayout& lay, int16_t* out,
                                 int max_keys, cudaStream_t s) {
#define PL_KEYS(N) pl::run_export_keys<N>(lat, scr, lay, out, max_keys, s)
    PL_PD_SWITCH(lay.pd, PL_KEYS)
#undef PL_KEYS
}

static int sm_count_current() {
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

// ---------------------------------------------------------------- call graphs

// A call whose launch sequence has been seen before with exactly the same
// buffers, sizes and settings is replayed as one CUDA graph: the second such
// call captures its launches (on a private stream of the context, in
// thread-local capture mode) into a graph, and every later one launches that
// graph on the caller's stream after pointing the status-reporting kernel at
// the call's status-ring slot.  One graph launch replaces the seven launches
// of a forward (three of a backward or of a kept-lattice filter) on the host.  Graphs are kept per CUDA
// context in a small least-recently-used cache; calls that profile, calls on
// a stream the caller is capturing, and the no-allocation entry point
// (instantiating a graph allocates) run directly.
namespace {

struct GraphKey {
    int kind;
    const void* p[8];
    size_t n[2];
    int v[12];
    bool operator==(const GraphKey& o) const {
        if (kind != o.kind || n[0] != o.n[0] || n[1] != o.n[1]) return false;
        for (int i = 0; i < 8; ++i)
            if (p[i] != o.p[i]) return false;
        for (int i = 0; i < 12; ++i)
            if (v[i] != o.v[i]) return false;
        return true;
    }
};

struct GraphEntry {
    GraphKey key;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    pl::StatusNode sn;
    unsigned long long used = 0;
};

struct GraphCache {
    cudaStream_t capture = nullptr;
    std::vector<GraphEntry*> entries;
    std::vector<GraphKey> seen;   // keys called once, most recent last
    unsigned long long clock = 0;
};

std::mutex g_graph_mu;
std::vector<std::pair<pl::CtxState*, GraphCache*>> g_graph_caches;
int g_graph_cap = -1;   // entries per context; 0 = off; -1: read PLATTICE_GRAPHS on first use
long long g_graph_captures = 0, g_graph_replays = 0;

int graph_capacity() {
    if (g_graph_cap < 0) {
        const char* e = getenv("PLATTICE_GRAPHS");
        g_graph_cap = (e && e[0] == '0' && e[1] == '\0') ? 0 : 16;
    }
    return g_graph_cap;
}

GraphCache* graph_cache() {
    cudaError_t e;
    pl::CtxState* c = pl::ctx_state(&e);
    if (!c) return nullptr;
    for (auto& pc : g_graph_caches)
        if (pc.first == c) return pc.second;
    g_graph_caches.emplace_back(c, new GraphCache());
    return g_graph_caches.back().second;
}

void graph_free(GraphEntry* g) {
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

}  // namespace

// Runs `dispatch(a)` directly, or as a captured graph (see above).
static cudaError_t run_call(const GraphKey& key, pl::CallArgs& a, cudaError_t (*dispatch)(const pl::CallArgs&)) {
    const int cap = graph_capacity();
    if (cap <= 0 || pl::prof_enabled()) return dispatch(a);
    // a caller that captures its own stream (e.g. into a CUDA graph of its
    // own) gets the launches themselves in its capture
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(a.stream, &cs) != cudaSuccess) {
        cudaGetLastError();
        return dispatch(a);
    }
    if (cs != cudaStreamCaptureStatusNone) return dispatch(a);
    std::lock_guard<std::mutex> lk(g_graph_mu);
    GraphCache* gc = graph_cache();
    if (!gc) return dispatch(a);
    ++gc->clock;
    for (GraphEntry* g : gc->entries) {
        if (g->key == key) {
            g->used = gc->clock;
            cudaError_t e = g->sn.retarget(g->exec, a.st.slot, a.st.seq);
            if (e == cudaSuccess) e = cudaGraphLaunch(g->exec, a.stream);
            if (e == cudaSuccess) ++g_graph_replays;
            return e;
        }
    }
    bool again = false;
    for (size_t i = 0; i < gc->seen.size(); ++i) {
        if (gc->seen[i] == key) {
            again = true;
            gc->seen.erase(gc->seen.begin() + (long)i);
            break;
        }
    }
    if (!again) {   // first sighting: run directly, remember the key
        gc->seen.push_back(key);
        if (gc->seen.size() > 32) gc->seen.erase(gc->seen.begin());
        return dispatch(a);
    }
    // second sighting: capture, instantiate, launch; anything that fails on
    // the way (e.g. while another thread captures in global mode) leaves the
    // call to run directly
    cudaError_t e = cudaSuccess;
    if (!gc->capture) e = cudaStreamCreateWithFlags(&gc->capture, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        gc->capture = nullptr;
        cudaGetLastError();
        return dispatch(a);
    }
    GraphEntry* g = new GraphEntry();
    g->key = key;
    pl::CallArgs c = a;
    c.stream = gc->capture;
    c.status_node = &g->sn;
    e = cudaStreamBeginCapture(gc->capture, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        delete g;
        cudaGetLastError();
        return dispatch(a);
    }
    const cudaError_t ed = dispatch(c);
    const cudaError_t ee = cudaStreamEndCapture(gc->capture, &g->graph);
    if (ed == cudaSuccess && ee == cudaSuccess && g->graph && g->sn.retarget)
        e = cudaGraphInstantiate(&g->exec, g->graph, 0);
    else
        e = ed != cudaSuccess ? ed : (ee != cudaSuccess ? ee : cudaErrorStreamCaptureInvalidated);
    if (e != cudaSuccess) {   // capture did not produce a usable graph: run directly
        cudaGetLastError();
        graph_free(g);
        return dispatch(a);
    }
    if ((int)gc->entries.size() >= cap) {   // evict the least recently used graph
        size_t lru = 0;
        for (size_t i = 1; i < gc->entries.size(); ++i)
            if (gc->entries[i]->used < gc->entries[lru]->used) lru = i;
        graph_free(gc->entries[lru]);
        gc->entries.erase(gc->entries.begin() + (long)lru);
    }
    g->used = gc->clock;
    gc->entries.push_back(g);
    ++g_graph_captures;
    e = g->sn.retarget(g->exec, a.st.slot, a.st.seq);
    if (e == cudaSuccess) e = cudaGraphLaunch(g->exec, a.stream);
    return e;
}

static GraphKey call_key(int kind, const pl::CallArgs& a, std::initializer_list<const void*> ptrs, size_t n0, size_t n1) {
    GraphKey k;
    memset(&k, 0, sizeof(k));
    k.kind = kind;
    int i = 0;
    for (const void* q : ptrs) k.p[i++] = q;
    k.n[0] = n0;
    k.n[1] = n1;
    k.v[0] = a.lay.b; k.v[1] = a.lay.h; k.v[2] = a.lay.w; k.v[3] = a.lay.pd; k.v[4] = a.lay.vd;
    k.v[5] = a.lattice_state; k.v[6] = a.cap_override_log2; k.v[7] = a.filter_min_log2; k.v[8] = a.blur_flags;
    k.v[9] = a.sm_count;
    return k;
}

static cudaError_t dispatch_prepare(const pl::CallArgs& a) {
#define PL_PREP(N) pl::run_prepare<N>(a)
    PL_PD_SWITCH(a.lay.pd, PL_PREP)
#undef PL_PREP
}

// dimension checks of permuto.cpp:37-40 plus the index range of this build
// (32-bit vertex ids and slot indices) for b images
static int check_dims_b(int b, int h, int w, int pd, int vd) {
    if (pd < 1 || pd > PL_MAX_PD || vd < 1 || vd > PL_MAX_VD) return PLATTICE_ERR_INVALID;
    if (b < 0 || h < 0 || w < 0) return PLATTICE_ERR_INVALID;
    if (b == 0 || h == 0 || w == 0) return PLATTICE_OK;
    PlLayout L;
    pl_layout_batch(&L, b, h, w, pd, vd);
    if (L.slots > (1ll << 29)) return PLATTICE_ERR_INVALID;
    if (L.tiles_y > 65535 || b > 65535) return PLATTICE_ERR_INVALID;   // per-tile grids (x, y, image)
    return PLATTICE_OK;
}

static int check_dims(int h, int w, int pd, int vd) { return check_dims_b(1, h, w, pd, vd); }

static thread_local char g_last_error[256] = "";

static int cuda_status(cudaError_t e, const char* where = "") {
    if (e == cudaSuccess) return PLATTICE_OK;
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
    if (e == cudaErrorInvalidValue) return PLATTICE_ERR_INVALID;
    return PLATTICE_ERR_CUDA;
}

static const char* status_bits_text(int st) {
    if (st & PL_ST_TABLE_FULL) return "hash table full";
    if (st & PL_ST_SPIN) return "a bounded wait gave up";
    if (st & PL_ST_SMEM_PROBE) return "tile table exhausted";
    return "device failure";
}

// Device failures of earlier calls: their last kernel left the status word in
// the host-mapped ring; the first call that finds a failure there returns
// PLATTICE_ERR_DEVICE (without enqueueing its own work) and names it.
static int poll_earlier(const char* call) {
    const char* name = nullptr;
    unsigned seq = 0;
    const int st = pl::status_poll(&name, &seq);
    if (st == 0) return PLATTICE_OK;
    snprintf(g_last_error, sizeof(g_last_error),
             "%s: an earlier call (%s, call #%u) reported device status bits %#x (%s); its outputs are invalid",
             call, name ? name : "?", seq, st, status_bits_text(st));
    return PLATTICE_ERR_DEVICE;
}

static void common_args(pl::CallArgs& a, void* stream, bool track, const char* call) {
    a.stream = static_cast<cudaStream_t>(stream);
    a.sm_count = sm_count_current();
    a.cap_override_log2 = g_cap_override_log2;
    a.filter_min_log2 = g_filter_min_log2;
    a.blur_flags = blur_flags();
    a.st = track ? pl::status_ticket(call) : pl::StatusTicket{nullptr, 0};
}

namespace pl {

// Forward of b images (b = 1: plattice_forward).  track = false: no status
// ticket (the no-allocation entry point, which allocates nothing).
int forward_images(float* weight_out, float* out, const float* values, const float* features, void* lattice,
                   size_t lattice_bytes, void* scratch, size_t scratch_bytes, int b, int pd, int vd, int w,
                   int h, void* stream, bool track, const char* call) {
    int rc = check_dims_b(b, h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (b == 0 || h == 0 || w == 0) return PLATTICE_OK;
    if (!weight_out || !out || !values || !features || !lattice || !scratch) return PLATTICE_ERR_INVALID;
    CallArgs a = {};
    pl_layout_batch(&a.lay, b, h, w, pd, vd);
    if (lattice_bytes < a.lay.lattice_bytes || scratch_bytes < a.lay.scratch_bytes) return PLATTICE_ERR_WORKSPACE;
    rc = poll_earlier(call);
    if (rc != PLATTICE_OK) return rc;
    a.features = features; a.values = values; a.weight_in = nullptr;
    a.out = out; a.wout = weight_out;
    a.lattice = lattice; a.scratch = scratch;
    rows_in_scratch(a, scratch);
    a.lattice_state = 0;
    common_args(a, stream, track, call);
    if (!track) return cuda_status(dispatch_forward(a), call);   // allocates nothing: no graph
    const GraphKey key = call_key(0, a, {weight_out, out, values, features, lattice, scratch}, lattice_bytes,
                                  scratch_bytes);
    return cuda_status(run_call(key, a, dispatch_forward), call);
}

}  // namespace pl

static int backward_images(float* grad_values_out, const float* grad, const float* weight_in,
                           const float* features, void* lattice, size_t lattice_bytes, int lattice_state,
                           void* scratch, size_t scratch_bytes, int b, int pd, int vd, int w, int h, void* stream,
                           const char* call) {
    int rc = check_dims_b(b, h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (b == 0 || h == 0 || w == 0) return PLATTICE_OK;
    if (lattice_state < 0 || lattice_state > 2) return PLATTICE_ERR_INVALID;
    if (!grad_values_out || !grad || !weight_in || !lattice || !scratch) return PLATTICE_ERR_INVALID;
    if (lattice_state == 0 && !features) return PLATTICE_ERR_INVALID;
    pl::CallArgs a = {};
    pl_layout_batch(&a.lay, b, h, w, pd, vd);
    if (lattice_bytes < a.lay.lattice_bytes) return PLATTICE_ERR_WORKSPACE;
    if (scratch_bytes < (lattice_state == 0 ? a.lay.scratch_bytes : a.lay.reuse_bytes)) return PLATTICE_ERR_WORKSPACE;
    rc = poll_earlier(call);
    if (rc != PLATTICE_OK) return rc;
    a.features = features; a.values = grad; a.weight_in = weight_in;
    a.out = grad_values_out; a.wout = nullptr;
    a.lattice = lattice;
    a.scratch = lattice_state == 0 ? scratch : nullptr;
    rows_in_scratch(a, scratch);
    a.v0 = pl::lattice_vb0(a);   // the splat target; the scratch's v1 is its ping-pong partner
    a.lattice_state = lattice_state;
    common_args(a, stream, true, call);
    const GraphKey key = call_key(1, a, {grad_values_out, grad, weight_in, features, lattice, scratch},
                                  lattice_bytes, scratch_bytes);
    return cuda_status(run_call(key, a, dispatch_backward), call);
}

extern "C" {

int plattice_abi_version(void) { return PLATTICE_ABI_VERSION; }

const char* plattice_last_error_detail(void) { return g_last_error; }

const char* plattice_error_string(int status) {
    switch (status) {
        case PLATTICE_OK: return "ok";
        case PLATTICE_ERR_INVALID: return "invalid argument (pd must be in [1, 16], vd in [1, 8], image within size limits, pointers non-null)";
        case PLATTICE_ERR_WORKSPACE: return "lattice or scratch buffer smaller than plattice_workspace_sizes requires";
        case PLATTICE_ERR_CUDA: return "CUDA runtime error";
        case PLATTICE_ERR_DEVICE: return "device-side failure reported in the lattice status word";
        default: return "unknown status";
    }
}

int plattice_batch_workspace_sizes(int b, int h, int w, int pd, int vd, size_t* lattice_bytes,
                                   size_t* scratch_bytes) {
    const int rc = check_dims_b(b, h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    size_t lb = 256, sb = 256;
    if (b > 0 && h > 0 && w > 0) {
        PlLayout L;
        pl_layout_batch(&L, b, h, w, pd, vd);
        lb = L.lattice_bytes;
        sb = L.scratch_bytes;
    }
    if (lattice_bytes) *lattice_bytes = lb;
    if (scratch_bytes) *scratch_bytes = sb;
    return PLATTICE_OK;
}

int plattice_workspace_sizes(int h, int w, int pd, int vd, size_t* lattice_bytes, size_t* scratch_bytes) {
    return plattice_batch_workspace_sizes(1, h, w, pd, vd, lattice_bytes, scratch_bytes);
}

int plattice_reuse_scratch_size(int b, int h, int w, int pd, int vd, size_t* bytes) {
    const int rc = check_dims_b(b, h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (!bytes) return PLATTICE_ERR_INVALID;
    *bytes = 256;
    if (b > 0 && h > 0 && w > 0) {
        PlLayout L;
        pl_layout_batch(&L, b, h, w, pd, vd);
        *bytes = L.reuse_bytes;
    }
    return PLATTICE_OK;
}

int plattice_forward(float* weight_out, float* out, const float* values, const float* features,
                     void* lattice, size_t lattice_bytes, void* scratch, size_t scratch_bytes, int pd,
                     int vd, int w, int h, void* stream) {
    return pl::forward_images(weight_out, out, values, features, lattice, lattice_bytes, scratch, scratch_bytes, 1,
                              pd, vd, w, h, stream, true, "plattice_forward");
}

int plattice_backward(float* grad_values_out, const float* grad, const float* weight_in, const float* features,
                      void* lattice, size_t lattice_bytes, int lattice_state, void* scratch, size_t scratch_bytes,
                      int pd, int vd, int w, int h, void* stream) {
    return backward_images(grad_values_out, grad, weight_in, features, lattice, lattice_bytes, lattice_state,
                           scratch, scratch_bytes, 1, pd, vd, w, h, stream, "plattice_backward");
}

int plattice_forward_batch(float* weight_out, float* out, const float* values, const float* features,
                           void* lattice, size_t lattice_bytes, void* scratch, size_t scratch_bytes, int b,
                           int pd, int vd, int w, int h, void* stream) {
    return pl::forward_images(weight_out, out, values, features, lattice, lattice_bytes, scratch, scratch_bytes, b,
                              pd, vd, w, h, stream, true, "plattice_forward_batch");
}

int plattice_backward_batch(float* grad_values_out, const float* grad, const float* weight_in, const float* features,
                            void* lattice, size_t lattice_bytes, int lattice_state, void* scratch,
                            size_t scratch_bytes, int b, int pd, int vd, int w, int h, void* stream) {
    return backward_images(grad_values_out, grad, weight_in, features, lattice, lattice_bytes, lattice_state,
                           scratch, scratch_bytes, b, pd, vd, w, h, stream, "plattice_backward_batch");
}

// ---------------------------------------------------------------- kept lattice

int plattice_filter_workspace_size(int h, int w, int pd, int vd, size_t* bytes) {
    const int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (!bytes) return PLATTICE_ERR_INVALID;
    *bytes = 256;
    if (h > 0 && w > 0) {
        PlLayout L;
        pl_layout(&L, h, w, pd, vd);
        *bytes = L.rows_bytes;   // both value-row buffers and the blur's bookkeeping
    }
    return PLATTICE_OK;
}

// The checks shared by the two kept-lattice calls; fills the layout and the
// value rows.
static int kept_lattice_args(pl::CallArgs& a, size_t lattice_bytes, void* ws, size_t ws_bytes, int pd, int vd,
                             int w, int h, void* stream, const char* call) {
    pl_layout(&a.lay, h, w, pd, vd);
    // a filter reads the arrays before vb0, whose size is the only part of the
    // lattice that depends on vd: a lattice built with any vd serves
    if (lattice_bytes < a.lay.off_vb0) return PLATTICE_ERR_WORKSPACE;
    if (ws_bytes < a.lay.rows_bytes) return PLATTICE_ERR_WORKSPACE;
    const int rc = poll_earlier(call);
    if (rc != PLATTICE_OK) return rc;
    rows_in_scratch(a, ws);
    common_args(a, stream, true, call);
    return PLATTICE_OK;
}

int plattice_filter(float* weight_out, float* out, const float* values, void* lattice, size_t lattice_bytes,
                    void* values_ws, size_t values_ws_bytes, int pd, int vd, int w, int h, void* stream) {
    int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (h == 0 || w == 0) return PLATTICE_OK;
    if (!weight_out || !out || !values || !lattice || !values_ws) return PLATTICE_ERR_INVALID;
    pl::CallArgs a = {};
    rc = kept_lattice_args(a, lattice_bytes, values_ws, values_ws_bytes, pd, vd, w, h, stream, "plattice_filter");
    if (rc != PLATTICE_OK) return rc;
    a.values = values;
    a.out = out;
    a.wout = weight_out;
    a.lattice = lattice;
    const GraphKey key = call_key(2, a, {weight_out, out, values, lattice, values_ws}, lattice_bytes, values_ws_bytes);
    return cuda_status(run_call(key, a, dispatch_filter), "plattice_filter");
}

int plattice_filter_backward(float* grad_values_out, const float* grad, const float* weight_in, void* lattice,
                             size_t lattice_bytes, void* values_ws, size_t values_ws_bytes, int pd, int vd, int w,
                             int h, void* stream) {
    int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (h == 0 || w == 0) return PLATTICE_OK;
    if (!grad_values_out || !grad || !weight_in || !lattice || !values_ws) return PLATTICE_ERR_INVALID;
    pl::CallArgs a = {};
    rc = kept_lattice_args(a, lattice_bytes, values_ws, values_ws_bytes, pd, vd, w, h, stream,
                           "plattice_filter_backward");
    if (rc != PLATTICE_OK) return rc;
    a.values = grad;
    a.weight_in = weight_in;
    a.out = grad_values_out;
    a.lattice = lattice;
    a.lattice_state = 2;   // kept lattice: zero the value rows, no rebuild
    const GraphKey key = call_key(3, a, {grad_values_out, grad, weight_in, lattice, values_ws}, lattice_bytes,
                                  values_ws_bytes);
    return cuda_status(run_call(key, a, dispatch_backward), "plattice_filter_backward");
}

// ---------------------------------------------------------------- feature gradient

// Workspace: two result flags, four lattice row buffers (R and H, ping-pong)
// of slots x pad(vd+1) floats, the blur's bookkeeping bytes, and the
// per-pixel (G, -G.out) rows.
struct FgradWs {
    size_t flags, r0, r1, h0, h1, bst, ev, total;
};

static FgradWs fgrad_ws(const PlLayout& L) {
    FgradWs W;
    const size_t rows = pl_align((size_t)L.slots * (size_t)L.CPf * 4);
    W.flags = 0;
    W.r0 = 256;
    W.r1 = W.r0 + rows;
    W.h0 = W.r1 + rows;
    W.h1 = W.h0 + rows;
    W.bst = W.h1 + rows;
    W.ev = W.bst + pl_align(2 * (size_t)L.slots);
    W.total = W.ev + pl_align((size_t)L.h * L.w * (size_t)(L.vd + 1) * 4);
    return W;
}

int plattice_feature_grad_workspace_size(int h, int w, int pd, int vd, size_t* bytes) {
    const int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (!bytes) return PLATTICE_ERR_INVALID;
    *bytes = 256;
    if (h > 0 && w > 0) {
        PlLayout L;
        pl_layout(&L, h, w, pd, vd);
        *bytes = fgrad_ws(L).total;
    }
    return PLATTICE_OK;
}

int plattice_feature_grad(float* grad_features_out, const float* grad, const float* out, const float* weight,
                          const float* values, const float* features, void* lattice, size_t lattice_bytes,
                          void* ws, size_t ws_bytes, int pd, int vd, int w, int h, void* stream) {
    int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (h == 0 || w == 0) return PLATTICE_OK;
    if (!grad_features_out || !grad || !out || !weight || !values || !features || !lattice || !ws)
        return PLATTICE_ERR_INVALID;
    pl::CallArgs a = {};
    pl_layout(&a.lay, h, w, pd, vd);
    if (lattice_bytes < a.lay.off_vb0) return PLATTICE_ERR_WORKSPACE;
    const FgradWs W = fgrad_ws(a.lay);
    if (ws_bytes < W.total) return PLATTICE_ERR_WORKSPACE;
    rc = poll_earlier("plattice_feature_grad");
    if (rc != PLATTICE_OK) return rc;
    char* b = static_cast<char*>(ws);
    a.flags = reinterpret_cast<int*>(b + W.flags);
    a.v0 = reinterpret_cast<float*>(b + W.r0);
    a.v1 = reinterpret_cast<float*>(b + W.r1);
    a.hbuf0 = reinterpret_cast<float*>(b + W.h0);
    a.hbuf1 = reinterpret_cast<float*>(b + W.h1);
    a.bstate = reinterpret_cast<uint8_t*>(b + W.bst);
    a.evec = reinterpret_cast<float*>(b + W.ev);
    a.features = features;
    a.values = values;
    a.weight_in = weight;
    a.grad_in = grad;
    a.out_in = out;
    a.out = grad_features_out;
    a.lattice = lattice;
    common_args(a, stream, true, "plattice_feature_grad");
    return cuda_status(dispatch_feature_grad(a), "plattice_feature_grad");
}

// ---------------------------------------------------------------- status, set-up, test support

int plattice_poll_status(void) { return poll_earlier("plattice_poll_status"); }

int plattice_prepare(int pd, int vd) {
    const int rc = check_dims(1, 1, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    pl::CallArgs a = {};
    pl_layout(&a.lay, 1, 1, pd, vd);
    return cuda_status(dispatch_prepare(a), "plattice_prepare");
}

int plattice_lattice_info(const void* lattice, int* status, int* m, int* u_total, int* cap_log2, void* stream) {
    if (!lattice) return PLATTICE_ERR_INVALID;
    LatticeHeader hh;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&hh, lattice, sizeof(hh), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e, "plattice_lattice_info");
    if (status) *status = hh.status;
    if (m) *m = hh.m;
    if (u_total) *u_total = hh.u_total;
    if (cap_log2) *cap_log2 = hh.cap_log2;
    return hh.status ? PLATTICE_ERR_DEVICE : PLATTICE_OK;
}

int plattice_vertex_keys(const void* lattice, const void* scratch, int pd, int vd, int w, int h,
                         int16_t* keys_dev, int max_keys, int* m, void* stream) {
    int rc = check_dims(h, w, pd, vd);
    if (rc != PLATTICE_OK) return rc;
    if (!lattice || !scratch || (!keys_dev && max_keys > 0)) return PLATTICE_ERR_INVALID;
    if (h == 0 || w == 0) { if (m) *m = 0; return PLATTICE_OK; }
    PlLayout L;
    pl_layout(&L, h, w, pd, vd);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (max_keys > 0) {
        cudaError_t e = dispatch_keys(lattice, scratch, L, keys_dev, max_keys, s);
        if (e != cudaSuccess) return cuda_status(e, "plattice_vertex_keys");
    }
    return plattice_lattice_info(lattice, nullptr, m, nullptr, nullptr, stream);
}

void plattice_profile_enable(int on) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_mode = (on == 1 || on == 2) ? on : 0;
}

int plattice_profile_read(double* ms_total, int* launches, int n_stages) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (int i = 0; i < n_stages; ++i) {
        if (ms_total) ms_total[i] = 0.0;
        if (launches) launches[i] = 0;
    }
    int rc = PLATTICE_OK;
    for (const ProfRec& r : g_prof_done) {
        float ms = 0.0f;
        if (cudaEventSynchronize(r.end) != cudaSuccess || cudaEventElapsedTime(&ms, r.begin, r.end) != cudaSuccess)
            rc = PLATTICE_ERR_CUDA;
        else if (r.stage < n_stages) {
            if (ms_total) ms_total[r.stage] += ms;
            if (launches) launches[r.stage] += 1;
        }
        g_prof_pool.push_back(r.begin);
        g_prof_pool.push_back(r.end);
    }
    g_prof_done.clear();
    return rc;
}

const char* plattice_profile_stage_name(int stage) {
    static const char* names[pl::STAGE_COUNT] = {
        "tile_build", "clear", "insert", "neighbors", "blur_fwd", "slice_fwd",
        "zero", "splat_bwd", "blur_bwd", "slice_bwd", "splat_fwd",
        "build", "filter_fwd", "filter_bwd"};
    return (stage >= 0 && stage < pl::STAGE_COUNT) ? names[stage] : "";
}

void plattice_debug_set_table_cap_log2(int log2_cells) {
    g_cap_override_log2 = (log2_cells > 0 && log2_cells < 31) ? log2_cells : 0;
}

void plattice_debug_set_miss_filter_log2(int log2_cells) {
    g_filter_min_log2 = (log2_cells > 0 && log2_cells < 31) ? log2_cells : 0;
}

int plattice_set_lattice_precision(int bits) {
    if (bits != 32 && bits != 16) return PLATTICE_ERR_INVALID;
    g_blur_half = bits == 16;
    return PLATTICE_OK;
}

int plattice_get_lattice_precision(void) { return g_blur_half ? 16 : 32; }

void plattice_debug_set_blur_streaming(int on) { g_blur_stream = on ? 1 : 0; }


int plattice_set_graph_cache(int entries) {
    if (entries < 0) return PLATTICE_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_graph_mu);
    g_graph_cap = entries;
    for (auto& pc : g_graph_caches) {   // graphs of every context are released
        for (GraphEntry* g : pc.second->entries) graph_free(g);
        pc.second->entries.clear();
        pc.second->seen.clear();
    }
    return PLATTICE_OK;
}

void plattice_graph_cache_stats(long long* captures, long long* replays) {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    if (captures) *captures = g_graph_captures;
    if (replays) *replays = g_graph_replays;
}

}  // extern "C"
