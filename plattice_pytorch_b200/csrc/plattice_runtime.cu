// plattice_runtime.cu -- per-context host state and the device status ring
// (declared in plattice_runtime.h).
#include "plattice_runtime.h"

#include <string.h>

#include <deque>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace pl {

// ---------------------------------------------------------------- contexts

namespace {

// driver entry points, fetched through the runtime (no link against libcuda)
typedef int (*CtxGetCurrentFn)(void** ctx);                       // cuCtxGetCurrent
typedef int (*CtxGetIdFn)(void* ctx, unsigned long long* id);      // cuCtxGetId

struct DriverFns {
    CtxGetCurrentFn get_current = nullptr;
    CtxGetIdFn get_id = nullptr;
    cudaError_t err = cudaSuccess;
};

const DriverFns& driver_fns() {
    static DriverFns f = [] {
        DriverFns d;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        d.err = cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q);
        if (d.err == cudaSuccess && q == cudaDriverEntryPointSuccess) d.get_current = (CtxGetCurrentFn)p;
        p = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q);
        if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) d.get_id = (CtxGetIdFn)p;
        if (!d.get_current || !d.get_id) d.err = cudaErrorNotSupported;
        return d;
    }();
    return f;
}

}  // namespace

struct CtxState {
    unsigned long long id = 0;
    std::mutex mu;        // guards the maps
    std::unordered_map<const void*, int> once;
    std::unordered_map<const void*, void*> symbols;
};

namespace {
std::mutex g_ctx_mu;
std::vector<std::unique_ptr<CtxState>> g_ctx;   // never shrinks: ids are never reused
thread_local CtxState* t_last = nullptr;
}  // namespace

// Unique id of the calling thread's current context; when none is current,
// the current device's primary context is made current first (cudaSetDevice
// initialises it).
static cudaError_t current_ctx_id(unsigned long long* id) {
    const DriverFns& d = driver_fns();
    if (d.err != cudaSuccess) return d.err;
    void* ctx = nullptr;
    if (d.get_current(&ctx) != 0) return cudaErrorDeviceUninitialized;
    if (!ctx) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaSetDevice(dev);
        if (e != cudaSuccess) return e;
        if (d.get_current(&ctx) != 0 || !ctx) return cudaErrorDeviceUninitialized;
    }
    return d.get_id(ctx, id) == 0 ? cudaSuccess : cudaErrorDeviceUninitialized;
}

CtxState* ctx_state(cudaError_t* err) {
    unsigned long long id = 0;
    const cudaError_t e = current_ctx_id(&id);
    if (e != cudaSuccess) {
        if (err) *err = e;
        return nullptr;
    }
    if (err) *err = cudaSuccess;
    CtxState* last = t_last;
    if (last && last->id == id) return last;
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    for (auto& s : g_ctx) {
        if (s->id == id) {
            t_last = s.get();
            return s.get();
        }
    }
    g_ctx.emplace_back(new CtxState());
    g_ctx.back()->id = id;
    t_last = g_ctx.back().get();
    return t_last;
}

cudaError_t kernel_once(const void* fn, cudaError_t (*set_attr)(int*), int* value) {
    cudaError_t e;
    CtxState* c = ctx_state(&e);
    if (!c) return e;
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->once.find(fn);
    if (it != c->once.end()) {
        *value = it->second;
        return cudaSuccess;
    }
    int v = 0;
    e = set_attr(&v);
    if (e != cudaSuccess) return e;
    c->once.emplace(fn, v);
    *value = v;
    return cudaSuccess;
}

cudaError_t symbol_address(const void* symbol, void** addr) {
    cudaError_t e;
    CtxState* c = ctx_state(&e);
    if (!c) return e;
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->symbols.find(symbol);
    if (it != c->symbols.end()) {
        *addr = it->second;
        return cudaSuccess;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, symbol);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    c->symbols.emplace(symbol, p);
    *addr = p;
    return cudaSuccess;
}

// ---------------------------------------------------------------- status ring

namespace {

constexpr unsigned kRing = 4096;

struct Ring {
    std::mutex mu;
    unsigned long long* host = nullptr;   // pinned, mapped into every context
    unsigned long long* dev = nullptr;
    bool unavailable = false;             // the pinned allocation failed: calls are not tracked
    unsigned next = 1;                    // sequence 0 is never issued (slots start at 0)
    const char* name[kRing] = {};
    unsigned seq_of[kRing] = {};
    std::deque<unsigned> pending;         // issued, not yet seen finished, in issue order
    int fail_status = 0;
    const char* fail_name = nullptr;
    unsigned fail_seq = 0;
};

Ring& ring() {
    static Ring r;
    return r;
}

}  // namespace

StatusTicket status_ticket(const char* call) {
    Ring& r = ring();
    std::lock_guard<std::mutex> lk(r.mu);
    if (!r.host && !r.unavailable) {
        void* p = nullptr;
        if (cudaHostAlloc(&p, kRing * sizeof(unsigned long long), cudaHostAllocPortable | cudaHostAllocMapped) !=
            cudaSuccess) {
            cudaGetLastError();
            r.unavailable = true;
        } else {
            memset(p, 0, kRing * sizeof(unsigned long long));
            void* d = nullptr;
            if (cudaHostGetDevicePointer(&d, p, 0) != cudaSuccess || !d) {
                cudaGetLastError();
                cudaFreeHost(p);
                r.unavailable = true;
            } else {
                r.host = static_cast<unsigned long long*>(p);
                r.dev = static_cast<unsigned long long*>(d);
            }
        }
    }
    if (r.unavailable) return StatusTicket{nullptr, 0};
    unsigned seq = r.next++;
    if (seq == 0) seq = r.next++;
    const unsigned slot = seq % kRing;
    // a slot still pending after kRing later calls is dropped (never in practice:
    // the launch queue holds far fewer calls)
    while (!r.pending.empty() && r.seq_of[r.pending.front() % kRing] != r.pending.front()) r.pending.pop_front();
    if (!r.pending.empty() && r.pending.front() % kRing == slot) r.pending.pop_front();
    r.seq_of[slot] = seq;
    r.name[slot] = call;
    reinterpret_cast<volatile unsigned long long*>(r.host)[slot] = 0ull;
    r.pending.push_back(seq);
    return StatusTicket{r.dev + slot, seq};
}

int status_poll(const char** name, unsigned* seq) {
    Ring& r = ring();
    std::lock_guard<std::mutex> lk(r.mu);
    if (r.host) {
        while (!r.pending.empty()) {
            const unsigned s = r.pending.front();
            const unsigned slot = s % kRing;
            if (r.seq_of[slot] != s) {   // dropped
                r.pending.pop_front();
                continue;
            }
            const unsigned long long v = reinterpret_cast<volatile unsigned long long*>(r.host)[slot];
            if ((unsigned)(v >> 32) != s) break;   // its kernels have not finished yet
            r.pending.pop_front();
            const int st = (int)(unsigned)(v & 0xffffffffull);
            if (st != 0 && r.fail_status == 0) {
                r.fail_status = st;
                r.fail_name = r.name[slot];
                r.fail_seq = s;
            }
        }
    }
    const int st = r.fail_status;
    if (st) {
        if (name) *name = r.fail_name;
        if (seq) *seq = r.fail_seq;
        r.fail_status = 0;
    }
    return st;
}

}  // namespace pl
