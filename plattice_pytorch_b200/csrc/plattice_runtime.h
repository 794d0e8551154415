// plattice_runtime.h -- host-side state of the library that belongs to a CUDA
// context: one-time kernel attribute settings and occupancy figures, the
// device address of the no-allocation entry point's fixed array; and the
// ring of per-call device status words that reports device-side failures
// (table full, a bounded wait that gave up) on a later call without
// synchronising.
//
// Everything cached is keyed by the calling thread's current CUDA context,
// identified by its unique id (cuCtxGetId: never reused, also not after
// cudaDeviceReset re-creates the primary context), so that a caller running
// in its own context (cuCtxCreate) or after a device reset gets state created
// in that context, never another context's handles or addresses.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace pl {

struct CtxState;

// The state of the current context (created on first use).  Returns nullptr
// and sets *err when the context cannot be determined.
CtxState* ctx_state(cudaError_t* err);

// Runs set_attr once per context for the kernel `fn` (a kernel attribute
// such as the dynamic shared-memory limit) and caches an int result (e.g. the
// resident CTAs per SM it implies).  Returns the cached value in *value.
cudaError_t kernel_once(const void* fn, cudaError_t (*set_attr)(int* value), int* value);

// Device address of a __device__ symbol in the current context (looked up
// with cudaGetSymbolAddress once per context and symbol).
cudaError_t symbol_address(const void* symbol, void** addr);

// Status ring.  A call that enqueues work takes a ticket: a slot of pinned,
// mapped host memory and a sequence number.  The call's last kernel stores
// (sequence << 32) | status word there; status_poll, run at the start of every
// call, reads the slots of earlier calls whose kernels have finished and
// returns the first non-zero status it finds (once), with the call's name.
struct StatusTicket {
    unsigned long long* slot;   // device-visible address (nullptr: not tracked)
    unsigned seq;
};
StatusTicket status_ticket(const char* call);
// 0 when no finished call reported a failure; else its status bits, with the
// call's name and sequence number in name/seq.
int status_poll(const char** name, unsigned* seq);

}  // namespace pl
