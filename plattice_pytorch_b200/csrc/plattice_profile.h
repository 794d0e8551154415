// plattice_profile.h -- optional per-kernel timing with CUDA events recorded
// on the launching stream around every launch (off by default; switched on
// by plattice_profile_enable, read by plattice_profile_read).
#pragma once
#include <cuda_runtime.h>

namespace pl {

enum Stage {
    STAGE_TILE_BUILD = 0,  // build: lattice embedding + tile dedup + staging
    STAGE_CLEAR,           // build: hash table clear
    STAGE_INSERT,          // build: global insert + vertex id compaction
    STAGE_NEIGHBORS,       // build: blur neighbour resolution
    STAGE_BLUR_FWD,        // fwd: the blur passes
    STAGE_SLICE_FWD,       // fwd: normalised slice
    STAGE_ZERO,            // bwd: re-zero of the value buffer (repeated backward)
    STAGE_SPLAT_BWD,       // bwd: splat of grad * weight
    STAGE_BLUR_BWD,        // bwd: the blur passes
    STAGE_SLICE_BWD,       // bwd: slice
    STAGE_SPLAT_FWD,       // fwd: splat of [v*w, w]
    STAGE_COUNT
};

bool prof_enabled();
void prof_mark(int stage, cudaStream_t s, bool begin);

}  // namespace pl

// Launch statement wrapped in optional begin/end events.
#define PL_LAUNCH(STAGE, STREAM, ...)                                  \
    do {                                                               \
        const bool pl_prof_ = ::pl::prof_enabled();                    \
        if (pl_prof_) ::pl::prof_mark((STAGE), (STREAM), true);        \
        __VA_ARGS__;                                                   \
        if (pl_prof_) ::pl::prof_mark((STAGE), (STREAM), false);       \
    } while (0)
