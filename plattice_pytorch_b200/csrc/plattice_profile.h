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
    STAGE_GROUP_BUILD,     // group mode: memset .. insert of a lattice build
    STAGE_GROUP_FILTER_FWD,// group mode: a forward's launches after the build (neighbours, splat, blur, slice)
    STAGE_GROUP_FILTER_BWD,// group mode: a backward's splat, blur and slice
    STAGE_COUNT
};

// 0 off; 1 events around every launch; 2 events around launch groups only
// (fewer events in the stream, so the groups' intervals are closer to the
// kernels' own time)
int prof_mode();
inline bool prof_enabled() { return prof_mode() != 0; }
void prof_mark(int stage, cudaStream_t s, bool begin);

}  // namespace pl

// Launch statement wrapped in optional begin/end events (per-launch mode).
#define PL_LAUNCH(STAGE, STREAM, ...)                                  \
    do {                                                               \
        const bool pl_prof_ = ::pl::prof_mode() == 1;                  \
        if (pl_prof_) ::pl::prof_mark((STAGE), (STREAM), true);        \
        __VA_ARGS__;                                                   \
        if (pl_prof_) ::pl::prof_mark((STAGE), (STREAM), false);       \
    } while (0)

// Begin / end event of a launch group (group mode).
#define PL_GROUP(STAGE, STREAM, BEGIN)                                 \
    do {                                                               \
        if (::pl::prof_mode() == 2) ::pl::prof_mark((STAGE), (STREAM), (BEGIN)); \
    } while (0)
