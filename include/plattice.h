/*
 * plattice.h -- C ABI of the sm_100a permutohedral-lattice filter
 * (libplattice_b200.so, built from plattice_pytorch_b200/csrc).
 *
 * Drop-in boundary for the reference OliveMY/plattice_pytorch, whose CUDA
 * entry points are
 *   permuto_filter      (permutohedral.cu:685-715, declared permuto.cpp:11-20)
 *   permuto_filter_grad (permutohedral.cu:717-748, declared permuto.cpp:21-31)
 * and whose workspace is sized by allocate_workspace (permuto.cpp:51-69).
 * The reference binds them to Python through a torch extension (permuto.cpp);
 * here the boundary is plain C: device pointers, sizes, an explicit CUDA
 * stream (passed as void*) and an int status.  No call synchronises the stream
 * except plattice_lattice_info, plattice_vertex_keys and
 * plattice_noalloc_status.
 *
 * Device-side failures (a hash table too small, a bounded wait that gave up)
 * are reported without synchronising: the last kernel of every call writes
 * the lattice's status word to a slot of pinned, host-mapped memory, and the
 * first call whose start finds a failed earlier call there -- once that
 * call's kernels have finished -- returns PLATTICE_ERR_DEVICE without
 * enqueueing its own work (plattice_last_error_detail names the failed call).
 * plattice_poll_status does the same check on its own.
 *
 * Tensors: features [h][w][pd], values / grad / out [h][w][vd],
 * weight [h][w] (one float per pixel), all float32, contiguous, on the current
 * CUDA device.  1 <= pd <= 16, 1 <= vd <= 8 (permuto.cpp:37-40).
 *
 * Memory.  The caller allocates two device buffers, sized by
 * plattice_workspace_sizes:
 *   lattice  -- the built lattice; kept from a forward call to the backward
 *               calls that reuse it (its size does not depend on vd).
 *   scratch  -- transient; only needed during a call.  A backward that
 *               reuses a kept lattice needs only its first
 *               plattice_reuse_scratch_size bytes (one value-row buffer of its
 *               blur and the blur's bookkeeping).
 * Calls that overlap in time must not share either buffer.
 */
#ifndef PLATTICE_H
#define PLATTICE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PLATTICE_ABI_VERSION 5

/* status codes */
#define PLATTICE_OK 0
#define PLATTICE_ERR_INVALID 1   /* bad dimensions, null pointer, or image too large */
#define PLATTICE_ERR_WORKSPACE 2 /* lattice or scratch buffer smaller than required */
#define PLATTICE_ERR_CUDA 3      /* a CUDA runtime call or kernel launch failed */
#define PLATTICE_ERR_DEVICE 4    /* a device status word reports a failure (this lattice's,
                                    or an earlier call's: see above) */

/* device status bits reported by plattice_lattice_info */
#define PLATTICE_DEV_TABLE_FULL 2 /* hash-table probe limit reached (table too small) */
#define PLATTICE_DEV_WAIT_LIMIT 4 /* a bounded wait on a concurrent insert gave up */
#define PLATTICE_DEV_ROUND_LIMIT 8

/* Version of this ABI (PLATTICE_ABI_VERSION). */
int plattice_abi_version(void);

/* Human-readable text of a status code. */
const char* plattice_error_string(int status);

/* The CUDA error name and text behind the last PLATTICE_ERR_CUDA returned on
 * the calling thread ("" if none). */
const char* plattice_last_error_detail(void);

/* Bytes of the lattice and scratch buffers for an h x w image.  Replaces the
 * workspace sizing of permuto.cpp:51-69. */
int plattice_workspace_sizes(int h, int w, int pd, int vd, size_t* lattice_bytes,
                             size_t* scratch_bytes);

/* Bytes of scratch that a backward reusing a kept lattice of b images needs
 * (lattice_state 1 or 2): the front part of the full scratch.  No reference
 * counterpart (the reference rebuilds, permutohedral.cu:615-635). */
int plattice_reuse_scratch_size(int b, int h, int w, int pd, int vd, size_t* bytes);

/* Forward filter: builds the lattice of `features` into `lattice`, splats
 * `values`, blurs along the pd+1 lattice axes in order 0..pd and slices:
 *   out[p] = sum_i w_pi L[v_pi][0:vd] / sum_i w_pi L[v_pi][vd],
 *   weight_out[p] = 1 / sum_i w_pi L[v_pi][vd].
 * Replaces permuto_filter (permutohedral.cu:685); same argument order, plus
 * buffer sizes and the stream. */
int plattice_forward(float* weight_out, float* out, const float* values, const float* features,
                     void* lattice, size_t lattice_bytes, void* scratch, size_t scratch_bytes,
                     int pd, int vd, int w, int h, void* stream);

/* Value gradient: grad_values_out = S^T B^T S'(grad * weight_in), the blur in
 * axis order pd..0.  lattice_state: 0 = `lattice` does not hold the lattice of
 * `features` (it is rebuilt, `scratch` and `features` required); 1 = it holds
 * the lattice built by the last plattice_forward on these features (1 and 2,
 * "not yet used by a backward" and "used", are treated alike).  `features` is
 * read only by a rebuild and may be NULL otherwise.  `scratch` is always
 * required: scratch_bytes from plattice_workspace_sizes for a rebuild, at
 * least plattice_reuse_scratch_size otherwise.  After any call on a kept
 * lattice returns an error, build the lattice again (plattice_forward) before
 * the next call on it.  Replaces permuto_filter_grad (permutohedral.cu:717),
 * which always rebuilds. */
int plattice_backward(float* grad_values_out, const float* grad, const float* weight_in,
                      const float* features, void* lattice, size_t lattice_bytes,
                      int lattice_state, void* scratch, size_t scratch_bytes, int pd, int vd,
                      int w, int h, void* stream);

/* Batches: B images of one shape, [B][h][w][...] contiguous (features,
 * values, outputs), in one call -- the dense-CRF use of many images.  Each
 * image has its own lattice vertices, but the B lattices share one buffer
 * and one launch of every stage: the key hash mixes in the image index, so
 * equal keys of two images never merge.  Sizes from
 * plattice_batch_workspace_sizes (b = 1 gives plattice_workspace_sizes).
 * The reference has no batch call (its callers loop over images in Python,
 * permuto.cpp:71-158 per image).  plattice_backward_batch takes the same
 * lattice_state values as plattice_backward, for all B images at once. */
int plattice_batch_workspace_sizes(int b, int h, int w, int pd, int vd, size_t* lattice_bytes,
                                   size_t* scratch_bytes);
int plattice_forward_batch(float* weight_out, float* out, const float* values, const float* features,
                           void* lattice, size_t lattice_bytes, void* scratch, size_t scratch_bytes,
                           int b, int pd, int vd, int w, int h, void* stream);
int plattice_backward_batch(float* grad_values_out, const float* grad, const float* weight_in,
                            const float* features, void* lattice, size_t lattice_bytes,
                            int lattice_state, void* scratch, size_t scratch_bytes, int b, int pd,
                            int vd, int w, int h, void* stream);

/* Kept lattice: filter further value tensors on the lattice that a
 * plattice_forward call built (same h, w, pd; any vd), without rebuilding it
 * -- e.g. the iterations of a mean-field CRF.  No counterpart in the
 * reference, which rebuilds the lattice on every call (permutohedral.cu:549-570
 * in the forward, 615-635 in the backward).
 *
 * plattice_filter: the forward filter of `values` (same outputs as
 * plattice_forward: out and weight_out) using `lattice`.
 * plattice_filter_backward: the value gradient of such a call, given its
 * weight_out as weight_in (same result as plattice_backward).
 * `values_ws` holds the lattice value rows of the call
 * (plattice_filter_workspace_size bytes; any allocator, reusable across
 * calls).  A lattice built with any vd serves every vd.
 * Both calls update bookkeeping in the lattice header, so calls on one
 * lattice must be issued one after the other (one stream). */
int plattice_filter_workspace_size(int h, int w, int pd, int vd, size_t* bytes);
int plattice_filter(float* weight_out, float* out, const float* values, void* lattice,
                    size_t lattice_bytes, void* values_ws, size_t values_ws_bytes, int pd, int vd,
                    int w, int h, void* stream);
int plattice_filter_backward(float* grad_values_out, const float* grad, const float* weight_in,
                             void* lattice, size_t lattice_bytes, void* values_ws,
                             size_t values_ws_bytes, int pd, int vd, int w, int h, void* stream);

/* Gradient of the forward filter with respect to the features (no
 * counterpart in the reference, whose Function returns None for them,
 * plattice.py:19): grad_features_out [h][w][pd] = dL/dfeatures for
 * dL/dout = `grad`, given the forward's `out` and `weight` (weight_out) on
 * `values`, and `lattice` as that forward on `features` left it.  The slope
 * is that of the piecewise-linear filter inside each pixel's simplex (the
 * vertex assignment is piecewise constant).  `ws`:
 * plattice_feature_grad_workspace_size bytes.  Updates lattice header
 * bookkeeping like plattice_filter (one stream per lattice). */
int plattice_feature_grad_workspace_size(int h, int w, int pd, int vd, size_t* bytes);
int plattice_feature_grad(float* grad_features_out, const float* grad, const float* out,
                          const float* weight, const float* values, const float* features,
                          void* lattice, size_t lattice_bytes, void* ws, size_t ws_bytes, int pd,
                          int vd, int w, int h, void* stream);

/* Synchronises `stream` and reads the lattice header: device status bits,
 * vertex count m, number of tile-unique keys staged, log2 of the hash-table
 * capacity used.  Any pointer may be NULL.  Returns PLATTICE_ERR_DEVICE when
 * the status word is non-zero.  No reference counterpart (the reference has
 * no error reporting). */
int plattice_lattice_info(const void* lattice, int* status, int* m, int* u_total, int* cap_log2,
                          void* stream);

/* Copies the vertex keys of the lattice just built (before `scratch` is
 * reused) into keys_dev [max_keys][pd] int16 on the device, in vertex-id
 * order; synchronises `stream` and stores the vertex count in *m.  Test
 * support: the reference keeps its keys inside its workspace
 * (permutohedral.cu:84) and exposes none. */
int plattice_vertex_keys(const void* lattice, const void* scratch, int pd, int vd, int w, int h,
                         int16_t* keys_dev, int max_keys, int* m, void* stream);

/* Reports device-side failures of earlier calls whose kernels have finished
 * (see the top of this file): PLATTICE_ERR_DEVICE once per failure, with
 * plattice_last_error_detail naming the call; PLATTICE_OK otherwise.  Does
 * not synchronise.  No reference counterpart. */
int plattice_poll_status(void);

/* Everything the first call for (pd, vd) does in the current CUDA context
 * apart from the filter itself: kernel attribute settings (dynamic shared
 * memory limits), occupancy queries of the cooperative kernels, and the
 * loading of every kernel of the forward and backward filter (with lazy
 * module loading each kernel is otherwise loaded at its first launch).  Call it before any stream capture, or before real-time work that
 * must not pay these costs.  No reference counterpart. */
int plattice_prepare(int pd, int vd);

/* Call graphs (no reference counterpart; the reference launches every kernel
 * from the host on every call, permutohedral.cu:549-596).  A forward or
 * backward call whose buffers, sizes and settings equal those of an earlier
 * call in the same CUDA context is run as a CUDA graph: the second such call
 * captures its launches into a graph (captured on a private stream of the
 * context, in thread-local capture mode), later ones launch that graph on
 * their stream -- one launch instead of seven (forward) or three (backward)
 * on the host.  Results are the same either way.  `entries` graphs per
 * context are kept (least recently used evicted; default 16, or 0 when the
 * environment variable PLATTICE_GRAPHS is "0"); 0 turns graphs off.  Changing
 * the setting releases every cached graph.  While profiling is enabled, and
 * for plattice_forward_noalloc, calls run without graphs. */
int plattice_set_graph_cache(int entries);
/* Graphs captured and graph launches made so far (process-wide counts). */
void plattice_graph_cache_stats(long long* captures, long long* replays);

/* Test support: force the hash-table capacity to 2^log2 cells (0 = automatic,
 * >= twice the staged keys).  A capacity below the vertex count makes the
 * build report PLATTICE_DEV_TABLE_FULL instead of looping. */
void plattice_debug_set_table_cap_log2(int log2_cells);

/* Test support: the table size (log2 cells) from which blur-neighbour lookups
 * consult the miss filter (0 = automatic: 2^22 cells and more), so that small
 * cases can exercise the filter.  No reference counterpart (the reference
 * probes its table for every neighbour lookup, permutohedral.cu:119-141 as
 * called from precomputeBlurNeighbors, permutohedral.cu:350-383). */
void plattice_debug_set_miss_filter_log2(int log2_cells);

/* Reduced-precision lattice values (off by default; process-wide, read when a
 * call is enqueued).  bits = 16: the blur passes of large lattices (more
 * vertices than the blur grid keeps in registers, about 150 k) store the rows
 * they write as bfloat16 and read them back widened, with float arithmetic;
 * the splat still accumulates in float and the slice reads float rows.
 * Outputs then differ from the float path by the bfloat16 rounding of up to
 * pd+1 passes (about 1 % of the output's range; the tests bound it at 2 %).
 * bits = 32 (default): float everywhere.  Returns PLATTICE_ERR_INVALID for any
 * other value.  The reference computes in float only (permutohedral.cu:321-348). */
int plattice_set_lattice_precision(int bits);
int plattice_get_lattice_precision(void);

/* Test support: run the blur's streaming passes (the large-lattice path, with
 * one grid barrier per pass) for every lattice, so that small cases exercise
 * them (0 = automatic choice by size). */
void plattice_debug_set_blur_streaming(int on);

/* Forward filter for callers that cannot allocate device memory (no
 * counterpart in the reference, whose host layer allocates a new workspace on
 * every call).  Same computation and outputs as plattice_forward, but the
 * lattice and scratch buffers live in one fixed 64 MiB array inside the
 * library (plattice_noalloc_capacity() bytes), held on every GPU that loads
 * the library until the process exits; the call allocates no device memory.
 * An image whose workspace exceeds the array returns PLATTICE_ERR_WORKSPACE
 * (plattice_noalloc_error_detail() says how much it needs).
 * First call in a CUDA context: it looks up the array's device address in
 * that context, sets kernel attributes, queries occupancies, and (lazy module
 * loading) loads the kernels it launches -- plattice_prepare(pd, vd) does all
 * of this except the address lookup, and plattice_noalloc_status does the
 * lookup; make these first calls before any stream capture.  All calls on a device share the array, so calls that
 * overlap on the GPU race: issue them one after the other.  Its device
 * failures are not reported through the status ring (whose pinned host slots
 * would be an allocation): plattice_noalloc_status reads them. */
int plattice_forward_noalloc(float* weight_out, float* out, const float* values, const float* features,
                             int pd, int vd, int w, int h, void* stream);
size_t plattice_noalloc_capacity(void);
const char* plattice_noalloc_error_detail(void);

/* Synchronises `stream` and reads the header of the lattice that the last
 * plattice_forward_noalloc in the current context left in the fixed array:
 * device status bits and vertex count (either pointer may be NULL).  Returns
 * PLATTICE_ERR_DEVICE when the status word is non-zero. */
int plattice_noalloc_status(int* status, int* m, void* stream);

/* Profiling (no reference counterpart).  plattice_profile_enable(1): every
 * kernel launch is bracketed by CUDA events recorded on its stream (stages
 * 0-10); plattice_profile_enable(2): only launch groups are (stages 11-13),
 * so that fewer events sit between the kernels; 0 turns it off.  While it is
 * on, calls run without call graphs.  plattice_profile_read waits for the
 * recorded events, writes per stage the summed milliseconds and the count
 * (stage order as plattice_profile_stage_name), and clears the record.
 * Stages: 0 tile_build, 1 clear, 2 insert (and compaction), 3 neighbors,
 * 4 blur_fwd, 5 slice_fwd, 6 zero, 7 splat_bwd, 8 blur_bwd, 9 slice_bwd,
 * 10 splat_fwd; groups: 11 build (header memset .. insert), 12 filter_fwd (a
 * forward's launches after the build), 13 filter_bwd (a backward's splat,
 * blur and slice). */
#define PLATTICE_PROFILE_STAGES 14
void plattice_profile_enable(int on);
int plattice_profile_read(double* ms_total, int* launches, int n_stages);
const char* plattice_profile_stage_name(int stage);

#ifdef __cplusplus
}
#endif

#endif /* PLATTICE_H */
