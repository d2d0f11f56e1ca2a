/*
 * rtgs2d -- B200 (sm_100a) Stage-1 2D gaussian splatting: C ABI.
 *
 * Plain C: device pointers, sizes and a CUDA stream passed as `void*` (a cudaStream_t; NULL is the
 * legacy default stream). Every function returns RTGS2D_OK (0) or a negative RTGS2D_ERR_* code;
 * rtgs2d_last_error() then returns a message (thread-local, valid until the next call on the same
 * thread). Functions act on the calling thread's current CUDA device. Unless stated otherwise
 * a call enqueues its work on `stream` and returns; calls that must read a device-side count
 * back to the host (the tile-entry count of a render) synchronise `stream` once.
 *
 * Array layouts follow the reference Python API (src/rtgs/image2gs/renderer2d.py:72-125):
 *   xy (M,2), chol (M,3) = (l11, l21, l22), color (M,3), weight (M,) float32, contiguous;
 *   images (B,H,W,3) and densities (B,H,W) float32, channel-last. In the batched entry points
 *   M = B*N and gaussian i belongs to view i / N.
 *
 * Results are deterministic: per-tile lists are in ascending gaussian index and gradients are
 * reduced in a fixed order, so repeated calls on the same inputs return identical bits.
 */
#ifndef RTGS2D_H_
#define RTGS2D_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define RTGS2D_API __attribute__((visibility("default")))
#else
#define RTGS2D_API
#endif

#define RTGS2D_ABI_VERSION 2

#define RTGS2D_OK 0
#define RTGS2D_ERR_INVALID (-1)  /* bad argument (shape, size, null pointer, wrong device) */
#define RTGS2D_ERR_CUDA (-2)     /* a CUDA runtime call or kernel launch failed */
#define RTGS2D_ERR_ALLOC (-3)    /* device or pinned allocation failed */
#define RTGS2D_ERR_CAPACITY (-4) /* problem larger than the 32-bit entry indexing supports, or (the
                                    allocation-free entry point) than its static scratch */

/* No reference counterpart: version and error string of this library. */
RTGS2D_API int rtgs2d_abi_version(void);
RTGS2D_API const char* rtgs2d_last_error(void);

/*
 * Scratch arena: owns the growable device buffers that projection, tile binning and the raster
 * kernels need (records, tile entries, sort buffers, per-entry gradient moments). One arena
 * serves one device; it grows on demand (cudaMalloc) and is reused across calls. Replaces the
 * per-call torch::zeros allocations of the reference extension
 * (src/rtgs/image2gs/cuda/renderer2d_ext.cu:198-199,234-237).
 *   - Streams: calls on one arena may use different streams without ordering them: each call's
 *     stream first waits (cudaStreamWaitEvent) for the end of the previous call's work on the
 *     arena, whatever stream that was, so their kernels never overlap on the arena's buffers. The
 *     price is that renders on two streams sharing one arena run one after the other on the
 *     device; give each stream its own arena for overlap.
 *   - Host threads: not safe for concurrent calls from two host threads (use one arena per
 *     thread, or a lock).
 */
typedef struct rtgs2d_arena rtgs2d_arena;
RTGS2D_API int rtgs2d_arena_create(rtgs2d_arena** out);
RTGS2D_API int rtgs2d_arena_destroy(rtgs2d_arena* arena);
/* Entries ((gaussian, tile) pairs) and pixel pairs of the last render/backward on this arena. */
RTGS2D_API int rtgs2d_arena_last_stats(const rtgs2d_arena* arena, int64_t* entries, int64_t* pairs);

/*
 * Reference ABI, forward. Replaces the pybind `forward` of
 * src/rtgs/image2gs/cuda/renderer2d_ext.cpp:87-101 (kernel renderer2d_ext.cu:26-85,186-218):
 *   xy (M,2), conics (M,3) = Sigma^-1 entries (i00, i01, i11), colors (M,3), weights (M,)
 *   float32; rects (M,4) int32 (x0, x1, y0, y1) inclusive pixel bounds, x1 < x0 when empty;
 *   view_index (M,) int32 in [0, n_views). Writes out (n_views,H,W,3) and, if den != NULL,
 *   den (n_views,H,W); every element is written (no pre-zeroing needed). A pair contributes
 *   exp(-q/2)*weight*color only if q < cutoff; non-finite means are dropped.
 */
RTGS2D_API int rtgs2d_forward(rtgs2d_arena* arena, const float* xy, const float* conics, const float* colors,
                   const float* weights, const int32_t* rects, const int32_t* view_index,
                   int64_t m, int64_t n_views, int64_t height, int64_t width, double cutoff,
                   float* out, float* den, void* stream);

/*
 * Reference ABI, backward. Replaces the pybind `backward` of
 * src/rtgs/image2gs/cuda/renderer2d_ext.cpp:103-128 (kernel renderer2d_ext.cu:87-182,220-260).
 * grad_out (n_views,H,W,3) and grad_den (n_views,H,W) may be NULL (treated as zeros). Writes
 * grad_xy (M,2), grad_conics (M,3) (dL/d(i00, i01, i11) with q = i00 dx^2 + 2 i01 dx dy + i11 dy^2),
 * grad_colors (M,3), grad_weights (M,).
 */
RTGS2D_API int rtgs2d_backward(rtgs2d_arena* arena, const float* grad_out, const float* grad_den,
                    const float* xy, const float* conics, const float* colors,
                    const float* weights, const int32_t* rects, const int32_t* view_index,
                    int64_t m, int64_t n_views, int64_t height, int64_t width, double cutoff,
                    float* grad_xy, float* grad_conics, float* grad_colors, float* grad_weights,
                    void* stream);

/*
 * No counterpart in the reference. rtgs2d_forward for callers that cannot allocate device
 * memory: a plugin whose host application owns all device memory, a latency-critical loop where
 * cudaMalloc/cudaFree would synchronise the device, or a process whose free device memory is
 * already reserved by another allocator. Same arguments (minus the arena) and same results as
 * rtgs2d_forward; all scratch comes from one 32 MiB static device array that every GPU loading
 * this library holds until exit, and nothing is allocated on the device or the host.
 *   - Problems that need more than 32 MiB of scratch (about 76 bytes per gaussian, 16 bytes per
 *     (gaussian, 16x16 tile) entry, 8 bytes per tile, plus sort/scan temporaries) fail with
 *     RTGS2D_ERR_CAPACITY and a message; use rtgs2d_forward for those.
 *   - Every call on a device shares the array and it keeps the last call's contents; calls whose
 *     GPU work overlaps on one device (different host threads, or streams not ordered with each
 *     other) race. Calls on different devices share nothing: each device has its own array and
 *     its own static host row for the statistics read back.
 *   - The first call on each device looks the array's address up with that device current. With
 *     lazy module loading (the CUDA 12 default) that first call is also what commits the 32 MiB
 *     on the device, so it fails with RTGS2D_ERR_CUDA (out of memory) if another allocator has
 *     already taken the device's free memory: make it at start-up, before other allocators
 *     reserve memory and before any stream capture.
 *   - Synchronises `stream` once (the tile-entry count is read back to the host).
 */
RTGS2D_API int rtgs2d_forward_noalloc(const float* xy, const float* conics, const float* colors,
                                      const float* weights, const int32_t* rects,
                                      const int32_t* view_index, int64_t m, int64_t n_views,
                                      int64_t height, int64_t width, double cutoff, float* out,
                                      float* den, void* stream);

/*
 * Batched render from Cholesky factors. Replaces
 * src/rtgs/image2gs/cuda_backend.py:127-170 `render_batched_cuda` (which built conics and support
 * rectangles with torch ops before calling the extension): conics, rectangles
 * (renderer2d.py:156-181, bit-exact) and tile binning are computed on the device.
 * xy (B*N,2), chol (B*N,3), color (B*N,3), weight (B*N,). Writes out (B,H,W,3) and, if den is
 * not NULL, den (B,H,W).
 */
RTGS2D_API int rtgs2d_render_forward(rtgs2d_arena* arena, const float* xy, const float* chol,
                          const float* color, const float* weight, int64_t n_views, int64_t n,
                          int64_t height, int64_t width, float* out, float* den, void* stream);

/*
 * Gradients of rtgs2d_render_forward with respect to xy, chol, color and weight (the autograd
 * path of cuda_backend.py:87-124 plus the conic -> Cholesky chain rule of gaussians2d.py:34-44).
 * grad_out / grad_den may be NULL (zeros). Any output pointer may be NULL to skip it.
 */
RTGS2D_API int rtgs2d_render_backward(rtgs2d_arena* arena, const float* grad_out, const float* grad_den,
                           const float* xy, const float* chol, const float* color,
                           const float* weight, int64_t n_views, int64_t n, int64_t height,
                           int64_t width, float* grad_xy, float* grad_chol, float* grad_color,
                           float* grad_weight, void* stream);

/*
 * rtgs2d_render_backward for the backward pass of an autograd graph (cuda_backend.py:87-124):
 * when the arena's last binning came from rtgs2d_render_forward with the same xy / chol / color /
 * weight pointers and sizes (and, if grad_den is given, that forward wrote the density), that
 * projection and binning are reused instead of recomputed; otherwise it is rtgs2d_render_backward.
 * The caller guarantees the inputs were not modified since that forward (autograd does: saved
 * tensors are kept alive and in-place changes to them are rejected). Any other binning on the
 * arena (every forward / backward entry point) ends the reuse.
 */
RTGS2D_API int rtgs2d_render_backward_after_forward(rtgs2d_arena* arena, const float* grad_out,
                                                    const float* grad_den, const float* xy,
                                                    const float* chol, const float* color,
                                                    const float* weight, int64_t n_views, int64_t n,
                                                    int64_t height, int64_t width, float* grad_xy,
                                                    float* grad_chol, float* grad_color,
                                                    float* grad_weight, void* stream);

/*
 * Support rectangles on the device, bit-exact with src/rtgs/image2gs/renderer2d.py:156-181 and in
 * the rectangle convention of src/rtgs/image2gs/cuda_backend.py:153-158: rects (M,4) int32
 * (x0, x1, y0, y1) with x1 = x0 - 1 when the support is empty, counts (M,) int64 pixels inside.
 * Either output may be NULL.
 */
RTGS2D_API int rtgs2d_support_rects(const float* xy, const float* chol, int64_t m, int64_t height,
                                    int64_t width, int32_t* rects, int64_t* counts, void* stream);

/*
 * No reference counterpart (the reference has no binning): copies the tile binning of the last
 * render/backward on `arena` to HOST memory -- gids (entries,) uint32 gaussian ids grouped by
 * tile, ascending inside a tile, and ranges (n_tiles, 2) int32 [start, end). Copies at most
 * max_entries ids and max_tiles ranges; reports the full sizes. Synchronises `stream`.
 */
RTGS2D_API int rtgs2d_arena_copy_binning(const rtgs2d_arena* arena, int64_t max_entries,
                                         uint32_t* gids, int64_t max_tiles, int32_t* ranges,
                                         int64_t* n_entries, int64_t* n_tiles, void* stream);

/*
 * Fit engine: the native Stage-1 fit loop on the device (fit.py:355-554 for one image,
 * batched.py:39-170 for stacked views). Each iteration runs tile binning, one fused forward +
 * L2-loss-gradient + backward raster kernel and one fused chain-rule + Adam + projection kernel;
 * the host only advances the cosine learning rate (CosineAnnealingLR(T_max=iterations,
 * eta_min=0.1*lr), fit.py:419-422) once per chunk of iterations.
 */
typedef struct rtgs2d_fit rtgs2d_fit;

#define RTGS2D_LOSS_MSE 0          /* sum over views of per-view MSE (fit.py:561, batched.py:142) */
#define RTGS2D_LOSS_MASK_WEIGHTED 1 /* mean((r-t)^2 * (0.1 + 0.9 mask)) per view (fit.py:562-563) */
#define RTGS2D_LOSS_MASK_ONLY 2    /* squared error over mask pixels / (3 * mask pixels) per view */

typedef struct rtgs2d_fit_options {
  double lr;               /* Adam learning rate (FitConfig.lr, default 1e-2) */
  int64_t iterations;      /* cosine schedule length T_max (FitConfig.iterations) */
  int64_t log_every;       /* record loss sums at it % log_every == 0 and at the last iteration */
  int64_t check_every;     /* also record at (it + 1) % check_every == 0 (0: never) */
  int32_t freeze_geometry; /* nonzero: only color/weight are optimised (FitConfig.freeze_geometry) */
  int32_t loss_mode;       /* RTGS2D_LOSS_* */
  double mask_coverage_weight; /* > 0: add weight * mean(coverage * (1 - mask)) to the loss, coverage
                                  = 1 - exp(-sum weight_i G_i) (fit.py:457-459,566-572); needs a
                                  mask loss mode */
} rtgs2d_fit_options;

RTGS2D_API int rtgs2d_fit_create(int64_t n_views, int64_t n, int64_t height, int64_t width,
                      const rtgs2d_fit_options* options, rtgs2d_fit** out);
RTGS2D_API int rtgs2d_fit_destroy(rtgs2d_fit* fit);
/* targets (B,H,W,3) float32 (copied); mask_bits (B, ceil(H*W/8)) uint8 little-endian bit order
 * (numpy packbits(bitorder="little") of the row-major mask), required for the mask loss modes.
 * Synchronises `stream` (per-view mask pixel counts are read back). */
RTGS2D_API int rtgs2d_fit_set_targets(rtgs2d_fit* fit, const float* targets, const uint8_t* mask_bits,
                           void* stream);
/* Raw (unconstrained) parameters in the reference layout: xy_raw (B,N,2), diag_raw (B,N,2),
 * off_raw (B,N), color_raw (B,N,3), weight_raw (B,N) (fit.py:375-380). Resets the Adam state
 * and the iteration counter. */
RTGS2D_API int rtgs2d_fit_set_raw(rtgs2d_fit* fit, const float* xy_raw, const float* diag_raw,
                       const float* off_raw, const float* color_raw, const float* weight_raw,
                       void* stream);
/*
 * Initialisation from constrained parameters in one pass: the reference's checks of an initial
 * Gaussians2D (src/rtgs/image2gs/fit.py:634-676) and its raw transform (fit.py:375-380, with the
 * non-finite raw check of fit.py:134-141) run on the device, followed by rtgs2d_fit_set_raw's
 * reset. Replaces the torch validation and transform ops of _fit_native_from_initialization
 * (fit.py:355-380) before the engine. xy (B,N,2), chol (B,N,3), color (B,N,3), weight (B,N)
 * float32 device arrays. *status receives 0 or the OR of the RTGS2D_INIT_* bits of the checks
 * that failed for some gaussian; the caller decides which failures to report (the rows are not
 * returned). The raw values are written whatever the status (the transform clamps as the
 * reference does); with RTGS2D_INIT_NONFINITE_RAW set the engine refuses to run until parameters
 * are set again. Synchronises `stream`.
 */
#define RTGS2D_INIT_NONFINITE_XY 1u
#define RTGS2D_INIT_NONFINITE_CHOL 2u
#define RTGS2D_INIT_NONFINITE_COLOR 4u
#define RTGS2D_INIT_NONFINITE_WEIGHT 8u
#define RTGS2D_INIT_OUTSIDE 16u        /* a mean outside [0, W) x [0, H) */
#define RTGS2D_INIT_DIAG 32u           /* a Cholesky diagonal entry not above 0.3 */
#define RTGS2D_INIT_COLOR_RANGE 64u    /* a colour outside [0, 1] */
#define RTGS2D_INIT_WEIGHT_RANGE 128u  /* a weight outside [0, 1] */
#define RTGS2D_INIT_NONFINITE_RAW 256u /* a non-finite raw parameter */
RTGS2D_API int rtgs2d_fit_set_initial(rtgs2d_fit* fit, const float* xy, const float* chol,
                                      const float* color, const float* weight, uint32_t* status,
                                      void* stream);
/*
 * Appearance parameterisation (FitConfig.appearance_parameterization, fit.py:27,381-411).
 * WEIGHT_COLOR_9P (the default) optimises colour and weight logits; UNIT_WEIGHT_8P optimises one
 * bounded amplitude per channel (colour = sigmoid(amplitude_raw)) with every weight fixed at 1.
 * Under UNIT_WEIGHT_8P the colour arrays of rtgs2d_fit_set_raw, rtgs2d_fit_get_raw and
 * rtgs2d_fit_write_rows carry amplitude_raw and their weight_raw arguments are ignored (NULL is
 * allowed), rtgs2d_fit_set_initial writes amplitude_raw = logit(sigmoid(weight_raw) *
 * sigmoid(color_raw)) from the clamped logits (fit.py:384-385), and rtgs2d_fit_get_params returns
 * weights of exactly 1. A change of parameterisation invalidates the raw parameters: the engine
 * refuses to run until rtgs2d_fit_set_raw or rtgs2d_fit_set_initial is called again.
 */
#define RTGS2D_APPEARANCE_WEIGHT_COLOR_9P 0
#define RTGS2D_APPEARANCE_UNIT_WEIGHT_8P 1
RTGS2D_API int rtgs2d_fit_set_appearance(rtgs2d_fit* fit, int32_t parameterization);
/* Runs `n_iterations` more iterations (capped at `iterations`). Synchronises `stream`. */
RTGS2D_API int rtgs2d_fit_run(rtgs2d_fit* fit, int64_t n_iterations, void* stream);
RTGS2D_API int rtgs2d_fit_get_raw(rtgs2d_fit* fit, float* xy_raw, float* diag_raw, float* off_raw,
                       float* color_raw, float* weight_raw, void* stream);
/* Constrained parameters (build(), fit.py:402-417): xy (B,N,2), chol (B,N,3), color (B,N,3),
 * weight (B,N). */
RTGS2D_API int rtgs2d_fit_get_params(rtgs2d_fit* fit, float* xy, float* chol, float* color, float* weight,
                          void* stream);
/* The fit loss's gradient with respect to the raw parameters at the current state, as the next
 * iteration's Adam step would receive it (the fit loop's own raster and chain rule), without an
 * update: what the reference's raw_parameters[name].grad hold after loss.backward() (fit.py:451-460,
 * read by its native fit diagnostics, fit.py:691-766). Layouts of rtgs2d_fit_get_raw; NULL
 * outputs are skipped. With `render` (B,H,W,3) the current render, with `sums` (B,2) host the
 * loss and clamped-PSNR numerators (as rtgs2d_fit_evaluate). Synchronises `stream`. */
RTGS2D_API int rtgs2d_fit_gradients(rtgs2d_fit* fit, float* xy_raw, float* diag_raw, float* off_raw,
                                    float* color_raw, float* weight_raw, float* render, double* sums,
                                    void* stream);
/* Adam moments of the raw parameters (torch Adam's exp_avg for which = 1, exp_avg_sq for 2, the
 * optimizer state the reference's diagnostics copy, fit.py:710-714), in the layouts of
 * rtgs2d_fit_get_raw; NULL outputs are skipped. The completed update count is rtgs2d_fit_stats'
 * step. */
RTGS2D_API int rtgs2d_fit_get_moments(rtgs2d_fit* fit, int32_t which, float* xy, float* diag, float* off,
                                      float* color, float* weight, void* stream);
/* Renders the current parameters; writes render (B,H,W,3) if not NULL and the per-view loss and
 * clamped-PSNR numerators to host sums (B,2). Synchronises `stream`. */
RTGS2D_API int rtgs2d_fit_evaluate(rtgs2d_fit* fit, float* render, double* sums, void* stream);
/* Recorded loss sums: copies up to max_rows rows; iters (rows,), sums (rows,B,2) on the host. */
RTGS2D_API int rtgs2d_fit_history(const rtgs2d_fit* fit, int64_t max_rows, int64_t* iters, double* sums,
                       int64_t* n_rows);
/*
 * Fused Adam step over up to RTGS2D_ADAM_MAX_TENSORS float32 device tensors in one launch: the
 * update of torch.optim.Adam (fit.py:419; no weight decay, amsgrad or maximize) that the fit loop
 * applies inside its Adam kernel, for callers that keep their own loop (a reference-style loop of
 * render, backward and optimizer step; rtgs_b200.image2gs.optim.FusedAdam wraps it). For every
 * element: exp_avg += (1 - beta1) (grad - exp_avg); exp_avg_sq = beta2 exp_avg_sq + (1 - beta2)
 * grad^2; param -= lr / (1 - beta1^step) * exp_avg / (sqrt(exp_avg_sq) / sqrt(1 - beta2^step)
 * + eps), the square root and the last division as fast hardware approximations (relative error
 * ~1e-7). `step` counts the updates including this one (1 for the first). Stream-ordered, no
 * synchronisation. Replaces the per-parameter ATen Adam kernels of the reference's loop.
 */
#define RTGS2D_ADAM_MAX_TENSORS 16
RTGS2D_API int rtgs2d_adam_step(int32_t n_tensors, float* const* params, const float* const* grads,
                                float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* sizes,
                                double lr, double beta1, double beta2, double eps, int64_t step,
                                void* stream);
/* No reference counterpart: tile-entry capacity of the fit loop. The loop bins into a fixed number
 * of (gaussian, tile) entries; a chunk of iterations that needed more is rolled back and re-run
 * with more room (results are unchanged). rtgs2d_fit_reserve pre-sizes the capacity;
 * rtgs2d_fit_capacity reports it and the number of re-run chunks. */
RTGS2D_API int rtgs2d_fit_reserve(rtgs2d_fit* fit, int64_t entries, void* stream);
RTGS2D_API int rtgs2d_fit_capacity(const rtgs2d_fit* fit, int64_t* entries, int64_t* retries);
/* No reference counterpart: stage timing. When enabled, every iteration records CUDA events on
 * `stream` around projection + binning, the fused raster kernel and the Adam kernel; the
 * accumulated device milliseconds are returned by rtgs2d_fit_stage_times (after a run). */
RTGS2D_API int rtgs2d_fit_set_profiling(rtgs2d_fit* fit, int32_t enable);
/* Pool rows (image2gs/pool.py:55-151: GaussianPool2D's active mask, park, activate and the
 * per-row Adam moment reset). rtgs2d_fit_set_active copies a device mask of M = n_views * n
 * bytes (0 = parked: the row is not rendered, so it has no contribution and no gradient; with
 * zero Adam moments it then stays unchanged); NULL makes every row live. rtgs2d_fit_write_rows
 * writes raw parameters (the layouts of rtgs2d_fit_set_raw, n_rows rows each; all five NULL keeps
 * the values) into the rows listed in the device array `rows` (indices into M; others skipped)
 * and zeroes both Adam moments of those rows. Both are ordered on `stream`. */
RTGS2D_API int rtgs2d_fit_set_active(rtgs2d_fit* fit, const uint8_t* active, void* stream);
RTGS2D_API int rtgs2d_fit_write_rows(rtgs2d_fit* fit, const int64_t* rows, int64_t n_rows,
                                     const float* xy_raw, const float* diag_raw,
                                     const float* off_raw, const float* color_raw,
                                     const float* weight_raw, void* stream);
/* No reference counterpart: CUDA-graph replay of the fit loop. A run proceeds in chunks of 64
 * iterations with no host synchronisation inside a chunk; once a chunk of a given shape (length,
 * binning path, buffer layout) has run eagerly, later chunks of that shape are captured into a
 * CUDA graph once and replayed (same kernels, same results). rtgs2d_fit_set_graphs(fit, 0) runs
 * every chunk eagerly; rtgs2d_fit_chunk_counts reports how many chunks ran each way. */
RTGS2D_API int rtgs2d_fit_set_graphs(rtgs2d_fit* fit, int32_t enable);
RTGS2D_API int rtgs2d_fit_chunk_counts(const rtgs2d_fit* fit, int64_t* graph_chunks,
                                       int64_t* eager_chunks);
/* No reference counterpart: how the fit loop bins (gaussian, tile) entries. Every mode gives the
 * same per-tile lists, so the same results bit for bit.
 *   RTGS2D_BINNING_AUTO     the first iteration of a chunk scatters its entries into tile lists;
 *                           each later projection writes its ids straight into per-tile segments
 *                           sized from the previous binning with slack (count + count/4 + 8), and
 *                           the fit raster sorts each tile's segment itself (lists up to 512; a
 *                           longer one makes the fit use SORTED from that chunk on). A segment
 *                           that fills up invalidates the chunk, which re-runs with SCATTER. The
 *                           rasters of later iterations take their tiles heaviest first. Up to
 *                           2^20 tiles (all views); more use SCATTER.
 *   RTGS2D_BINNING_SORTED   AUTO with the segments sorted by a separate per-tile sort kernel
 *                           before the raster (lists up to 2048).
 *   RTGS2D_BINNING_SCATTER  every iteration: entries, tile-count scan, scatter, per-tile sort.
 *   RTGS2D_BINNING_RADIX    every iteration: entries, radix sort by (tile, id), tile ranges.
 *   RTGS2D_BINNING_TIGHT    AUTO with segments of exactly the previous counts (no slack): any tile
 *                           that gains an entry overflows. Exercises the overflow re-run.
 * Re-runs after an overflow count in rtgs2d_fit_capacity's `retries`. */
#define RTGS2D_BINNING_AUTO 0
#define RTGS2D_BINNING_SCATTER 1
#define RTGS2D_BINNING_RADIX 2
#define RTGS2D_BINNING_TIGHT 3
#define RTGS2D_BINNING_SORTED 4
RTGS2D_API int rtgs2d_fit_set_binning(rtgs2d_fit* fit, int32_t mode);
RTGS2D_API int rtgs2d_fit_stage_times(const rtgs2d_fit* fit, double* bin_ms, double* raster_ms,
                                      double* adam_ms, int64_t* iterations_timed,
                                      double* pairs_timed);
/* Completed iterations, entries/pairs of the last iteration, pairs summed over all iterations. */
RTGS2D_API int rtgs2d_fit_stats(const rtgs2d_fit* fit, int64_t* step, int64_t* last_entries,
                     int64_t* last_pairs, double* total_pairs);

#ifdef __cplusplus
}
#endif

#endif /* RTGS2D_H_ */
