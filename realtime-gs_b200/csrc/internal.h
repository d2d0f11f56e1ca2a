// Host-side internal interfaces shared by the translation units of librtgs2d.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "common.cuh"

namespace rtgs2d {

// ---- error reporting --------------------------------------------------------------------------
// Every C entry point returns 0 or a negative RTGS2D_ERR_* code and leaves a message that
// rtgs2d_last_error() returns (thread-local).
int set_error(int code, const std::string& msg);
int check_cuda(cudaError_t err, const char* what);
#define RTGS_TRY(expr)            \
  do {                            \
    int _rc = (expr);             \
    if (_rc != 0) return _rc;     \
  } while (0)
#define RTGS_CUDA(expr, what) RTGS_TRY(::rtgs2d::check_cuda((expr), (what)))


// ---- device memory ------------------------------------------------------------------------------
// A growable device buffer. ensure() reallocates only when more bytes are needed; before freeing
// the old allocation it synchronises `stream` so no queued kernel still reads it.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  int ensure(size_t need, cudaStream_t stream);
  void release();
  template <typename T>
  T* as() const { return static_cast<T*>(ptr); }
};

// Blocks of every radix-sort pass (sort.cu); the per-pass digit-count array holds 256 x this.
constexpr int kSortGrid = 592;

// Device statistics slots (unsigned long long each).
enum StatSlot : int {
  kStatEntries = 0,      // (gaussian, tile) entries of the current projection
  kStatPairs = 1,        // (gaussian, pixel-in-rectangle) pairs of the current projection
  kStatPairsTotal = 2,   // pairs accumulated over projections until reset by the caller
  kStatMaxEntries = 3,   // largest entry count binned since reset by the caller (capacity check)
  kStatLongTile = 4,     // largest tile list longer than kSegSortMax since reset (0: none)
  kStatLastEntries = 5,  // entries of the last binned projection (copied by the binning)
  kStatLastPairs = 6,    // pairs of the last binned projection
  kStatSegOverflow = 7,  // a direct placement found a tile segment full (its binning is invalid)
  kStatFusedLong = 8,    // a fit raster that sorts its own tile found a list above kFusedSortMax
  kStatSlots = 9
};

// Tile lists up to this length are sorted by the tile-sort kernel (one warp per tile, in shared
// memory); a binning with a longer list uses the global radix sort instead.
constexpr int kSegSortMax = 2048;
// Tile lists up to this length are sorted by the fused fit raster itself (one warp, in registers),
// in the direct-placement iterations of the fit loop; a longer list makes the chunk re-run with
// the separate tile-sort kernel.
constexpr int kFusedSortMax = 512;

// Scratch used by projection + tile binning + raster for one render / one fit iteration.
struct BinBuffers {
  DevBuf records;     // GaussRecord[M]
  DevBuf weights;     // float[M] (density variants)
  DevBuf spans;       // TileSpan[M]
  DevBuf counts;      // int[M]  tiles per gaussian
  DevBuf offsets;     // int[M]  entry index of each gaussian's first tile (see bin_entries)
  DevBuf list;        // uint32[capacity] gaussian ids grouped by tile, ascending inside a tile
  DevBuf tile_count;  // int[n_tiles] entries per tile (counted up by the projection, back down
                      //   to zero by the scatter)
  DevBuf tile_end;    // int[n_tiles] inclusive scan of tile_count
  DevBuf entries[2];  // uint64[capacity] (tile key << 32 | gaussian id), radix-sort double buffer
  DevBuf ranges;      // int2[n_tiles] [start, end) of every tile in the list (or sorted entries)
  DevBuf seg;         // int2[2][n_tiles] direct placement: (start, slots) of each tile's segment
  DevBuf cursor;      // int[2][n_tiles] direct placement: next free list position of each tile
  DevBuf tile_order;  // int[2][n_tiles] raster block order (tiles by descending entry count)
  DevBuf partials;    // float[capacity][8] per (gaussian, tile) gradient moments
  DevBuf partial_d;   // float[capacity]   per (gaussian, tile) density-gradient moment
  DevBuf cub_temp;    // exclusive-scan temporaries
  DevBuf sort_counts; // int[256 * kSortGrid] radix-sort digit counts
  DevBuf stats;       // unsigned long long[kStatSlots]
  unsigned long long* host_stats = nullptr;  // pinned mirror of `stats`
  int sorted_sel = 0;                         // which entries buffer holds the sorted result
  bool presorted = false;                     // radix path (entries + ranges) produced the binning
  bool counts_cleared = false;                // the last binning left stats slots 0-1 at zero
                                              //   and tile_count at zero for the next projection
                                              //   (after a scatter; a layout leaves fresh cursors)
  bool entries_emitted = false;               // the last projection emitted the entries
  int64_t capacity = 0;                       // entries the entry buffers can hold
  int64_t n_entries = 0;                      // host-known entry count (synchronous binning)
  int64_t n_pairs = 0;
  bool long_tile = false;                     // host-known: some tile list exceeds kSegSortMax
  ~BinBuffers();
  void release();
};

struct Geometry {
  int n_views = 1;
  int height = 0, width = 0;
  int tiles_x = 0, tiles_y = 0, tiles_per_view = 0;
  int64_t n_tiles() const { return static_cast<int64_t>(n_views) * tiles_per_view; }
};
Geometry make_geometry(int n_views, int height, int width);

// ---- projection (project.cu) --------------------------------------------------------------------
// All projection launchers zero bb.stats first and fill records/spans/counts/offsets (+weights
// if asked), and count entries per tile into bb.tile_count (zeroed here). With `emit`
// (launch_project_raw) they also write the entries themselves into bb.entries[0], up to the
// current capacity (see project_tail); otherwise the binning emits them. `active` (nullable, one
// byte per gaussian): rows with 0 are parked -- no entries, so no contribution and no gradient.
int launch_project_chol(BinBuffers& bb, const Geometry& g, const float* xy, const float* chol,
                        const float* color, const float* weight, int64_t m, int64_t n_per_view,
                        bool want_weights, cudaStream_t s);
int launch_project_conic(BinBuffers& bb, const Geometry& g, const float* xy, const float* conics,
                         const float* colors, const float* weights, const int32_t* rects,
                         const int32_t* view_index, int64_t m, bool want_weights, cudaStream_t s);
// unit_weight: weight = 1 instead of sigmoid(raw weight) (the unit-weight appearance).
int launch_project_raw(BinBuffers& bb, const Geometry& g, const float* raw, int64_t m,
                       int64_t n_per_view, bool emit, const uint8_t* active, bool want_weights,
                       bool unit_weight, cudaStream_t s);
// Bit-exact support rectangles only: rects (M,4) (x0, x1, y0, y1; x1 = x0 - 1 if empty), counts (M,).
int launch_support_rects(const float* xy, const float* chol, int64_t m, int height, int width,
                         int32_t* rects, int64_t* counts, cudaStream_t s);
// raw (planar 9 x M) -> constrained (xy (M,2), chol (M,3), color (M,3), weight (M)); with
// unit_weight every weight is 1.
int launch_build_params(const float* raw, int64_t m, int height, int width, bool unit_weight,
                        float* xy, float* chol, float* color, float* weight, cudaStream_t s);

// ---- binning (binning.cu, sort.cu) --------------------------------------------------------------
// Synchronous binning: scan counts, read the entry count back to the host (synchronises `s`),
// grow the entry buffers to fit, then bin asynchronously -- by tile scatter when every tile list
// fits kSegSortMax, else by the global radix sort. Requires a projection launcher before it.
int bin_entries(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s);
// The two halves of bin_entries: read_bin_stats flags long tile lists, reads the stats back into
// bb.host_stats (synchronises `s`) and sets n_entries, n_pairs and long_tile; bin_known then grows
// the entry buffers only if they cannot hold n_entries and bins (radix path when long_tile).
int read_bin_stats(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s);
int bin_known(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s);
// stats[kStatLongTile] = the longest tile list if any is longer than kSegSortMax (tile counts
// must be complete, i.e. after the projection).
int check_long_tiles(BinBuffers& bb, const Geometry& g, cudaStream_t s);
// Asynchronous binning into the current capacity (no host synchronisation). Tile scatter path:
// scan of tile counts, atomic-slot scatter of gaussian ids (the raster sorts each tile's list);
// radix path (radix = true): emit (tile key, id), stable radix sort, tile ranges. Entries past
// the capacity are dropped and show up as stats[kStatMaxEntries] > capacity; a tile list longer
// than kSegSortMax on the scatter path is flagged by the raster in stats[kStatLongTile].
int bin_entries_async(BinBuffers& bb, const Geometry& g, int64_t m, bool radix, cudaStream_t s);
// Direct placement (fit loop): a projection with ProjOut::list set writes each gaussian id straight
// into its tile's segment, at the position that an atomic on the tile's cursor returns; segments
// are sized from the previous binning's counts with slack. Segments and cursors are double
// buffered (bb.seg, bb.cursor: buffer 0 and 1 of n_tiles each), so that the layout for the next
// placement can run beside a raster that still reads the current one.
// direct_layout computes the segments of buffer `out` from the last binning (after_scatter: from
// tile_end; else from buffer 1 - out: count = cursor - segment start; slack: count + count/4 + 8
// slots, else count) and sets every cursor of buffer `out` to its segment's start; direct_sort
// reads buffer `in` (count = cursor - start), flags a cursor past its segment's end in
// stats[kStatSegOverflow] and sorts the filled segments into bb.ranges. With `order`,
// direct_layout also writes the tiles in descending order of their entry count (a permutation of
// the tiles, ties in any order) for the next raster: heaviest tiles first shortens the launch's
// tail. Up to kDirectMaxTiles tiles.
constexpr int64_t kDirectMaxTiles = int64_t{1} << 20;
bool direct_binning_supported(const Geometry& g);
int direct_layout(BinBuffers& bb, const Geometry& g, bool after_scatter, bool slack, int out,
                  int* order, cudaStream_t s);
int direct_sort(BinBuffers& bb, const Geometry& g, int in, cudaStream_t s);
// Allocate the entry-sized buffers (list, entries, partials[, partial_d]) for `capacity` entries.
int ensure_entry_capacity(BinBuffers& bb, int64_t capacity, bool density, cudaStream_t s);
// Zero per-tile counts before a projection (projection launchers call it).
int reset_tile_counts(BinBuffers& bb, const Geometry& g, cudaStream_t s);
// Stable LSD radix sort of packed entries by their key bits; the count is read on the device.
int radix_sort_entries(uint64_t* buf0, uint64_t* buf1, const unsigned long long* d_n, int64_t cap,
                       int key_bits, int* counts, cudaStream_t s, int* result_sel);
int sort_plan_passes(int key_bits);
size_t sort_counts_bytes();
int key_bits_for(int64_t n_tiles);

// ---- raster (raster.cu) -------------------------------------------------------------------------
enum LossMode : int { kLossMse = 0, kLossMaskWeighted = 1, kLossMaskOnly = 2 };

struct FitRasterArgs {
  const float* targets = nullptr;     // (B, H, W, 3)
  const uint8_t* mask_bits = nullptr; // (B, mask_bytes_per_view) little-endian bits, or null
  int64_t mask_bytes_per_view = 0;
  const float* view_scale = nullptr;  // (B,) loss-gradient scale per view
  int loss_mode = kLossMse;
  double* tile_loss = nullptr;        // (n_tiles, 2): loss numerator, clamped PSNR numerator
  float* render_out = nullptr;        // optional (B, H, W, 3)
  float coverage_coef = 0.f;          // > 0: mask coverage penalty weight / (H * W) (density pass)
  const int* tile_order = nullptr;    // optional: block b rasterises tile tile_order[b]
  // Optional (direct placement): the raster sorts its own tile's list -- tile t's ids are
  // list[seg[t].x, seg[t].x + cursor[t] - seg[t].x), clipped to seg[t].y -- instead of reading
  // the ranges of a tile-sort kernel; block 0 retires the projection's stats.
  const int2* seg = nullptr;
  const int* cursor = nullptr;
  unsigned long long* stats = nullptr;
  // Launch as a programmatic dependent of the Adam kernel before it (only with seg set).
  bool pdl = false;
};

int launch_raster_forward(const BinBuffers& bb, const Geometry& g, float cutoff, float* out,
                          float* den, cudaStream_t s);
int launch_raster_backward(BinBuffers& bb, const Geometry& g, float cutoff, const float* grad_out,
                           const float* grad_den, cudaStream_t s);
int launch_raster_fit(BinBuffers& bb, const Geometry& g, float cutoff, const FitRasterArgs& fa,
                      bool backward, cudaStream_t s);
// Deterministic per-view sum of tile_loss -> dst[(view, 2)].
int launch_loss_reduce(const double* tile_loss, const Geometry& g, double* dst, cudaStream_t s);

// ---- gradient finalisation + Adam (optim.cu) ----------------------------------------------------
int launch_finalize_chol(const BinBuffers& bb, int64_t m, const float* chol, const float* color,
                         const float* weight, bool with_density, float* grad_xy, float* grad_chol,
                         float* grad_color, float* grad_weight, cudaStream_t s);
int launch_finalize_conic(const BinBuffers& bb, int64_t m, const float* conics,
                          const float* colors, const float* weights, bool with_density,
                          float* grad_xy, float* grad_conics, float* grad_colors,
                          float* grad_weights, cudaStream_t s);

struct AdamScalars {
  float neg_step_size;   // -(lr / (1 - beta1^t))
  float inv_bc2_sqrt;    // 1 / sqrt(1 - beta2^t)
  float beta1, beta2, one_minus_beta1, one_minus_beta2, eps;
  int freeze_geometry;
  int unit_weight;  // weight fixed at 1 (no weight parameter)
};
// Per-iteration constants of a fit chunk, read by the Adam kernel from a device table (so the
// launches of every chunk are identical and can be replayed from one CUDA graph).
struct IterScalars {
  AdamScalars adam;
  int log_slot;  // >= 0: also reduce this iteration's loss into log row log_slot
};
// Where the Adam kernel's loss logging reads and writes.
struct LossLog {
  const double* tile_loss;  // (n_tiles, 2) from the raster
  double* log;              // (rows, n_views, 2)
  int n_views, tiles_per_view;
};
// The raw-parameter gradients (planar 9 x M) from the last fit raster's entry moments, no update.
int launch_raw_grad(const BinBuffers& bb, int64_t m, int height, int width, const float* raw,
                    bool unit_weight, bool density, float* grad_out, cudaStream_t s);
// Adam step from the last raster's entry moments, with the constants of table[k]; with
// project_next the updated parameters are also projected (records, spans, counts, offsets,
// stats) for the next iteration's binning: entries for the scatter path, or with `direct` the ids
// placed directly into the tile segments at the tile cursors (see direct_layout).
// `cursors` (direct placement) are the tile cursors of the segment buffer the placement fills
// (bb.cursor + buffer * n_tiles); null projects for the scatter binning. `pdl`: launch as a
// programmatic dependent of the fit raster before it.
int launch_adam_fit(BinBuffers& bb, const Geometry& g, int64_t m, int64_t n_per_view, float* raw,
                    float* m1, float* m2, const IterScalars* table, int k, const LossLog& lg,
                    bool project_next, const uint8_t* active, bool density, int* cursors,
                    bool pdl, cudaStream_t s);
// Whether the Adam kernel's grid for m gaussians is resident all at once on the current device
// (one wave). The fit loop pairs its raster and Adam launches as programmatic dependents only
// then: measured on B200, the pairing shortens a 50k-gaussian fit (one wave of Adam blocks) by
// 2% and lengthens the 560k- and 960k-gaussian multi-view fits (many waves) by 10-20%.
bool adam_single_wave(int64_t m, bool density);

}  // namespace rtgs2d
