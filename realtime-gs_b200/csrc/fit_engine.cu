// Fit engine: the native Stage-1 fit loop, driven from C++ (no Python per iteration).
//
// Per iteration (fit.py:451-482, batched.py:128-145):
//   binning       tile-count scan, count-down scatter, per-tile sort (or the radix fallback)
//   raster fit    forward, L2-loss gradient, backward -> per-entry moments   (1 kernel)
//   adam          entry sums -> chain rule -> Adam on all 9 raw params, then the projection
//                 of the updated parameters for the next iteration; at logging iterations its
//                 first blocks also reduce the loss                           (1 kernel)
// The host advances torch's CosineAnnealingLR recursion in double precision and writes every
// iteration's bias-corrected step size into a small device table once per chunk. Nothing is read
// back inside a chunk of kChunk iterations, so a chunk is one fixed sequence of launches: after a
// chunk of the same shape has run once eagerly, it is captured into a CUDA graph and replayed
// (stage profiling runs eagerly, with events between the stages). At the end of a chunk the
// largest entry count of the chunk is read back; if it exceeded the capacity (entries were
// dropped) or a tile list was too long for the tile sort, the chunk is rolled back to a device
// snapshot of the raw parameters and Adam moments taken at its start and re-run with a larger
// capacity or the radix binning.
#include <cmath>
#include <new>
#include <vector>

#include "../../include/rtgs2d.h"
#include "internal.h"

using namespace rtgs2d;

struct rtgs2d_fit {
  int device = 0;
  int64_t n_views = 0, n = 0, m = 0;
  int height = 0, width = 0;
  rtgs2d_fit_options opt{};
  Geometry geo;
  BinBuffers bb;
  DevBuf raw, m1, m2;  // planar (9, M)
  DevBuf snap;         // raw, m1, m2 at the start of the current chunk (overflow roll-back)
  DevBuf targets;      // (B, H, W, 3)
  DevBuf mask;         // (B, mask_bytes)
  int64_t mask_bytes = 0;
  DevBuf mask_counts;  // (B,) int
  DevBuf view_scale;   // (B,) float
  DevBuf tile_loss;    // (n_tiles, 2) double
  DevBuf log;          // (max_logs, B, 2) double
  DevBuf eval_sums;    // (B, 2) double
  DevBuf grad_raw;     // planar (9, M): rtgs2d_fit_gradients' scratch
  DevBuf active;       // (M,) uint8: 0 = parked row (rtgs2d_fit_set_active); unused until set
  bool use_active = false;
  int64_t max_logs = 0;
  std::vector<int64_t> log_iters;
  int64_t step = 0;
  double lr_current = 0.0;
  double total_pairs = 0.0;
  int64_t last_entries = 0, last_pairs = 0;
  int64_t retries = 0;  // chunks re-run after an entry-capacity overflow or a long tile list
  bool use_radix = false;  // some tile list exceeded the shared-memory sort: bin by radix sort
  int32_t binning = RTGS2D_BINNING_AUTO;  // rtgs2d_fit_set_binning
  bool direct_retry = false;   // the current chunk overflowed a segment: re-run it by scatter
  bool fused_off = false;      // a tile list exceeded the fit raster's own sort: tile-sort kernel
  int64_t segment_retries = 0;
  cudaStream_t side_stream = nullptr;  // segment layout beside the raster
  cudaEvent_t fork_event = nullptr;
  cudaEvent_t join_event = nullptr;
  bool have_targets = false, have_raw = false;
  bool unit_weight = false;  // RTGS2D_APPEARANCE_UNIT_WEIGHT_8P: weight = 1, no weight parameter
  bool scale_uploaded = false;            // view_scale holds the constant scale of the MSE modes
  DevBuf init_status;                     // uint32: failed checks of rtgs2d_fit_set_initial
  uint32_t* host_status = nullptr;        // pinned mirror of init_status
  // per-iteration constants of the current chunk, and the replayable chunks
  DevBuf iter_table;                  // IterScalars[kChunk]
  IterScalars* host_table = nullptr;  // pinned staging for iter_table
  cudaStream_t capture_stream = nullptr;
  struct ChunkGraph {
    std::vector<uintptr_t> key;
    cudaGraphExec_t exec = nullptr;
  };
  std::vector<ChunkGraph> graphs;        // most recent last
  std::vector<uintptr_t> last_eager_key;  // layout of the last chunk that ran eagerly and held
  bool graphs_enabled = true;
  int64_t graph_chunks = 0, eager_chunks = 0;
  // stage timing (rtgs2d_fit_set_profiling)
  bool profiling = false;
  std::vector<cudaEvent_t> events;  // 4 per iteration of the current run
  double bin_ms = 0.0, raster_ms = 0.0, adam_ms = 0.0, pairs_timed = 0.0;
  int64_t iterations_timed = 0;
  void release_events() {
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    events.clear();
  }
  void release_graphs() {
    for (ChunkGraph& g : graphs) cudaGraphExecDestroy(g.exec);
    graphs.clear();
  }
};

namespace {

constexpr int kThreads = 256;

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
unsigned grid_for(int64_t m) { return static_cast<unsigned>((m + kThreads - 1) / kThreads); }

// Reference layout (M,2)/(M,2)/(M,)/(M,3)/(M,) <-> planar (9, M).
__global__ void pack_raw_kernel(int64_t m, const float* __restrict__ xy, const float* __restrict__ diag,
                                const float* __restrict__ off, const float* __restrict__ color,
                                const float* __restrict__ weight, float* __restrict__ raw) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= m) return;
  raw[kXr * m + i] = xy[2 * i];
  raw[kYr * m + i] = xy[2 * i + 1];
  raw[kD0 * m + i] = diag[2 * i];
  raw[kD1 * m + i] = diag[2 * i + 1];
  raw[kOff * m + i] = off[i];
  raw[kCr * m + i] = color[3 * i];
  raw[kCg * m + i] = color[3 * i + 1];
  raw[kCb * m + i] = color[3 * i + 2];
  raw[kWr * m + i] = weight ? weight[i] : 0.f;
}

__global__ void unpack_raw_kernel(int64_t m, const float* __restrict__ raw, float* xy, float* diag,
                                  float* off, float* color, float* weight) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= m) return;
  if (xy) {
    xy[2 * i] = raw[kXr * m + i];
    xy[2 * i + 1] = raw[kYr * m + i];
  }
  if (diag) {
    diag[2 * i] = raw[kD0 * m + i];
    diag[2 * i + 1] = raw[kD1 * m + i];
  }
  if (off) off[i] = raw[kOff * m + i];
  if (color) {
    color[3 * i] = raw[kCr * m + i];
    color[3 * i + 1] = raw[kCg * m + i];
    color[3 * i + 2] = raw[kCb * m + i];
  }
  if (weight) weight[i] = raw[kWr * m + i];
}

// rtgs2d_fit_set_initial: the reference's checks of an initialisation (fit.py:634-676: finite
// fields, means inside the image, Cholesky diagonal above _MIN_DIAG, colours and weights in [0,1])
// and its raw transform (fit.py:375-387: logit of the clamped normalised mean, inverse softplus of
// the diagonal minus _MIN_DIAG, the off-diagonal as is, logit of the clamped colour and weight --
// or, with unit_weight, the amplitude logit(sigmoid(weight_raw) * sigmoid(color_raw)) in the
// colour slots and nothing in the weight slot; non-finite raw values are the reference's
// NonFiniteRawParameterError, fit.py:134-141), one thread per gaussian, written straight into the
// planar raw parameters. Failed checks are OR-ed into *status (RTGS2D_INIT_* bits).
__device__ __forceinline__ float logit_f(float p) { return logf(__fdiv_rn(p, 1.0f - p)); }
__device__ __forceinline__ float softplus_inv_f(float x) { return x + logf(-expm1f(-x)); }
__device__ __forceinline__ float sigmoid_rn(float x) { return __frcp_rn(__fadd_rn(1.0f, expf(-x))); }

__global__ void init_raw_kernel(int64_t m, const float* __restrict__ xy, const float* __restrict__ chol,
                                const float* __restrict__ color, const float* __restrict__ weight,
                                int height, int width, bool unit_weight, float* __restrict__ raw,
                                float* __restrict__ m1, float* __restrict__ m2,
                                unsigned* __restrict__ status) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= m) return;
  const float x = xy[2 * i], y = xy[2 * i + 1];
  const float l11 = chol[3 * i], l21 = chol[3 * i + 1], l22 = chol[3 * i + 2];
  const float c[3] = {color[3 * i], color[3 * i + 1], color[3 * i + 2]};
  const float w = weight[i];
  unsigned bad = 0;
  if (!(isfinite(x) && isfinite(y))) bad |= RTGS2D_INIT_NONFINITE_XY;
  if (!(isfinite(l11) && isfinite(l21) && isfinite(l22))) bad |= RTGS2D_INIT_NONFINITE_CHOL;
  if (!(isfinite(c[0]) && isfinite(c[1]) && isfinite(c[2]))) bad |= RTGS2D_INIT_NONFINITE_COLOR;
  if (!isfinite(w)) bad |= RTGS2D_INIT_NONFINITE_WEIGHT;
  if (!(x >= 0.f && x < static_cast<float>(width) && y >= 0.f && y < static_cast<float>(height))) {
    bad |= RTGS2D_INIT_OUTSIDE;
  }
  if (!(l11 > kMinDiag && l22 > kMinDiag)) bad |= RTGS2D_INIT_DIAG;
  if (!(c[0] >= 0.f && c[0] <= 1.f && c[1] >= 0.f && c[1] <= 1.f && c[2] >= 0.f && c[2] <= 1.f)) {
    bad |= RTGS2D_INIT_COLOR_RANGE;
  }
  if (!(w >= 0.f && w <= 1.f)) bad |= RTGS2D_INIT_WEIGHT_RANGE;
  // torch.clamp: NaN propagates (so a NaN input gives a non-finite raw value, as in the reference)
  auto clamp = [](float v, float lo, float hi) { return v != v ? v : fminf(fmaxf(v, lo), hi); };
  constexpr float kXyLo = 1e-4f, kXyHi = 1.0f - 1e-4f, kLo = 1e-3f, kHi = 1.0f - 1e-3f;
  float r[kRawSlots];
  r[kXr] = logit_f(clamp(__fdiv_rn(x, static_cast<float>(width)), kXyLo, kXyHi));
  r[kYr] = logit_f(clamp(__fdiv_rn(y, static_cast<float>(height)), kXyLo, kXyHi));
  r[kD0] = softplus_inv_f(__fsub_rn(l11, kMinDiag));
  r[kD1] = softplus_inv_f(__fsub_rn(l22, kMinDiag));
  r[kOff] = l21;
  r[kCr] = logit_f(clamp(c[0], kLo, kHi));
  r[kCg] = logit_f(clamp(c[1], kLo, kHi));
  r[kCb] = logit_f(clamp(c[2], kLo, kHi));
  r[kWr] = logit_f(clamp(w, kLo, kHi));
  if (unit_weight) {  // fit.py:384-385: one bounded amplitude per channel, weight fixed at 1
    const float sw = sigmoid_rn(r[kWr]);
    for (int ch = kCr; ch <= kCb; ++ch) r[ch] = logit_f(__fmul_rn(sw, sigmoid_rn(r[ch])));
    r[kWr] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < kRawSlots; ++k) {
    if (!isfinite(r[k])) bad |= RTGS2D_INIT_NONFINITE_RAW;
    raw[k * m + i] = r[k];
    m1[k * m + i] = 0.f;
    m2[k * m + i] = 0.f;
  }
  if (bad) atomicOr(status, bad);
}

__global__ void mask_count_kernel(const uint8_t* __restrict__ bits, int64_t bytes_per_view,
                                  int64_t pixels_per_view, int* __restrict__ counts) {
  __shared__ int s[kThreads];
  const int view = blockIdx.x;
  const uint8_t* v = bits + static_cast<int64_t>(view) * bytes_per_view;
  int c = 0;
  for (int64_t b = threadIdx.x; b < bytes_per_view; b += kThreads) {
    unsigned byte = v[b];
    const int64_t valid = pixels_per_view - 8 * b;  // bits past the last pixel are padding
    if (valid < 8) byte &= (1u << valid) - 1u;
    c += __popc(byte);
  }
  s[threadIdx.x] = c;
  __syncthreads();
  for (int stride = kThreads / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) s[threadIdx.x] += s[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[view] = s[0];
}

int check_fit(const rtgs2d_fit* f) {
  if (!f) return set_error(RTGS2D_ERR_INVALID, "fit is NULL");
  int dev = -1;
  RTGS_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != f->device) {
    return set_error(RTGS2D_ERR_INVALID, "fit engine belongs to device " + std::to_string(f->device) +
                                             ", current device is " + std::to_string(dev));
  }
  return 0;
}

bool is_log_iter(const rtgs2d_fit_options& o, int64_t it) {
  if (o.log_every > 0 && it % o.log_every == 0) return true;
  if (it == o.iterations - 1) return true;
  if (o.check_every > 0 && (it + 1) % o.check_every == 0) return true;
  return false;
}

// torch.optim.lr_scheduler.CosineAnnealingLR.get_lr() for last_epoch = epoch >= 1 (recursive form).
double cosine_next_lr(double lr, double base_lr, double eta_min, int64_t epoch, int64_t t_max) {
  const int64_t period = 2 * t_max;
  int64_t r = (epoch - 1 - t_max) % period;
  if (r < 0) r += period;
  if (r == 0) {
    return lr + (base_lr - eta_min) * (1.0 - std::cos(M_PI / static_cast<double>(t_max))) / 2.0;
  }
  return (1.0 + std::cos(M_PI * static_cast<double>(epoch) / static_cast<double>(t_max))) /
             (1.0 + std::cos(M_PI * static_cast<double>(epoch - 1) / static_cast<double>(t_max))) *
             (lr - eta_min) +
         eta_min;
}

int ensure_events(rtgs2d_fit* f, size_t need) {
  while (f->events.size() < need) {
    cudaEvent_t e;
    RTGS_CUDA(cudaEventCreate(&e), "cudaEventCreate");
    f->events.push_back(e);
  }
  return 0;
}

bool coverage(const rtgs2d_fit* f) { return f->opt.mask_coverage_weight > 0.0; }

// Bin by radix sort: chosen by the caller, or after a tile list too long for the tile sort.
bool radix(const rtgs2d_fit* f) { return f->use_radix || f->binning == RTGS2D_BINNING_RADIX; }

// Direct placement for this chunk: not on the radix path, at most 2^20 tiles, and not right after
// a chunk that overflowed a tile segment (that chunk re-runs with the scatter binning).
bool direct_chunk(const rtgs2d_fit* f) {
  const bool mode = f->binning == RTGS2D_BINNING_AUTO || f->binning == RTGS2D_BINNING_TIGHT ||
                    f->binning == RTGS2D_BINNING_SORTED;
  return mode && !f->direct_retry && !radix(f) && direct_binning_supported(f->geo);
}

// In a direct chunk, the fit raster sorts its own tile's list (no tile-sort kernel) unless the
// caller chose the separate sort, or a list of this fit exceeded kFusedSortMax.
bool fused_sort(const rtgs2d_fit* f) {
  return direct_chunk(f) && f->binning != RTGS2D_BINNING_SORTED && !f->fused_off;
}

// The stream and events that run the segment layout beside the raster.
int ensure_side_stream(rtgs2d_fit* f) {
  if (!f->side_stream) {
    RTGS_CUDA(cudaStreamCreateWithFlags(&f->side_stream, cudaStreamNonBlocking), "side stream");
  }
  if (!f->fork_event) RTGS_CUDA(cudaEventCreateWithFlags(&f->fork_event, cudaEventDisableTiming), "fork event");
  if (!f->join_event) RTGS_CUDA(cudaEventCreateWithFlags(&f->join_event, cudaEventDisableTiming), "join event");
  return 0;
}

// The list holds the direct segments: entries + a quarter + 8 slots per tile, with headroom.
int ensure_segment_room(rtgs2d_fit* f, cudaStream_t s) {
  if (!direct_binning_supported(f->geo)) return 0;
  const int64_t cap = f->bb.capacity;
  const size_t want = static_cast<size_t>(cap + cap / 4 + 16 * f->geo.n_tiles()) * sizeof(uint32_t);
  RTGS_TRY(f->bb.seg.ensure(static_cast<size_t>(2 * f->geo.n_tiles()) * sizeof(int2), s));
  RTGS_TRY(f->bb.cursor.ensure(static_cast<size_t>(2 * f->geo.n_tiles()) * sizeof(int), s));
  RTGS_TRY(f->bb.tile_order.ensure(static_cast<size_t>(2 * f->geo.n_tiles()) * sizeof(int), s));
  return f->bb.list.ensure(want, s);
}

const uint8_t* active_rows(const rtgs2d_fit* f) {
  return f->use_active ? f->active.as<uint8_t>() : nullptr;
}

// Rows `rows[0..n)` of the planar raw parameters: write the given values (reference layouts, like
// rtgs2d_fit_set_raw; all null = keep the values) and zero both Adam moments. Indices outside
// [0, m) are skipped.
__global__ void write_rows_kernel(int64_t m, const int64_t* __restrict__ rows, int64_t n,
                                  const float* __restrict__ xy, const float* __restrict__ diag,
                                  const float* __restrict__ off, const float* __restrict__ color,
                                  const float* __restrict__ weight, float* __restrict__ raw,
                                  float* __restrict__ m1, float* __restrict__ m2) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (r >= n) return;
  const int64_t i = rows[r];
  if (i < 0 || i >= m) return;
  if (xy) {
    raw[kXr * m + i] = xy[2 * r];
    raw[kYr * m + i] = xy[2 * r + 1];
    raw[kD0 * m + i] = diag[2 * r];
    raw[kD1 * m + i] = diag[2 * r + 1];
    raw[kOff * m + i] = off[r];
    raw[kCr * m + i] = color[3 * r];
    raw[kCg * m + i] = color[3 * r + 1];
    raw[kCb * m + i] = color[3 * r + 2];
    raw[kWr * m + i] = weight ? weight[r] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < kRawSlots; ++k) {
    m1[k * m + i] = 0.f;
    m2[k * m + i] = 0.f;
  }
}

// Projection + synchronous binning (exact entry count; used outside the iteration loop).
int project_and_bin(rtgs2d_fit* f, cudaStream_t s) {
  RTGS_TRY(launch_project_raw(f->bb, f->geo, f->raw.as<float>(), f->m, f->n, false, active_rows(f),
                              coverage(f), f->unit_weight, s));
  RTGS_TRY(bin_entries(f->bb, f->geo, f->m, s));
  f->last_entries = f->bb.n_entries;
  f->last_pairs = f->bb.n_pairs;
  return 0;
}

constexpr int64_t kChunk = 64;

// Copy raw/m1/m2 to the snapshot (to_snap) or back.
int snapshot(rtgs2d_fit* f, bool to_snap, cudaStream_t s) {
  const size_t bytes = static_cast<size_t>(kRawSlots) * (f->m > 0 ? f->m : 1) * sizeof(float);
  RTGS_TRY(f->snap.ensure(3 * bytes, s));
  char* sp = f->snap.as<char>();
  DevBuf* bufs[3] = {&f->raw, &f->m1, &f->m2};
  for (int k = 0; k < 3; ++k) {
    void* dst = to_snap ? static_cast<void*>(sp + k * bytes) : bufs[k]->ptr;
    const void* src = to_snap ? static_cast<const void*>(bufs[k]->ptr) : static_cast<const void*>(sp + k * bytes);
    RTGS_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s), "snapshot copy");
  }
  return 0;
}

FitRasterArgs raster_args(rtgs2d_fit* f) {
  FitRasterArgs fa;
  fa.targets = f->targets.as<float>();
  fa.mask_bits = f->mask.as<uint8_t>();
  fa.mask_bytes_per_view = f->mask_bytes;
  fa.view_scale = f->view_scale.as<float>();
  fa.loss_mode = f->opt.loss_mode;
  fa.tile_loss = f->tile_loss.as<double>();
  fa.render_out = nullptr;
  // mean over the H x W pixels of coverage * (1 - mask), times the weight (fit.py:566-572)
  fa.coverage_coef = static_cast<float>(f->opt.mask_coverage_weight /
                                        (static_cast<double>(f->height) * f->width));
  return fa;
}


// Everything a captured chunk depends on besides the contents of device memory: its length, the
// binning path and the address and size of every buffer its launches use.
std::vector<uintptr_t> chunk_key(const rtgs2d_fit* f, int64_t chunk) {
  const BinBuffers& bb = f->bb;
  std::vector<uintptr_t> k = {static_cast<uintptr_t>(chunk), static_cast<uintptr_t>(radix(f)),
                              static_cast<uintptr_t>(bb.capacity), static_cast<uintptr_t>(f->use_active),
                              static_cast<uintptr_t>(direct_chunk(f)), static_cast<uintptr_t>(fused_sort(f)),
                              static_cast<uintptr_t>(adam_single_wave(f->m, coverage(f))),
                              static_cast<uintptr_t>(f->unit_weight)};
  for (const DevBuf* b : {&bb.records, &bb.weights, &bb.spans, &bb.counts, &bb.offsets, &bb.list,
                          &bb.tile_count, &bb.tile_end, &bb.seg, &bb.cursor, &bb.tile_order, &bb.entries[0], &bb.entries[1], &bb.ranges,
                          &bb.partials, &bb.partial_d, &bb.cub_temp, &bb.sort_counts, &bb.stats,
                          &f->raw, &f->m1, &f->m2, &f->targets, &f->mask, &f->view_scale,
                          &f->tile_loss, &f->log, &f->iter_table, &f->active}) {
    k.push_back(reinterpret_cast<uintptr_t>(b->ptr));
    k.push_back(static_cast<uintptr_t>(b->bytes));
  }
  return k;
}

// The launches of one chunk: the chunk's first projection, then per iteration binning, raster and
// Adam (+ projection of the next iteration, except after the last). With `ev` (profiling), four
// events per iteration bracket the stages. `capturing`: `s` is in stream capture.
int enqueue_chunk(rtgs2d_fit* f, int64_t chunk, cudaStream_t s, cudaEvent_t* ev, bool capturing) {
  BinBuffers& bb = f->bb;
  const LossLog lg{f->tile_loss.as<double>(), f->log.as<double>(), static_cast<int>(f->n_views),
                   f->geo.tiles_per_view};
  const FitRasterArgs fa = raster_args(f);
  // External records: under stream capture they become event-record nodes of the graph (a plain
  // record would only order the capture), so the replayed chunk still times its stages.
  auto record = [s, capturing](cudaEvent_t e) {
    return capturing ? cudaEventRecordWithFlags(e, s, cudaEventRecordExternal) : cudaEventRecord(e, s);
  };
  RTGS_TRY(launch_project_raw(bb, f->geo, f->raw.as<float>(), f->m, f->n, true, active_rows(f),
                              coverage(f), f->unit_weight, s));
  // Binning: the chunk's first iteration scatters the projection's entries; with direct placement
  // (direct_chunk), every later projection (fused into Adam) writes its ids straight into tile
  // segments sized from the previous binning, and the binning is just the per-tile sort: done by
  // the fit raster itself (fused_sort), or by the tile-sort kernel.
  // The layout of the next segments runs on the side stream beside the raster and joins before
  // Adam (the projection that fills them). Segments, cursors and tile orders alternate between two
  // buffers: the layout of iteration k writes buffer (k + 1) & 1 while raster k reads buffer k & 1.
  const bool direct = direct_chunk(f);
  const bool fuse = fused_sort(f);
  // Raster and Adam as programmatic dependents of each other: only with a single wave of Adam blocks.
  const bool pdl = fuse && adam_single_wave(f->m, coverage(f));
  if (direct) RTGS_TRY(ensure_side_stream(f));
  const int64_t n_tiles = f->geo.n_tiles();
  int* orders = bb.tile_order.as<int>();
  for (int64_t k = 0; k < chunk; ++k) {
    cudaEvent_t* e = ev ? ev + 4 * k : nullptr;
    const int cur = static_cast<int>(k & 1), next = static_cast<int>((k + 1) & 1);
    if (e) RTGS_CUDA(record(e[0]), "event record");
    if (direct && k > 0) {
      if (!fuse) RTGS_TRY(direct_sort(bb, f->geo, cur, s));
    } else {
      RTGS_TRY(bin_entries_async(bb, f->geo, f->m, radix(f), s));
    }
    const bool layout = direct && k + 1 < chunk;
    if (layout) {
      RTGS_CUDA(cudaEventRecord(f->fork_event, s), "fork record");
      RTGS_CUDA(cudaStreamWaitEvent(f->side_stream, f->fork_event, 0), "fork wait");
      RTGS_TRY(direct_layout(bb, f->geo, k == 0, f->binning != RTGS2D_BINNING_TIGHT, next,
                             orders + next * n_tiles, f->side_stream));
      RTGS_CUDA(cudaEventRecord(f->join_event, f->side_stream), "join record");
    }
    if (e) RTGS_CUDA(record(e[1]), "event record");
    FitRasterArgs fk = fa;
    if (direct && k > 0) {
      fk.tile_order = orders + cur * n_tiles;
      if (fuse) {
        fk.seg = bb.seg.as<int2>() + cur * n_tiles;
        fk.cursor = bb.cursor.as<int>() + cur * n_tiles;
        fk.stats = bb.stats.as<unsigned long long>();
        fk.pdl = pdl;
      }
    }
    RTGS_TRY(launch_raster_fit(bb, f->geo, kCutoff, fk, true, s));
    if (e) RTGS_CUDA(record(e[2]), "event record");
    if (layout) RTGS_CUDA(cudaStreamWaitEvent(s, f->join_event, 0), "join wait");
    RTGS_TRY(launch_adam_fit(bb, f->geo, f->m, f->n, f->raw.as<float>(), f->m1.as<float>(),
                             f->m2.as<float>(), f->iter_table.as<IterScalars>(),
                             static_cast<int>(k), lg, k + 1 < chunk, active_rows(f), coverage(f),
                             layout ? bb.cursor.as<int>() + next * n_tiles : nullptr, pdl, s));
    if (e) RTGS_CUDA(record(e[3]), "event record");
  }
  return 0;
}

// Capture the chunk into a graph (nothing runs). Returns null if capture is not possible (the
// caller then runs the chunk eagerly); errors of the attempt are cleared.
cudaGraphExec_t capture_chunk(rtgs2d_fit* f, int64_t chunk, cudaEvent_t* ev) {
  if (!f->capture_stream &&
      cudaStreamCreateWithFlags(&f->capture_stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaStreamBeginCapture(f->capture_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  const int rc = enqueue_chunk(f, chunk, f->capture_stream, ev, true);
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(f->capture_stream, &graph);
  cudaGraphExec_t exec = nullptr;
  if (rc == 0 && end == cudaSuccess && graph) {
    if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) exec = nullptr;
  }
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  return exec;
}

// Run one chunk: replay its graph when a chunk of the same key has already run eagerly, else run
// it eagerly. With stage profiling the event records are part of the chunk (and of its graph).
int run_chunk(rtgs2d_fit* f, int64_t chunk, cudaStream_t s) {
  cudaEvent_t* ev = nullptr;
  if (f->profiling) {
    RTGS_TRY(ensure_events(f, static_cast<size_t>(4 * kChunk)));  // fixed size: a stable address
    ev = f->events.data();
  }
  std::vector<uintptr_t> key = chunk_key(f, chunk);
  key.push_back(reinterpret_cast<uintptr_t>(ev));
  if (!f->graphs_enabled) key.clear();  // matches no graph and no eager key
  for (auto& g : f->graphs) {
    if (g.key == key) {
      f->graph_chunks += 1;
      return check_cuda(cudaGraphLaunch(g.exec, s), "chunk graph launch");
    }
  }
  if (!key.empty() && key == f->last_eager_key) {
    cudaGraphExec_t exec = capture_chunk(f, chunk, ev);
    if (exec) {
      constexpr size_t kMaxGraphs = 4;
      if (f->graphs.size() == kMaxGraphs) {
        cudaGraphExecDestroy(f->graphs.front().exec);
        f->graphs.erase(f->graphs.begin());
      }
      f->graphs.push_back({key, exec});
      f->graph_chunks += 1;
      return check_cuda(cudaGraphLaunch(exec, s), "chunk graph launch");
    }
  }
  f->eager_chunks += 1;
  RTGS_TRY(enqueue_chunk(f, chunk, s, ev, false));
  // The buffers as the next chunk of this shape finds them.
  f->last_eager_key = chunk_key(f, chunk);
  f->last_eager_key.push_back(reinterpret_cast<uintptr_t>(ev));
  return 0;
}

}  // namespace

extern "C" {

int rtgs2d_fit_create(int64_t n_views, int64_t n, int64_t height, int64_t width,
                      const rtgs2d_fit_options* options, rtgs2d_fit** out) {
  if (!out || !options) return set_error(RTGS2D_ERR_INVALID, "out/options is NULL");
  *out = nullptr;
  if (n_views <= 0 || n < 0 || height <= 0 || width <= 0) {
    return set_error(RTGS2D_ERR_INVALID, "n_views, height, width must be positive and n >= 0");
  }
  if (height > 32768 || width > 32768 || n_views * n > INT32_MAX) {
    return set_error(RTGS2D_ERR_CAPACITY, "problem too large for 32-bit indexing");
  }
  if (options->iterations < 0 || !(options->lr > 0.0)) {
    return set_error(RTGS2D_ERR_INVALID, "iterations must be >= 0 and lr > 0");
  }
  if (options->loss_mode < RTGS2D_LOSS_MSE || options->loss_mode > RTGS2D_LOSS_MASK_ONLY) {
    return set_error(RTGS2D_ERR_INVALID, "unknown loss_mode");
  }
  if (!(options->mask_coverage_weight >= 0.0)) {
    return set_error(RTGS2D_ERR_INVALID, "mask_coverage_weight must be non-negative");
  }
  if (options->mask_coverage_weight > 0.0 && options->loss_mode == RTGS2D_LOSS_MSE) {
    return set_error(RTGS2D_ERR_INVALID, "mask_coverage_weight requires a mask");
  }
  rtgs2d_fit* f = new (std::nothrow) rtgs2d_fit();
  if (!f) return set_error(RTGS2D_ERR_ALLOC, "host allocation failed");
  int rc = 0;
  do {
    if ((rc = check_cuda(cudaGetDevice(&f->device), "cudaGetDevice"))) break;
    f->n_views = n_views;
    f->n = n;
    f->m = n_views * n;
    f->height = static_cast<int>(height);
    f->width = static_cast<int>(width);
    f->opt = *options;
    f->geo = make_geometry(static_cast<int>(n_views), f->height, f->width);
    f->lr_current = options->lr;
    f->mask_bytes = (height * width + 7) / 8;
    for (int64_t it = 0; it < options->iterations; ++it) f->max_logs += is_log_iter(options[0], it);
    const size_t mm = static_cast<size_t>(f->m > 0 ? f->m : 1);
    cudaStream_t s = nullptr;
    if ((rc = f->raw.ensure(kRawSlots * mm * sizeof(float), s))) break;
    if ((rc = f->m1.ensure(kRawSlots * mm * sizeof(float), s))) break;
    if ((rc = f->m2.ensure(kRawSlots * mm * sizeof(float), s))) break;
    if ((rc = f->targets.ensure(static_cast<size_t>(n_views * height * width * 3) * sizeof(float), s))) break;
    if ((rc = f->view_scale.ensure(static_cast<size_t>(n_views) * sizeof(float), s))) break;
    if ((rc = f->mask_counts.ensure(static_cast<size_t>(n_views) * sizeof(int), s))) break;
    if ((rc = f->tile_loss.ensure(static_cast<size_t>(f->geo.n_tiles()) * 2 * sizeof(double), s))) break;
    if ((rc = f->eval_sums.ensure(static_cast<size_t>(n_views) * 2 * sizeof(double), s))) break;
    if ((rc = f->log.ensure(static_cast<size_t>(f->max_logs > 0 ? f->max_logs : 1) * n_views * 2 * sizeof(double), s))) break;
    if (options->loss_mode != RTGS2D_LOSS_MSE) {
      if ((rc = f->mask.ensure(static_cast<size_t>(n_views * f->mask_bytes), s))) break;
    }
  } while (false);
  if (rc) {
    delete f;
    return rc;
  }
  *out = f;
  return RTGS2D_OK;
}

int rtgs2d_fit_destroy(rtgs2d_fit* fit) {
  if (!fit) return RTGS2D_OK;
  const int dev = fit->device;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  fit->raw.release();
  fit->m1.release();
  fit->m2.release();
  fit->targets.release();
  fit->mask.release();
  fit->mask_counts.release();
  fit->view_scale.release();
  fit->tile_loss.release();
  fit->log.release();
  fit->eval_sums.release();
  fit->active.release();
  fit->snap.release();
  fit->iter_table.release();
  fit->release_events();
  fit->release_graphs();
  if (fit->capture_stream) cudaStreamDestroy(fit->capture_stream);
  if (fit->side_stream) cudaStreamDestroy(fit->side_stream);
  if (fit->fork_event) cudaEventDestroy(fit->fork_event);
  if (fit->join_event) cudaEventDestroy(fit->join_event);
  if (fit->host_table) cudaFreeHost(fit->host_table);
  if (fit->host_status) cudaFreeHost(fit->host_status);
  fit->init_status.release();
  delete fit;
  if (prev != dev) cudaSetDevice(prev);
  return RTGS2D_OK;
}

int rtgs2d_fit_set_targets(rtgs2d_fit* f, const float* targets, const uint8_t* mask_bits,
                           void* stream) {
  RTGS_TRY(check_fit(f));
  if (!targets) return set_error(RTGS2D_ERR_INVALID, "targets is NULL");
  const bool masked = f->opt.loss_mode != RTGS2D_LOSS_MSE;
  if (masked && !mask_bits) return set_error(RTGS2D_ERR_INVALID, "mask loss mode needs mask_bits");
  cudaStream_t s = as_stream(stream);
  const size_t tbytes = static_cast<size_t>(f->n_views) * f->height * f->width * 3 * sizeof(float);
  RTGS_CUDA(cudaMemcpyAsync(f->targets.ptr, targets, tbytes, cudaMemcpyDeviceToDevice, s),
            "copy targets");
  std::vector<float> scale(static_cast<size_t>(f->n_views));
  const double numel = 3.0 * f->height * f->width;
  if (f->opt.loss_mode == RTGS2D_LOSS_MASK_ONLY) {
    RTGS_CUDA(cudaMemcpyAsync(f->mask.ptr, mask_bits, static_cast<size_t>(f->n_views * f->mask_bytes),
                              cudaMemcpyDeviceToDevice, s),
              "copy mask");
    mask_count_kernel<<<static_cast<unsigned>(f->n_views), kThreads, 0, s>>>(
        f->mask.as<uint8_t>(), f->mask_bytes, static_cast<int64_t>(f->height) * f->width,
        f->mask_counts.as<int>());
    RTGS_CUDA(cudaGetLastError(), "mask_count_kernel");
    std::vector<int> counts(static_cast<size_t>(f->n_views));
    RTGS_CUDA(cudaMemcpyAsync(counts.data(), f->mask_counts.ptr, counts.size() * sizeof(int),
                              cudaMemcpyDeviceToHost, s),
              "mask counts readback");
    RTGS_CUDA(cudaStreamSynchronize(s), "mask counts sync");
    for (size_t b = 0; b < counts.size(); ++b) {
      scale[b] = counts[b] > 0 ? static_cast<float>(2.0 / (3.0 * counts[b])) : 0.0f;
    }
  } else {
    if (masked) {
      RTGS_CUDA(cudaMemcpyAsync(f->mask.ptr, mask_bits, static_cast<size_t>(f->n_views * f->mask_bytes),
                                cudaMemcpyDeviceToDevice, s),
                "copy mask");
    }
    // The scale of these modes is a constant of the engine: uploaded by the first call only.
    if (f->scale_uploaded) {
      f->have_targets = true;
      return RTGS2D_OK;
    }
    for (auto& v : scale) v = static_cast<float>(2.0 / numel);
  }
  RTGS_CUDA(cudaMemcpyAsync(f->view_scale.ptr, scale.data(), scale.size() * sizeof(float),
                            cudaMemcpyHostToDevice, s),
            "view scale upload");
  RTGS_CUDA(cudaStreamSynchronize(s), "set_targets sync");  // `scale` is host stack memory
  f->scale_uploaded = f->opt.loss_mode != RTGS2D_LOSS_MASK_ONLY;
  f->have_targets = true;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_raw(rtgs2d_fit* f, const float* xy_raw, const float* diag_raw,
                       const float* off_raw, const float* color_raw, const float* weight_raw,
                       void* stream) {
  RTGS_TRY(check_fit(f));
  if (f->m > 0 && (!xy_raw || !diag_raw || !off_raw || !color_raw || (!weight_raw && !f->unit_weight))) {
    return set_error(RTGS2D_ERR_INVALID, "raw parameter pointer is NULL");
  }
  cudaStream_t s = as_stream(stream);
  const size_t bytes = static_cast<size_t>(kRawSlots) * (f->m > 0 ? f->m : 1) * sizeof(float);
  RTGS_CUDA(cudaMemsetAsync(f->m1.ptr, 0, bytes, s), "zero exp_avg");
  RTGS_CUDA(cudaMemsetAsync(f->m2.ptr, 0, bytes, s), "zero exp_avg_sq");
  if (f->m > 0) {
    pack_raw_kernel<<<grid_for(f->m), kThreads, 0, s>>>(f->m, xy_raw, diag_raw, off_raw, color_raw,
                                                        weight_raw, f->raw.as<float>());
    RTGS_CUDA(cudaGetLastError(), "pack_raw_kernel");
  }
  f->step = 0;
  f->lr_current = f->opt.lr;
  f->log_iters.clear();
  f->total_pairs = 0.0;
  f->have_raw = true;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_initial(rtgs2d_fit* f, const float* xy, const float* chol, const float* color,
                           const float* weight, uint32_t* status, void* stream) {
  RTGS_TRY(check_fit(f));
  if (!status) return set_error(RTGS2D_ERR_INVALID, "status is NULL");
  if (f->m > 0 && (!xy || !chol || !color || !weight)) {
    return set_error(RTGS2D_ERR_INVALID, "initial parameter pointer is NULL");
  }
  cudaStream_t s = as_stream(stream);
  if (!f->host_status) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&f->host_status), sizeof(uint32_t)), "pinned status");
  }
  RTGS_TRY(f->init_status.ensure(sizeof(uint32_t), s));
  RTGS_CUDA(cudaMemsetAsync(f->init_status.ptr, 0, sizeof(uint32_t), s), "zero status");
  if (f->m > 0) {
    init_raw_kernel<<<grid_for(f->m), kThreads, 0, s>>>(f->m, xy, chol, color, weight, f->height,
                                                        f->width, f->unit_weight, f->raw.as<float>(),
                                                        f->m1.as<float>(), f->m2.as<float>(),
                                                        f->init_status.as<unsigned>());
    RTGS_CUDA(cudaGetLastError(), "init_raw_kernel");
  }
  RTGS_CUDA(cudaMemcpyAsync(f->host_status, f->init_status.ptr, sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
            "status readback");
  RTGS_CUDA(cudaStreamSynchronize(s), "set_initial sync");
  *status = *f->host_status;
  f->step = 0;
  f->lr_current = f->opt.lr;
  f->log_iters.clear();
  f->total_pairs = 0.0;
  f->have_raw = (*status & RTGS2D_INIT_NONFINITE_RAW) == 0;
  return RTGS2D_OK;
}

int rtgs2d_fit_run(rtgs2d_fit* f, int64_t n_iterations, void* stream) {
  RTGS_TRY(check_fit(f));
  if (!f->have_targets || !f->have_raw) {
    return set_error(RTGS2D_ERR_INVALID, "set targets and raw parameters before running");
  }
  cudaStream_t s = as_stream(stream);
  const double base_lr = f->opt.lr;
  const double eta_min = f->opt.lr * 0.1;
  const int64_t t_max = f->opt.iterations;
  BinBuffers& bb = f->bb;
  if (!bb.host_stats) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&bb.host_stats),
                             kStatSlots * sizeof(unsigned long long)),
              "pinned stats");
  }
  if (!f->host_table) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&f->host_table), kChunk * sizeof(IterScalars)),
              "pinned iteration table");
  }
  RTGS_TRY(f->iter_table.ensure(kChunk * sizeof(IterScalars), s));
  if (!bb.stats.ptr) {
    RTGS_TRY(bb.stats.ensure(kStatSlots * sizeof(unsigned long long), s));
    RTGS_CUDA(cudaMemsetAsync(bb.stats.ptr, 0, kStatSlots * sizeof(unsigned long long), s),
              "zero stats");
  }
  // Initial capacity: the current entry count with headroom (gaussians grow and shrink).
  if (bb.capacity == 0) {
    RTGS_TRY(project_and_bin(f, s));
    RTGS_TRY(ensure_entry_capacity(bb, f->last_entries + f->last_entries / 2 + 4096, coverage(f), s));
  }
  RTGS_TRY(ensure_segment_room(f, s));
  int64_t remaining = t_max - f->step < n_iterations ? t_max - f->step : n_iterations;
  while (remaining > 0) {
    const int64_t chunk = remaining < kChunk ? remaining : kChunk;
    // Host state to restore if the chunk must be re-run.
    const int64_t step0 = f->step;
    const double lr0 = f->lr_current;
    const size_t logs0 = f->log_iters.size();
    // Per-iteration constants: Adam's bias corrections at the current learning rate, the log row.
    for (int64_t k = 0; k < chunk; ++k) {
      const int64_t it = f->step;
      IterScalars& row = f->host_table[k];
      const double t = static_cast<double>(it + 1);
      const double bc1 = 1.0 - std::pow(0.9, t);
      const double bc2 = 1.0 - std::pow(0.999, t);
      row.adam.neg_step_size = static_cast<float>(-(f->lr_current / bc1));
      row.adam.inv_bc2_sqrt = static_cast<float>(1.0 / std::sqrt(bc2));
      row.adam.beta1 = 0.9f;
      row.adam.beta2 = 0.999f;
      row.adam.one_minus_beta1 = static_cast<float>(1.0 - 0.9);
      row.adam.one_minus_beta2 = static_cast<float>(1.0 - 0.999);
      row.adam.eps = 1e-8f;
      row.adam.freeze_geometry = f->opt.freeze_geometry;
      row.adam.unit_weight = f->unit_weight;
      row.log_slot = -1;
      if (is_log_iter(f->opt, it)) {
        const int64_t slot = static_cast<int64_t>(f->log_iters.size());
        if (slot < f->max_logs) {
          row.log_slot = static_cast<int>(slot);
          f->log_iters.push_back(it);
        }
      }
      f->step += 1;
      f->lr_current = cosine_next_lr(f->lr_current, base_lr, eta_min, f->step, t_max);
    }
    RTGS_CUDA(cudaMemcpyAsync(f->iter_table.ptr, f->host_table,
                              static_cast<size_t>(chunk) * sizeof(IterScalars),
                              cudaMemcpyHostToDevice, s),
              "iteration table upload");
    RTGS_TRY(snapshot(f, true, s));
    RTGS_CUDA(cudaMemsetAsync(bb.stats.as<unsigned long long>() + kStatPairsTotal, 0,
                              (kStatSlots - kStatPairsTotal) * sizeof(unsigned long long), s),
              "reset chunk stats");
    RTGS_TRY(run_chunk(f, chunk, s));
    RTGS_CUDA(cudaMemcpyAsync(bb.host_stats, bb.stats.ptr, kStatSlots * sizeof(unsigned long long),
                              cudaMemcpyDeviceToHost, s),
              "chunk stats readback");
    RTGS_CUDA(cudaStreamSynchronize(s), "chunk sync");
    const int64_t max_entries = static_cast<int64_t>(bb.host_stats[kStatMaxEntries]);
    const bool long_tile = !radix(f) && bb.host_stats[kStatLongTile] > 0;
    const bool seg_full = bb.host_stats[kStatSegOverflow] > 0;
    const bool fused_long = bb.host_stats[kStatFusedLong] > 0;
    if (max_entries > bb.capacity || long_tile || seg_full || fused_long) {
      // Entries were dropped in this chunk: roll back and re-run it with room for them.
      if (max_entries > INT32_MAX) return set_error(RTGS2D_ERR_CAPACITY, "more than 2^31 tile entries");
      RTGS_TRY(snapshot(f, false, s));
      f->step = step0;
      f->lr_current = lr0;
      f->log_iters.resize(logs0);
      f->retries += 1;
      if (long_tile) f->use_radix = true;  // a tile list too long for the tile sort
      if (fused_long) f->fused_off = true;  // a tile list too long for the raster's own sort
      if (seg_full) {                      // a tile segment too short: this chunk bins by scatter
        f->direct_retry = true;
        f->segment_retries += 1;
      }
      if (max_entries > bb.capacity) {
        RTGS_TRY(ensure_entry_capacity(bb, max_entries + max_entries / 2 + 4096, coverage(f), s));
        RTGS_TRY(ensure_segment_room(f, s));
      }
      continue;
    }
    f->direct_retry = false;
    f->last_entries = static_cast<int64_t>(bb.host_stats[kStatLastEntries]);
    f->last_pairs = static_cast<int64_t>(bb.host_stats[kStatLastPairs]);
    const double chunk_pairs = static_cast<double>(bb.host_stats[kStatPairsTotal]);
    f->total_pairs += chunk_pairs;
    if (f->profiling) {
      for (int64_t k = 0; k < chunk; ++k) {
        float t01 = 0.f, t12 = 0.f, t23 = 0.f;
        const size_t e = static_cast<size_t>(4 * k);
        RTGS_CUDA(cudaEventElapsedTime(&t01, f->events[e], f->events[e + 1]), "elapsed");
        RTGS_CUDA(cudaEventElapsedTime(&t12, f->events[e + 1], f->events[e + 2]), "elapsed");
        RTGS_CUDA(cudaEventElapsedTime(&t23, f->events[e + 2], f->events[e + 3]), "elapsed");
        f->bin_ms += t01;
        f->raster_ms += t12;
        f->adam_ms += t23;
      }
      f->pairs_timed += chunk_pairs;
      f->iterations_timed += chunk;
    }
    remaining -= chunk;
  }
  return RTGS2D_OK;
}

int rtgs2d_fit_reserve(rtgs2d_fit* f, int64_t entries, void* stream) {
  RTGS_TRY(check_fit(f));
  if (entries < 0 || entries > INT32_MAX) return set_error(RTGS2D_ERR_CAPACITY, "entries out of range");
  if (entries <= f->bb.capacity) return RTGS2D_OK;
  return ensure_entry_capacity(f->bb, entries, coverage(f), as_stream(stream));
}

int rtgs2d_fit_capacity(const rtgs2d_fit* f, int64_t* entries, int64_t* retries) {
  if (!f) return set_error(RTGS2D_ERR_INVALID, "fit is NULL");
  if (entries) *entries = f->bb.capacity;
  if (retries) *retries = f->retries;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_profiling(rtgs2d_fit* f, int32_t enable) {
  RTGS_TRY(check_fit(f));
  f->profiling = enable != 0;
  f->bin_ms = f->raster_ms = f->adam_ms = f->pairs_timed = 0.0;
  f->iterations_timed = 0;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_active(rtgs2d_fit* f, const uint8_t* active, void* stream) {
  RTGS_TRY(check_fit(f));
  if (!active) {
    f->use_active = false;
    return RTGS2D_OK;
  }
  cudaStream_t s = as_stream(stream);
  RTGS_TRY(f->active.ensure(static_cast<size_t>(f->m > 0 ? f->m : 1), s));
  if (f->m > 0) {
    RTGS_CUDA(cudaMemcpyAsync(f->active.ptr, active, static_cast<size_t>(f->m), cudaMemcpyDeviceToDevice, s),
              "copy active rows");
  }
  f->use_active = true;
  return RTGS2D_OK;
}

int rtgs2d_fit_write_rows(rtgs2d_fit* f, const int64_t* rows, int64_t n_rows, const float* xy_raw,
                          const float* diag_raw, const float* off_raw, const float* color_raw,
                          const float* weight_raw, void* stream) {
  RTGS_TRY(check_fit(f));
  if (n_rows < 0) return set_error(RTGS2D_ERR_INVALID, "n_rows must be >= 0");
  if (n_rows == 0 || f->m == 0) return RTGS2D_OK;
  if (!rows) return set_error(RTGS2D_ERR_INVALID, "rows is NULL");
  if (f->unit_weight) weight_raw = nullptr;  // no weight parameter
  const int given = (xy_raw != nullptr) + (diag_raw != nullptr) + (off_raw != nullptr) +
                    (color_raw != nullptr) + (weight_raw != nullptr);
  const int all = f->unit_weight ? 4 : 5;
  if (given != 0 && given != all) {
    return set_error(RTGS2D_ERR_INVALID, "give all raw parameter arrays or none");
  }
  write_rows_kernel<<<grid_for(n_rows), kThreads, 0, as_stream(stream)>>>(
      f->m, rows, n_rows, xy_raw, diag_raw, off_raw, color_raw, weight_raw, f->raw.as<float>(),
      f->m1.as<float>(), f->m2.as<float>());
  return check_cuda(cudaGetLastError(), "write_rows_kernel");
}

int rtgs2d_fit_set_appearance(rtgs2d_fit* f, int32_t parameterization) {
  RTGS_TRY(check_fit(f));
  if (parameterization != RTGS2D_APPEARANCE_WEIGHT_COLOR_9P &&
      parameterization != RTGS2D_APPEARANCE_UNIT_WEIGHT_8P) {
    return set_error(RTGS2D_ERR_INVALID, "unknown appearance parameterization");
  }
  const bool unit = parameterization == RTGS2D_APPEARANCE_UNIT_WEIGHT_8P;
  if (unit != f->unit_weight) f->have_raw = false;  // the raw slots change meaning: set them again
  f->unit_weight = unit;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_binning(rtgs2d_fit* f, int32_t mode) {
  RTGS_TRY(check_fit(f));
  if (mode < RTGS2D_BINNING_AUTO || mode > RTGS2D_BINNING_SORTED) {
    return set_error(RTGS2D_ERR_INVALID, "unknown binning mode");
  }
  f->binning = mode;
  return RTGS2D_OK;
}

int rtgs2d_fit_set_graphs(rtgs2d_fit* f, int32_t enable) {
  RTGS_TRY(check_fit(f));
  f->graphs_enabled = enable != 0;
  if (!f->graphs_enabled) {
    f->release_graphs();
    f->last_eager_key.clear();
  }
  return RTGS2D_OK;
}

int rtgs2d_fit_chunk_counts(const rtgs2d_fit* f, int64_t* graph_chunks, int64_t* eager_chunks) {
  if (!f) return set_error(RTGS2D_ERR_INVALID, "fit is NULL");
  if (graph_chunks) *graph_chunks = f->graph_chunks;
  if (eager_chunks) *eager_chunks = f->eager_chunks;
  return RTGS2D_OK;
}

int rtgs2d_fit_stage_times(const rtgs2d_fit* f, double* bin_ms, double* raster_ms, double* adam_ms,
                           int64_t* iterations_timed, double* pairs_timed) {
  if (!f) return set_error(RTGS2D_ERR_INVALID, "fit is NULL");
  if (bin_ms) *bin_ms = f->bin_ms;
  if (raster_ms) *raster_ms = f->raster_ms;
  if (adam_ms) *adam_ms = f->adam_ms;
  if (iterations_timed) *iterations_timed = f->iterations_timed;
  if (pairs_timed) *pairs_timed = f->pairs_timed;
  return RTGS2D_OK;
}

int rtgs2d_fit_get_raw(rtgs2d_fit* f, float* xy_raw, float* diag_raw, float* off_raw,
                       float* color_raw, float* weight_raw, void* stream) {
  RTGS_TRY(check_fit(f));
  if (f->m == 0) return RTGS2D_OK;
  unpack_raw_kernel<<<grid_for(f->m), kThreads, 0, as_stream(stream)>>>(
      f->m, f->raw.as<float>(), xy_raw, diag_raw, off_raw, color_raw,
      f->unit_weight ? nullptr : weight_raw);
  return check_cuda(cudaGetLastError(), "unpack_raw_kernel");
}

int rtgs2d_fit_get_params(rtgs2d_fit* f, float* xy, float* chol, float* color, float* weight,
                          void* stream) {
  RTGS_TRY(check_fit(f));
  if (f->m > 0 && (!xy || !chol || !color || !weight)) {
    return set_error(RTGS2D_ERR_INVALID, "output pointer is NULL");
  }
  return launch_build_params(f->raw.as<float>(), f->m, f->height, f->width, f->unit_weight, xy,
                             chol, color, weight, as_stream(stream));
}

int rtgs2d_fit_evaluate(rtgs2d_fit* f, float* render, double* sums, void* stream) {
  RTGS_TRY(check_fit(f));
  if (!f->have_targets || !f->have_raw) {
    return set_error(RTGS2D_ERR_INVALID, "set targets and raw parameters before evaluating");
  }
  cudaStream_t s = as_stream(stream);
  RTGS_TRY(project_and_bin(f, s));
  FitRasterArgs fa = raster_args(f);
  fa.render_out = render;
  RTGS_TRY(launch_raster_fit(f->bb, f->geo, kCutoff, fa, false, s));
  RTGS_TRY(launch_loss_reduce(f->tile_loss.as<double>(), f->geo, f->eval_sums.as<double>(), s));
  if (sums) {
    RTGS_CUDA(cudaMemcpyAsync(sums, f->eval_sums.ptr, static_cast<size_t>(f->n_views) * 2 * sizeof(double),
                              cudaMemcpyDeviceToHost, s),
              "eval sums readback");
  }
  RTGS_CUDA(cudaStreamSynchronize(s), "evaluate sync");
  return RTGS2D_OK;
}

int rtgs2d_fit_gradients(rtgs2d_fit* f, float* xy_raw, float* diag_raw, float* off_raw,
                         float* color_raw, float* weight_raw, float* render, double* sums,
                         void* stream) {
  RTGS_TRY(check_fit(f));
  if (!f->have_targets || !f->have_raw) {
    return set_error(RTGS2D_ERR_INVALID, "set targets and raw parameters before taking gradients");
  }
  cudaStream_t s = as_stream(stream);
  RTGS_TRY(project_and_bin(f, s));
  FitRasterArgs fa = raster_args(f);
  fa.render_out = render;
  RTGS_TRY(launch_raster_fit(f->bb, f->geo, kCutoff, fa, true, s));
  RTGS_TRY(launch_loss_reduce(f->tile_loss.as<double>(), f->geo, f->eval_sums.as<double>(), s));
  if (f->m > 0) {
    RTGS_TRY(f->grad_raw.ensure(static_cast<size_t>(kRawSlots) * f->m * sizeof(float), s));
    RTGS_TRY(launch_raw_grad(f->bb, f->m, f->height, f->width, f->raw.as<float>(), f->unit_weight,
                             coverage(f), f->grad_raw.as<float>(), s));
    unpack_raw_kernel<<<grid_for(f->m), kThreads, 0, s>>>(f->m, f->grad_raw.as<float>(), xy_raw, diag_raw,
                                                          off_raw, color_raw,
                                                          f->unit_weight ? nullptr : weight_raw);
    RTGS_CUDA(cudaGetLastError(), "unpack_raw_kernel");
  }
  if (sums) {
    RTGS_CUDA(cudaMemcpyAsync(sums, f->eval_sums.ptr, static_cast<size_t>(f->n_views) * 2 * sizeof(double),
                              cudaMemcpyDeviceToHost, s),
              "gradient sums readback");
  }
  RTGS_CUDA(cudaStreamSynchronize(s), "gradients sync");
  return RTGS2D_OK;
}

int rtgs2d_fit_get_moments(rtgs2d_fit* f, int32_t which, float* xy, float* diag, float* off,
                           float* color, float* weight, void* stream) {
  RTGS_TRY(check_fit(f));
  if (which != 1 && which != 2) return set_error(RTGS2D_ERR_INVALID, "which must be 1 or 2");
  if (f->m == 0) return RTGS2D_OK;
  const DevBuf& src = which == 1 ? f->m1 : f->m2;
  unpack_raw_kernel<<<grid_for(f->m), kThreads, 0, as_stream(stream)>>>(
      f->m, src.as<float>(), xy, diag, off, color, f->unit_weight ? nullptr : weight);
  return check_cuda(cudaGetLastError(), "unpack_raw_kernel");
}

int rtgs2d_fit_history(const rtgs2d_fit* f, int64_t max_rows, int64_t* iters, double* sums,
                       int64_t* n_rows) {
  RTGS_TRY(check_fit(f));
  const int64_t rows = static_cast<int64_t>(f->log_iters.size());
  if (n_rows) *n_rows = rows;
  const int64_t copy = rows < max_rows ? rows : max_rows;
  if (copy <= 0) return RTGS2D_OK;
  if (iters) {
    for (int64_t r = 0; r < copy; ++r) iters[r] = f->log_iters[static_cast<size_t>(r)];
  }
  if (sums) {
    RTGS_CUDA(cudaMemcpy(sums, f->log.ptr, static_cast<size_t>(copy * f->n_views * 2) * sizeof(double),
                         cudaMemcpyDeviceToHost),
              "history readback");
  }
  return RTGS2D_OK;
}

int rtgs2d_fit_stats(const rtgs2d_fit* f, int64_t* step, int64_t* last_entries,
                     int64_t* last_pairs, double* total_pairs) {
  if (!f) return set_error(RTGS2D_ERR_INVALID, "fit is NULL");
  if (last_entries) *last_entries = f->last_entries;
  if (step) *step = f->step;
  if (last_entries) *last_entries = f->last_entries;
  if (last_pairs) *last_pairs = f->last_pairs;
  if (total_pairs) *total_pairs = f->total_pairs;
  return RTGS2D_OK;
}

}  // extern "C"
