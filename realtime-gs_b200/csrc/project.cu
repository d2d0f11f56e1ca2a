// Projection + culling: per-gaussian raster record, support rectangle and tile span.
//
// One thread per gaussian. Three input forms share one tail:
//   - constrained (xy, chol, color, weight): the B200-native render path (replaces the torch ops
//     of cuda_backend.py:151-158 that built conics and rectangles on the host side);
//   - reference ABI (xy, conics, colors, weights, rects, view_index): renderer2d_ext.cpp:87-128;
//   - raw fit parameters (planar 9 x M): the fit loop's build() (fit.py:402-417) fused in.
#include "internal.h"
#include "kernels.cuh"

namespace rtgs2d {
namespace {

constexpr int kThreads = kProjThreads;

__global__ void __launch_bounds__(kThreads)
project_chol_kernel(const float* __restrict__ xy, const float* __restrict__ chol,
                    const float* __restrict__ color, const float* __restrict__ weight, int64_t m,
                    int64_t n_per_view, int height, int width, int tiles_x, int tiles_per_view,
                    ProjOut o) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  float mx = 0.f, my = 0.f, w = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
  Conic k{0.f, 0.f, 0.f};
  Rect r{0, -1, 0, -1, 0};
  int view = 0;
  if (active) {
    mx = xy[2 * i];
    my = xy[2 * i + 1];
    const float l11 = chol[3 * i], l21 = chol[3 * i + 1], l22 = chol[3 * i + 2];
    k = conic_from_chol(l11, l21, l22);
    r = support_rect(mx, my, l11, l21, l22, height, width);
    w = weight[i];
    cr = color[3 * i];
    cg = color[3 * i + 1];
    cb = color[3 * i + 2];
    view = static_cast<int>(i / n_per_view);
  }
  project_tail(i, active, mx, my, k, r.x0, r.x1, r.y0, r.y1, r.pixels, w, cr, cg, cb, view,
               tiles_x, tiles_per_view, o);
}

__global__ void __launch_bounds__(kThreads)
project_conic_kernel(const float* __restrict__ xy, const float* __restrict__ conics,
                     const float* __restrict__ colors, const float* __restrict__ weights,
                     const int32_t* __restrict__ rects, const int32_t* __restrict__ view_index,
                     int64_t m, int n_views, int height, int width, int tiles_x,
                     int tiles_per_view, ProjOut o) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  bool active = i < m;
  float mx = 0.f, my = 0.f, w = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
  Conic k{0.f, 0.f, 0.f};
  int x0 = 0, x1 = -1, y0 = 0, y1 = -1, view = 0;
  long long pixels = 0;
  if (active) {
    mx = xy[2 * i];
    my = xy[2 * i + 1];
    k.i00 = conics[3 * i];
    k.i01 = conics[3 * i + 1];
    k.i11 = conics[3 * i + 2];
    // The reference kernel trusts the host-made rectangles; clamping keeps a malformed
    // rectangle from addressing outside the image and changes nothing for valid ones.
    x0 = max(rects[4 * i], 0);
    x1 = min(rects[4 * i + 1], width - 1);
    y0 = max(rects[4 * i + 2], 0);
    y1 = min(rects[4 * i + 3], height - 1);
    view = view_index[i];
    if (x1 >= x0 && y1 >= y0 && view >= 0 && view < n_views) {
      pixels = static_cast<long long>(x1 - x0 + 1) * (y1 - y0 + 1);
    }
    w = weights[i];
    cr = colors[3 * i];
    cg = colors[3 * i + 1];
    cb = colors[3 * i + 2];
  }
  project_tail(i, active, mx, my, k, x0, x1, y0, y1, pixels, w, cr, cg, cb, view, tiles_x,
               tiles_per_view, o);
}

__global__ void __launch_bounds__(kThreads)
project_raw_kernel(const float* __restrict__ raw, int64_t m, int64_t n_per_view, int height,
                   int width, int tiles_x, int tiles_per_view, bool unit_weight, ProjOut o) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  float mx = 0.f, my = 0.f, w = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
  Conic k{0.f, 0.f, 0.f};
  Rect r{0, -1, 0, -1, 0};
  int view = 0;
  if (active) {
    mx = __fmul_rn(sigmoid_f(raw[kXr * m + i]), static_cast<float>(width));
    my = __fmul_rn(sigmoid_f(raw[kYr * m + i]), static_cast<float>(height));
    const float l11 = __fadd_rn(softplus_f(raw[kD0 * m + i]), kMinDiag);
    const float l22 = __fadd_rn(softplus_f(raw[kD1 * m + i]), kMinDiag);
    const float l21 = raw[kOff * m + i];
    k = conic_from_chol(l11, l21, l22);
    r = support_rect(mx, my, l11, l21, l22, height, width);
    cr = sigmoid_f(raw[kCr * m + i]);
    cg = sigmoid_f(raw[kCg * m + i]);
    cb = sigmoid_f(raw[kCb * m + i]);
    w = unit_weight ? 1.0f : sigmoid_f(raw[kWr * m + i]);
    view = static_cast<int>(i / n_per_view);
  }
  project_tail(i, active, mx, my, k, r.x0, r.x1, r.y0, r.y1, r.pixels, w, cr, cg, cb, view,
               tiles_x, tiles_per_view, o);
}

__global__ void __launch_bounds__(kThreads)
build_params_kernel(const float* __restrict__ raw, int64_t m, int height, int width,
                    bool unit_weight, float* __restrict__ xy, float* __restrict__ chol, float* __restrict__ color,
                    float* __restrict__ weight) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= m) return;
  xy[2 * i] = __fmul_rn(sigmoid_f(raw[kXr * m + i]), static_cast<float>(width));
  xy[2 * i + 1] = __fmul_rn(sigmoid_f(raw[kYr * m + i]), static_cast<float>(height));
  chol[3 * i] = __fadd_rn(softplus_f(raw[kD0 * m + i]), kMinDiag);
  chol[3 * i + 1] = raw[kOff * m + i];
  chol[3 * i + 2] = __fadd_rn(softplus_f(raw[kD1 * m + i]), kMinDiag);
  color[3 * i] = sigmoid_f(raw[kCr * m + i]);
  color[3 * i + 1] = sigmoid_f(raw[kCg * m + i]);
  color[3 * i + 2] = sigmoid_f(raw[kCb * m + i]);
  weight[i] = unit_weight ? 1.0f : sigmoid_f(raw[kWr * m + i]);
}

__global__ void __launch_bounds__(kThreads)
support_rects_kernel(const float* __restrict__ xy, const float* __restrict__ chol, int64_t m,
                     int height, int width, int32_t* __restrict__ rects,
                     int64_t* __restrict__ counts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= m) return;
  const Rect r = support_rect(xy[2 * i], xy[2 * i + 1], chol[3 * i], chol[3 * i + 1],
                              chol[3 * i + 2], height, width);
  if (rects) {
    rects[4 * i] = r.x0;
    rects[4 * i + 1] = r.pixels > 0 ? r.x1 : r.x0 - 1;
    rects[4 * i + 2] = r.y0;
    rects[4 * i + 3] = r.y1;
  }
  if (counts) counts[i] = r.pixels;
}

int prepare(BinBuffers& bb, const Geometry& g, int64_t m, bool want_weights, cudaStream_t s,
            ProjOut* o) {
  const size_t mm = static_cast<size_t>(m > 0 ? m : 1);
  RTGS_TRY(bb.records.ensure(mm * sizeof(GaussRecord), s));
  RTGS_TRY(bb.spans.ensure(mm * sizeof(TileSpan), s));
  RTGS_TRY(bb.counts.ensure(mm * sizeof(int), s));
  RTGS_TRY(bb.offsets.ensure(mm * sizeof(int), s));
  RTGS_TRY(bb.stats.ensure(kStatSlots * sizeof(unsigned long long), s));
  if (want_weights) RTGS_TRY(bb.weights.ensure(mm * sizeof(float), s));
  RTGS_CUDA(cudaMemsetAsync(bb.stats.ptr, 0, kStatSlots * sizeof(unsigned long long), s), "memset stats");
  o->records = bb.records.as<GaussRecord>();
  o->weights = want_weights ? bb.weights.as<float>() : nullptr;
  o->spans = bb.spans.as<TileSpan>();
  o->counts = bb.counts.as<int>();
  o->offsets = bb.offsets.as<int>();
  o->stats = bb.stats.as<unsigned long long>();
  RTGS_TRY(reset_tile_counts(bb, g, s));
  bb.counts_cleared = false;  // the projection is about to count
  o->tile_count = bb.tile_count.as<int>();
  o->entries = nullptr;  // count only; a launcher that emits sets entries and cap
  o->cap = 0;
  o->active = nullptr;
  o->list = nullptr;  // direct placement is set up by the fit loop's Adam launcher only
  o->list_cap = 0;
  bb.entries_emitted = false;
  o->tiles_x = g.tiles_x;
  return 0;
}

unsigned grid_for(int64_t m) { return static_cast<unsigned>((m + kThreads - 1) / kThreads); }

}  // namespace

int launch_project_chol(BinBuffers& bb, const Geometry& g, const float* xy, const float* chol,
                        const float* color, const float* weight, int64_t m, int64_t n_per_view,
                        bool want_weights, cudaStream_t s) {
  ProjOut o;
  RTGS_TRY(prepare(bb, g, m, want_weights, s, &o));
  if (m == 0) return 0;
  project_chol_kernel<<<grid_for(m), kThreads, 0, s>>>(xy, chol, color, weight, m, n_per_view,
                                                       g.height, g.width, g.tiles_x,
                                                       g.tiles_per_view, o);
  return check_cuda(cudaGetLastError(), "project_chol_kernel");
}

int launch_project_conic(BinBuffers& bb, const Geometry& g, const float* xy, const float* conics,
                         const float* colors, const float* weights, const int32_t* rects,
                         const int32_t* view_index, int64_t m, bool want_weights, cudaStream_t s) {
  ProjOut o;
  RTGS_TRY(prepare(bb, g, m, want_weights, s, &o));
  if (m == 0) return 0;
  project_conic_kernel<<<grid_for(m), kThreads, 0, s>>>(xy, conics, colors, weights, rects,
                                                        view_index, m, g.n_views, g.height,
                                                        g.width, g.tiles_x, g.tiles_per_view, o);
  return check_cuda(cudaGetLastError(), "project_conic_kernel");
}

int launch_project_raw(BinBuffers& bb, const Geometry& g, const float* raw, int64_t m,
                       int64_t n_per_view, bool emit, const uint8_t* active, bool want_weights,
                       bool unit_weight, cudaStream_t s) {
  ProjOut o;
  RTGS_TRY(prepare(bb, g, m, want_weights, s, &o));
  o.active = active;
  if (emit && bb.entries[0].ptr) {
    o.entries = bb.entries[0].as<uint64_t>();
    o.cap = bb.capacity;
    bb.entries_emitted = true;
  }
  if (m == 0) return 0;
  project_raw_kernel<<<grid_for(m), kThreads, 0, s>>>(raw, m, n_per_view, g.height, g.width,
                                                      g.tiles_x, g.tiles_per_view, unit_weight, o);
  return check_cuda(cudaGetLastError(), "project_raw_kernel");
}

int launch_support_rects(const float* xy, const float* chol, int64_t m, int height, int width,
                         int32_t* rects, int64_t* counts, cudaStream_t s) {
  if (m == 0) return 0;
  support_rects_kernel<<<grid_for(m), kThreads, 0, s>>>(xy, chol, m, height, width, rects, counts);
  return check_cuda(cudaGetLastError(), "support_rects_kernel");
}

int launch_build_params(const float* raw, int64_t m, int height, int width, bool unit_weight,
                        float* xy, float* chol, float* color, float* weight, cudaStream_t s) {
  if (m == 0) return 0;
  build_params_kernel<<<grid_for(m), kThreads, 0, s>>>(raw, m, height, width, unit_weight, xy, chol,
                                                       color, weight);
  return check_cuda(cudaGetLastError(), "build_params_kernel");
}

}  // namespace rtgs2d
