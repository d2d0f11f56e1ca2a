// Per-gaussian gradient finalisation and the fused Adam step.
//
// The raster backward leaves 8 moments per (gaussian, tile) entry (see raster.cu). Entries of one
// gaussian are contiguous (gaussian-major emission), so each gaussian sums its own entries in
// index order -- deterministic, no atomics -- and applies the chain rule:
//
//   dL/dmx = Gx = sum dq (i00 dx + i01 dy)        dL/dmy = Gy = sum dq (i01 dx + i11 dy)
//   (renderer moments; the fused fit kernel's are sum dq dx, sum dq dy, chained by the Adam kernel)
//   dL/di00 = -Sxx/2   dL/di01 = -Sxy   dL/di11 = -Syy/2        (q = i00 dx^2 + 2 i01 dx dy + i11 dy^2)
//   dL/dcolor_k = weight * S_k         dL/dweight = sum_k color_k S_k (+ Sd for density)
//
// which is the reference backward (renderer2d_ext.cu:159-171) regrouped so that per-pair work
// carries no per-gaussian constants. Conic -> Cholesky follows gaussians2d.py:34-44, the raw
// transforms fit.py:402-417, and the update torch.optim.Adam (fit.py:419) with the cosine
// schedule's learning rate supplied by the host.
#include <cmath>

#include "../../include/rtgs2d.h"
#include "internal.h"
#include "kernels.cuh"

namespace rtgs2d {
namespace {

constexpr int kThreads = kProjThreads;

template <bool DEN>
__global__ void __launch_bounds__(kThreads)
finalize_chol_kernel(int64_t m, int64_t cap, const int* __restrict__ counts, const int* __restrict__ offsets,
                     const float4* __restrict__ partials, const float* __restrict__ partial_d,
                     const float* __restrict__ chol, const float* __restrict__ color,
                     const float* __restrict__ weight, float* __restrict__ grad_xy,
                     float* __restrict__ grad_chol, float* __restrict__ grad_color,
                     float* __restrict__ grad_weight) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  cnt = clamp_to_capacity(cnt, off, cap);
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);
  if (!active) return;
  const float l11 = chol[3 * i], l21 = chol[3 * i + 1], l22 = chol[3 * i + 2];
  const Conic k = conic_from_chol(l11, l21, l22);
  const GeoGrad gg = geo_grad(mo, k, true);
  const float w = weight[i];
  const float cr = color[3 * i], cg = color[3 * i + 1], cb = color[3 * i + 2];
  if (grad_xy) {
    grad_xy[2 * i] = gg.gmx;
    grad_xy[2 * i + 1] = gg.gmy;
  }
  if (grad_chol) {
    grad_chol[3 * i] = gg.gl11;
    grad_chol[3 * i + 1] = gg.gl21;
    grad_chol[3 * i + 2] = gg.gl22;
  }
  if (grad_color) {
    grad_color[3 * i] = w * mo.s[5];
    grad_color[3 * i + 1] = w * mo.s[6];
    grad_color[3 * i + 2] = w * mo.s[7];
  }
  if (grad_weight) grad_weight[i] = fmaf(cr, mo.s[5], fmaf(cg, mo.s[6], cb * mo.s[7])) + mo.sd;
}

template <bool DEN>
__global__ void __launch_bounds__(kThreads)
finalize_conic_kernel(int64_t m, int64_t cap, const int* __restrict__ counts, const int* __restrict__ offsets,
                      const float4* __restrict__ partials, const float* __restrict__ partial_d,
                      const float* __restrict__ conics, const float* __restrict__ colors,
                      const float* __restrict__ weights, float* __restrict__ grad_xy,
                      float* __restrict__ grad_conics, float* __restrict__ grad_colors,
                      float* __restrict__ grad_weights) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  cnt = clamp_to_capacity(cnt, off, cap);
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);
  if (!active) return;
  const GeoGrad gg =
      geo_grad(mo, Conic{conics[3 * i], conics[3 * i + 1], conics[3 * i + 2]}, false);
  const float w = weights[i];
  grad_xy[2 * i] = gg.gmx;
  grad_xy[2 * i + 1] = gg.gmy;
  grad_conics[3 * i] = gg.gi00;
  grad_conics[3 * i + 1] = gg.gi01;
  grad_conics[3 * i + 2] = gg.gi11;
  grad_colors[3 * i] = w * mo.s[5];
  grad_colors[3 * i + 1] = w * mo.s[6];
  grad_colors[3 * i + 2] = w * mo.s[7];
  grad_weights[i] = fmaf(colors[3 * i], mo.s[5],
                         fmaf(colors[3 * i + 1], mo.s[6], colors[3 * i + 2] * mo.s[7])) + mo.sd;
}

// Gradient of the fit loss with respect to one gaussian's raw parameters (slots kXr .. kWr) from
// its summed entry moments: the chain rule through Sigma^-1 of the Cholesky factor and the raw
// transforms of fit.py:402-417 (sigmoid for the mean, colour and weight, softplus + _MIN_DIAG for
// the diagonal). With unit_weight the weight is 1 and has no gradient (the unit-weight fit).
template <bool DEN>
__device__ __forceinline__ void raw_gradient(const float (&r)[kRawSlots], const Moments& mo, int height,
                                             int width, bool unit_weight, float (&grad)[kRawSlots]) {
  const float sx = sigmoid_f(r[kXr]), sy = sigmoid_f(r[kYr]);
  const float l11 = __fadd_rn(softplus_f(r[kD0]), kMinDiag);
  const float l22 = __fadd_rn(softplus_f(r[kD1]), kMinDiag);
  const float l21 = r[kOff];
  const Conic k = conic_from_chol(l11, l21, l22);
  GeoGrad gg = geo_grad(mo, k, true);
  // The fused fit raster leaves the plain first moments sum dq dx, sum dq dy: apply Sigma^-1.
  gg.gmx = fmaf(k.i00, mo.s[0], k.i01 * mo.s[1]);
  gg.gmy = fmaf(k.i01, mo.s[0], k.i11 * mo.s[1]);
  const float cr = sigmoid_f(r[kCr]), cg = sigmoid_f(r[kCg]), cb = sigmoid_f(r[kCb]);
  const float w = unit_weight ? 1.0f : sigmoid_f(r[kWr]);
  grad[kXr] = gg.gmx * static_cast<float>(width) * (1.0f - sx) * sx;
  grad[kYr] = gg.gmy * static_cast<float>(height) * (1.0f - sy) * sy;
  grad[kD0] = gg.gl11 * softplus_grad_f(r[kD0]);
  grad[kD1] = gg.gl22 * softplus_grad_f(r[kD1]);
  grad[kOff] = gg.gl21;
  grad[kCr] = w * mo.s[5] * (1.0f - cr) * cr;
  grad[kCg] = w * mo.s[6] * (1.0f - cg) * cg;
  grad[kCb] = w * mo.s[7] * (1.0f - cb) * cb;
  // dL/dweight = sum_k color_k S_k (+ the density moment of the mask coverage penalty)
  grad[kWr] = unit_weight ? 0.f
                          : (fmaf(cr, mo.s[5], fmaf(cg, mo.s[6], cb * mo.s[7])) + (DEN ? mo.sd : 0.f)) *
                                (1.0f - w) * w;
}

// rtgs2d_fit_gradients: the raw-parameter gradient of every gaussian, planar (9, M), without an
// Adam step.
template <bool DEN>
__global__ void __launch_bounds__(kThreads)
raw_grad_kernel(int64_t m, int64_t cap, const int* __restrict__ counts, const int* __restrict__ offsets,
                const float4* __restrict__ partials, const float* __restrict__ partial_d, int height,
                int width, const float* __restrict__ raw, bool unit_weight, float* __restrict__ grad_out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  cnt = clamp_to_capacity(cnt, off, cap);
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);
  if (!active) return;
  float r[kRawSlots], grad[kRawSlots];
#pragma unroll
  for (int k = 0; k < kRawSlots; ++k) r[k] = raw[k * m + i];
  raw_gradient<DEN>(r, mo, height, width, unit_weight, grad);
#pragma unroll
  for (int k = 0; k < kRawSlots; ++k) grad_out[k * m + i] = grad[k];
}

// Adam step of every gaussian from the previous raster's entry moments; with PROJECT the updated
// parameters are projected for the next iteration in the same pass (the projection of
// project_raw_kernel), which saves a launch and a re-read of the raw parameters per iteration.
// `counts` is read (previous binning) before the projection rewrites it, by the same thread.
template <bool PROJECT, bool DEN>
__global__ void __launch_bounds__(kThreads)
adam_fit_kernel(int64_t m, int64_t cap, int* counts, const int* __restrict__ offsets,
                const float4* __restrict__ partials, const float* __restrict__ partial_d,
                int height, int width, float* __restrict__ raw,
                float* __restrict__ m1, float* __restrict__ m2,
                const IterScalars* __restrict__ table, int k_iter, LossLog lg, int64_t n_per_view,
                int tiles_x, int tiles_per_view, ProjOut o) {
  // With direct placement this kernel is a programmatic dependent of the fit raster before it
  // (launch_adam_fit): it may start while the raster still runs. Everything read before the
  // griddepcontrol.wait below (the iteration's constants, the raw parameters and Adam moments, the
  // previous projection's tile counts and entry offsets) was written before that raster started;
  // the entry moments and tile losses are read after it. The next raster may launch right away: it
  // waits for this kernel before it reads anything this kernel writes.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const AdamScalars a = table[k_iter].adam;
  const int log_slot = table[k_iter].log_slot;
  const bool active = i < m;
  float r[kRawSlots], v1[kRawSlots], v2[kRawSlots];
  if (active) {
#pragma unroll
    for (int k = 0; k < kRawSlots; ++k) {
      r[k] = raw[k * m + i];
      v1[k] = m1[k * m + i];
      v2[k] = m2[k * m + i];
    }
  }
  int cnt = active ? counts[i] : 0;
  const int off_any = active ? offsets[i] : 0;  // loaded together with counts[i], not after it
  const int off = cnt > 0 ? off_any : 0;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the raster's entry moments and tile losses
  if (log_slot >= 0) {  // the first blocks also log this iteration's loss, one view per block
    for (int v = blockIdx.x; v < lg.n_views; v += gridDim.x) {
      reduce_view_loss(lg.tile_loss, lg.tiles_per_view, v,
                       lg.log + static_cast<int64_t>(log_slot) * lg.n_views * 2);
    }
  }
  cnt = clamp_to_capacity(cnt, off, cap);
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);

  if (active) {
    float grad[kRawSlots];
    raw_gradient<DEN>(r, mo, height, width, a.unit_weight, grad);
    const int first = a.freeze_geometry ? kCr : 0;
    const int last = a.unit_weight ? kWr : kRawSlots;  // the unit-weight fit has no weight parameter
#pragma unroll
    for (int s = 0; s < kRawSlots; ++s) {
      if (s < first || s >= last) continue;
      adam_update(r[s], v1[s], v2[s], grad[s], a);
      raw[s * m + i] = r[s];
      m1[s * m + i] = v1[s];
      m2[s * m + i] = v2[s];
    }
  }

  if constexpr (PROJECT) {
    float mx = 0.f, my = 0.f, w = 0.f, cr = 0.f, cg = 0.f, cb = 0.f;
    Conic k{0.f, 0.f, 0.f};
    Rect rc{0, -1, 0, -1, 0};
    int view = 0;
    if (active) {
      mx = __fmul_rn(sigmoid_f(r[kXr]), static_cast<float>(width));
      my = __fmul_rn(sigmoid_f(r[kYr]), static_cast<float>(height));
      const float l11 = __fadd_rn(softplus_f(r[kD0]), kMinDiag);
      const float l22 = __fadd_rn(softplus_f(r[kD1]), kMinDiag);
      const float l21 = r[kOff];
      k = conic_from_chol(l11, l21, l22);
      rc = support_rect(mx, my, l11, l21, l22, height, width);
      cr = sigmoid_f(r[kCr]);
      cg = sigmoid_f(r[kCg]);
      cb = sigmoid_f(r[kCb]);
      w = a.unit_weight ? 1.0f : sigmoid_f(r[kWr]);
      view = static_cast<int>(i / n_per_view);
    }
    project_tail(i, active, mx, my, k, rc.x0, rc.x1, rc.y0, rc.y1, rc.pixels, w, cr, cg, cb, view,
                 tiles_x, tiles_per_view, o);
  }
}

unsigned grid_for(int64_t m) { return static_cast<unsigned>((m + kThreads - 1) / kThreads); }

}  // namespace

int launch_finalize_chol(const BinBuffers& bb, int64_t m, const float* chol, const float* color,
                         const float* weight, bool with_density, float* grad_xy, float* grad_chol,
                         float* grad_color, float* grad_weight, cudaStream_t s) {
  if (m == 0) return 0;
  if (with_density) {
    finalize_chol_kernel<true><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(),
        bb.partial_d.as<float>(), chol, color, weight, grad_xy, grad_chol, grad_color, grad_weight);
  } else {
    finalize_chol_kernel<false><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(), nullptr, chol,
        color, weight, grad_xy, grad_chol, grad_color, grad_weight);
  }
  return check_cuda(cudaGetLastError(), "finalize_chol_kernel");
}

int launch_finalize_conic(const BinBuffers& bb, int64_t m, const float* conics,
                          const float* colors, const float* weights, bool with_density,
                          float* grad_xy, float* grad_conics, float* grad_colors,
                          float* grad_weights, cudaStream_t s) {
  if (m == 0) return 0;
  if (with_density) {
    finalize_conic_kernel<true><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(),
        bb.partial_d.as<float>(), conics, colors, weights, grad_xy, grad_conics, grad_colors,
        grad_weights);
  } else {
    finalize_conic_kernel<false><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(), nullptr, conics,
        colors, weights, grad_xy, grad_conics, grad_colors, grad_weights);
  }
  return check_cuda(cudaGetLastError(), "finalize_conic_kernel");
}

int launch_raw_grad(const BinBuffers& bb, int64_t m, int height, int width, const float* raw,
                    bool unit_weight, bool density, float* grad_out, cudaStream_t s) {
  if (m == 0) return 0;
  if (density) {
    raw_grad_kernel<true><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(),
        bb.partial_d.as<float>(), height, width, raw, unit_weight, grad_out);
  } else {
    raw_grad_kernel<false><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.capacity, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(), nullptr,
        height, width, raw, unit_weight, grad_out);
  }
  return check_cuda(cudaGetLastError(), "raw_grad_kernel");
}

int launch_adam_fit(BinBuffers& bb, const Geometry& g, int64_t m, int64_t n_per_view, float* raw,
                    float* m1, float* m2, const IterScalars* table, int k, const LossLog& lg,
                    bool project_next, const uint8_t* active, bool density, int* cursors,
                    bool pdl, cudaStream_t s) {
  if (m == 0) return 0;
  ProjOut o{};
  const float* pd = density ? bb.partial_d.as<float>() : nullptr;
  if (project_next) {
    // Same buffers as a projection launcher; tile counts and stats slots 0-1 restart at zero.
    o.records = bb.records.as<GaussRecord>();
    o.weights = density ? bb.weights.as<float>() : nullptr;
    o.spans = bb.spans.as<TileSpan>();
    o.counts = bb.counts.as<int>();
    o.offsets = bb.offsets.as<int>();
    o.stats = bb.stats.as<unsigned long long>();
    o.entries = bb.entries[0].as<uint64_t>();
    o.cap = bb.capacity;
    o.active = active;
    o.tiles_x = g.tiles_x;
    if (cursors) {
      // Direct placement into the segments of a layout (direct_layout): the tile cursors advance
      // and the ids go to the list. The binning before this kernel (tile sort, or the fit raster
      // that sorts its own tile) left stats slots 0-1 at zero.
      o.tile_count = cursors;
      o.list = bb.list.as<uint32_t>();
      o.list_cap = static_cast<int64_t>(bb.list.bytes / sizeof(uint32_t));
    } else {
      o.tile_count = bb.tile_count.as<int>();
      if (!bb.counts_cleared) {  // the scatter binning leaves both at zero; the radix path does not
        RTGS_TRY(reset_tile_counts(bb, g, s));
        RTGS_CUDA(cudaMemsetAsync(bb.stats.ptr, 0, 2 * sizeof(unsigned long long), s), "memset stats");
      }
    }
    bb.counts_cleared = false;
    bb.entries_emitted = true;
  }
  // With direct placement and `pdl`, a programmatic dependent launch of the fit raster before it:
  // the blocks are scheduled during the raster's last wave and load what does not depend on it
  // (the kernel waits before it reads the raster's output), which hides the launch gap and that
  // round trip.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid_for(m));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cursors && pdl ? 1 : 0;
  const int64_t cap = bb.capacity;
  int* counts = bb.counts.as<int>();
  const int* offsets = bb.offsets.as<int>();
  const float4* partials = bb.partials.as<float4>();
#define RTGS_ADAM(P, D)                                                                              \
  RTGS_CUDA(cudaLaunchKernelEx(&cfg, adam_fit_kernel<P, D>, m, cap, counts, offsets, partials, pd,  \
                               g.height, g.width, raw, m1, m2, table, k, lg, n_per_view, g.tiles_x, \
                               g.tiles_per_view, o),                                                 \
            "adam_fit_kernel")
  if (project_next) {
    if (density) RTGS_ADAM(true, true); else RTGS_ADAM(true, false);
  } else {
    if (density) RTGS_ADAM(false, true); else RTGS_ADAM(false, false);
  }
#undef RTGS_ADAM
  return check_cuda(cudaGetLastError(), "adam_fit_kernel");
}

bool adam_single_wave(int64_t m, bool density) {
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const cudaError_t err = density
      ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adam_fit_kernel<true, true>, kThreads, 0)
      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adam_fit_kernel<true, false>, kThreads, 0);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return static_cast<int64_t>(grid_for(m)) <= static_cast<int64_t>(per_sm) * sms;
}

// ---- rtgs2d_adam_step: torch.optim.Adam's update over several tensors in one launch ----------

namespace {

constexpr int kMaxAdamTensors = RTGS2D_ADAM_MAX_TENSORS;

struct AdamTensors {
  float* param[kMaxAdamTensors];
  const float* grad[kMaxAdamTensors];
  float* exp_avg[kMaxAdamTensors];
  float* exp_avg_sq[kMaxAdamTensors];
  int64_t end[kMaxAdamTensors];  // inclusive prefix of the sizes: tensor k owns [end[k-1], end[k])
  int n;
};

// Grid-stride over the concatenated elements; each element finds its tensor by a scan of the
// (at most 16) prefix ends, then takes adam_update (the same update as the fit loop).
__global__ void __launch_bounds__(256)
adam_step_kernel(const AdamTensors t, int64_t total, AdamScalars a) {
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * 256) {
    int k = 0;
    while (k + 1 < t.n && idx >= t.end[k]) ++k;
    const int64_t j = idx - (k > 0 ? t.end[k - 1] : 0);
    float p = t.param[k][j], m1 = t.exp_avg[k][j], m2 = t.exp_avg_sq[k][j];
    adam_update(p, m1, m2, t.grad[k][j], a);
    t.param[k][j] = p;
    t.exp_avg[k][j] = m1;
    t.exp_avg_sq[k][j] = m2;
  }
}

}  // namespace
}  // namespace rtgs2d

using namespace rtgs2d;

int rtgs2d_adam_step(int32_t n_tensors, float* const* params, const float* const* grads,
                     float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* sizes,
                     double lr, double beta1, double beta2, double eps, int64_t step, void* stream) {
  if (n_tensors < 0 || n_tensors > kMaxAdamTensors) {
    return set_error(RTGS2D_ERR_INVALID, "n_tensors must be in [0, RTGS2D_ADAM_MAX_TENSORS]");
  }
  if (step < 1) return set_error(RTGS2D_ERR_INVALID, "step must be >= 1 (the step this update completes)");
  if (n_tensors == 0) return RTGS2D_OK;
  if (!params || !grads || !exp_avgs || !exp_avg_sqs || !sizes) {
    return set_error(RTGS2D_ERR_INVALID, "tensor array pointer is NULL");
  }
  AdamTensors t{};
  int64_t total = 0;
  for (int k = 0; k < n_tensors; ++k) {
    if (sizes[k] < 0) return set_error(RTGS2D_ERR_INVALID, "tensor size is negative");
    if (sizes[k] > 0 && (!params[k] || !grads[k] || !exp_avgs[k] || !exp_avg_sqs[k])) {
      return set_error(RTGS2D_ERR_INVALID, "tensor pointer is NULL");
    }
    t.param[k] = params[k];
    t.grad[k] = grads[k];
    t.exp_avg[k] = exp_avgs[k];
    t.exp_avg_sq[k] = exp_avg_sqs[k];
    total += sizes[k];
    t.end[k] = total;
  }
  t.n = n_tensors;
  if (total == 0) return RTGS2D_OK;
  // Bias corrections in double, as torch evaluates them on the host (Python floats).
  const double bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(beta2, static_cast<double>(step));
  AdamScalars a{};
  a.neg_step_size = static_cast<float>(-(lr / bc1));
  a.inv_bc2_sqrt = static_cast<float>(1.0 / std::sqrt(bc2));
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.one_minus_beta1 = static_cast<float>(1.0 - beta1);
  a.one_minus_beta2 = static_cast<float>(1.0 - beta2);
  a.eps = static_cast<float>(eps);
  const int64_t blocks64 = (total + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
  adam_step_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(t, total, a);
  return check_cuda(cudaGetLastError(), "adam_step_kernel");
}
