// Per-gaussian gradient finalisation and the fused Adam step.
//
// The raster backward leaves 8 moments per (gaussian, tile) entry (see raster.cu). Entries of one
// gaussian are contiguous (gaussian-major emission), so each gaussian sums its own entries in
// index order -- deterministic, no atomics -- and applies the chain rule:
//
//   dL/dmx = i00*Sdx + i01*Sdy        dL/dmy = i01*Sdx + i11*Sdy
//   dL/di00 = -Sxx/2   dL/di01 = -Sxy   dL/di11 = -Syy/2        (q = i00 dx^2 + 2 i01 dx dy + i11 dy^2)
//   dL/dcolor_k = weight * S_k         dL/dweight = sum_k color_k S_k (+ Sd for density)
//
// which is the reference backward (renderer2d_ext.cu:159-171) regrouped so that per-pair work
// carries no per-gaussian constants. Conic -> Cholesky follows gaussians2d.py:34-44, the raw
// transforms fit.py:402-417, and the update torch.optim.Adam (fit.py:419) with the cosine
// schedule's learning rate supplied by the host.
#include "internal.h"

namespace rtgs2d {
namespace {

constexpr int kThreads = 256;
constexpr int kSmallEntries = 8;  // gaussians with more entries are summed by the whole warp

struct Moments {
  float s[8];
  float sd;
};

// Sum a gaussian's entries [off, off + cnt) in index order. Small counts: the owning thread;
// larger counts: the whole warp, lanes striding and a fixed butterfly -- the choice depends only
// on the count, so results are reproducible run to run.
template <bool DEN>
__device__ __forceinline__ Moments gather_moments(const float4* __restrict__ partials,
                                                  const float* __restrict__ partial_d, int cnt,
                                                  int off) {
  Moments mo;
#pragma unroll
  for (int k = 0; k < 8; ++k) mo.s[k] = 0.f;
  mo.sd = 0.f;
  if (cnt > 0 && cnt <= kSmallEntries) {
    for (int j = 0; j < cnt; ++j) {
      const float4 p0 = partials[2 * static_cast<int64_t>(off + j)];
      const float4 p1 = partials[2 * static_cast<int64_t>(off + j) + 1];
      mo.s[0] += p0.x; mo.s[1] += p0.y; mo.s[2] += p0.z; mo.s[3] += p0.w;
      mo.s[4] += p1.x; mo.s[5] += p1.y; mo.s[6] += p1.z; mo.s[7] += p1.w;
      if constexpr (DEN) mo.sd += partial_d[off + j];
    }
  }
  const int lane = threadIdx.x & 31;
  unsigned big = __ballot_sync(0xffffffffu, cnt > kSmallEntries);
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    const int c = __shfl_sync(0xffffffffu, cnt, src);
    const int o = __shfl_sync(0xffffffffu, off, src);
    float t[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float td = 0.f;
    for (int j = lane; j < c; j += 32) {
      const float4 p0 = partials[2 * static_cast<int64_t>(o + j)];
      const float4 p1 = partials[2 * static_cast<int64_t>(o + j) + 1];
      t[0] += p0.x; t[1] += p0.y; t[2] += p0.z; t[3] += p0.w;
      t[4] += p1.x; t[5] += p1.y; t[6] += p1.z; t[7] += p1.w;
      if constexpr (DEN) td += partial_d[o + j];
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) {
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] += __shfl_xor_sync(0xffffffffu, t[k], sh);
      if constexpr (DEN) td += __shfl_xor_sync(0xffffffffu, td, sh);
    }
    if (lane == src) {
#pragma unroll
      for (int k = 0; k < 8; ++k) mo.s[k] = t[k];
      mo.sd = td;
    }
  }
  return mo;
}

struct GeoGrad {
  float gmx, gmy, gi00, gi01, gi11;  // conic gradient (reference grad_conics convention)
  float gl11, gl21, gl22;            // Cholesky gradient
};

__device__ __forceinline__ GeoGrad geo_grad(const Moments& mo, float i00, float i01, float i11,
                                            float l11, float l21, float l22, bool want_chol) {
  GeoGrad r;
  r.gmx = fmaf(i00, mo.s[0], i01 * mo.s[1]);
  r.gmy = fmaf(i01, mo.s[0], i11 * mo.s[1]);
  r.gi00 = -0.5f * mo.s[2];
  r.gi01 = -mo.s[3];
  r.gi11 = -0.5f * mo.s[4];
  r.gl11 = r.gl21 = r.gl22 = 0.f;
  if (want_chol) {
    const float a = 1.0f / l11;
    const float b = -l21 / (l11 * l22);
    const float c = 1.0f / l22;
    const float ga = 2.0f * a * r.gi00;
    const float gb = fmaf(2.0f * b, r.gi00, c * r.gi01);
    const float gc = fmaf(b, r.gi01, 2.0f * c * r.gi11);
    r.gl11 = -a * fmaf(ga, a, gb * b);
    r.gl21 = -gb * a * c;
    r.gl22 = -c * fmaf(gb, b, gc * c);
  }
  return r;
}

template <bool DEN>
__global__ void __launch_bounds__(kThreads)
finalize_chol_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
                     const float4* __restrict__ partials, const float* __restrict__ partial_d,
                     const float* __restrict__ chol, const float* __restrict__ color,
                     const float* __restrict__ weight, float* __restrict__ grad_xy,
                     float* __restrict__ grad_chol, float* __restrict__ grad_color,
                     float* __restrict__ grad_weight) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  const int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);
  if (!active) return;
  const float l11 = chol[3 * i], l21 = chol[3 * i + 1], l22 = chol[3 * i + 2];
  const Conic k = conic_from_chol(l11, l21, l22);
  const GeoGrad gg = geo_grad(mo, k.i00, k.i01, k.i11, l11, l21, l22, true);
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
finalize_conic_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
                      const float4* __restrict__ partials, const float* __restrict__ partial_d,
                      const float* __restrict__ conics, const float* __restrict__ colors,
                      const float* __restrict__ weights, float* __restrict__ grad_xy,
                      float* __restrict__ grad_conics, float* __restrict__ grad_colors,
                      float* __restrict__ grad_weights) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  const int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  const Moments mo = gather_moments<DEN>(partials, partial_d, cnt, off);
  if (!active) return;
  const GeoGrad gg =
      geo_grad(mo, conics[3 * i], conics[3 * i + 1], conics[3 * i + 2], 1.f, 0.f, 1.f, false);
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

// One Adam update of a single float parameter, in the order of torch's single-tensor Adam
// (exp_avg.lerp_, exp_avg_sq.mul_.addcmul_, denom = sqrt(v)/bc2_sqrt + eps, p.addcdiv_).
__device__ __forceinline__ void adam_update(float& p, float& m1, float& m2, float g,
                                            const AdamScalars& a) {
  m1 = __fadd_rn(m1, __fmul_rn(a.one_minus_beta1, __fsub_rn(g, m1)));
  m2 = __fadd_rn(__fmul_rn(m2, a.beta2), __fmul_rn(__fmul_rn(a.one_minus_beta2, g), g));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(m2), a.bc2_sqrt), a.eps);
  p = __fadd_rn(p, __fmul_rn(a.neg_step_size, __fdiv_rn(m1, denom)));
}

__global__ void __launch_bounds__(kThreads)
adam_fit_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
                const float4* __restrict__ partials, int height, int width, float* __restrict__ raw,
                float* __restrict__ m1, float* __restrict__ m2, const AdamScalars a) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const bool active = i < m;
  const int cnt = active ? counts[i] : 0;
  const int off = cnt > 0 ? offsets[i] : 0;
  const Moments mo = gather_moments<false>(partials, nullptr, cnt, off);
  if (!active) return;

  float r[kRawSlots];
#pragma unroll
  for (int k = 0; k < kRawSlots; ++k) r[k] = raw[k * m + i];
  const float sx = sigmoid_f(r[kXr]), sy = sigmoid_f(r[kYr]);
  const float l11 = __fadd_rn(softplus_f(r[kD0]), kMinDiag);
  const float l22 = __fadd_rn(softplus_f(r[kD1]), kMinDiag);
  const float l21 = r[kOff];
  const Conic k = conic_from_chol(l11, l21, l22);
  const GeoGrad gg = geo_grad(mo, k.i00, k.i01, k.i11, l11, l21, l22, true);
  const float cr = sigmoid_f(r[kCr]), cg = sigmoid_f(r[kCg]), cb = sigmoid_f(r[kCb]);
  const float w = sigmoid_f(r[kWr]);

  float grad[kRawSlots];
  grad[kXr] = gg.gmx * static_cast<float>(width) * (1.0f - sx) * sx;
  grad[kYr] = gg.gmy * static_cast<float>(height) * (1.0f - sy) * sy;
  grad[kD0] = gg.gl11 * softplus_grad_f(r[kD0]);
  grad[kD1] = gg.gl22 * softplus_grad_f(r[kD1]);
  grad[kOff] = gg.gl21;
  grad[kCr] = w * mo.s[5] * (1.0f - cr) * cr;
  grad[kCg] = w * mo.s[6] * (1.0f - cg) * cg;
  grad[kCb] = w * mo.s[7] * (1.0f - cb) * cb;
  grad[kWr] = fmaf(cr, mo.s[5], fmaf(cg, mo.s[6], cb * mo.s[7])) * (1.0f - w) * w;

  const int first = a.freeze_geometry ? kCr : 0;
#pragma unroll
  for (int s = 0; s < kRawSlots; ++s) {
    if (s < first) continue;
    float p = r[s], v1 = m1[s * m + i], v2 = m2[s * m + i];
    adam_update(p, v1, v2, grad[s], a);
    raw[s * m + i] = p;
    m1[s * m + i] = v1;
    m2[s * m + i] = v2;
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
        m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(),
        bb.partial_d.as<float>(), chol, color, weight, grad_xy, grad_chol, grad_color, grad_weight);
  } else {
    finalize_chol_kernel<false><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(), nullptr, chol,
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
        m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(),
        bb.partial_d.as<float>(), conics, colors, weights, grad_xy, grad_conics, grad_colors,
        grad_weights);
  } else {
    finalize_conic_kernel<false><<<grid_for(m), kThreads, 0, s>>>(
        m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.partials.as<float4>(), nullptr, conics,
        colors, weights, grad_xy, grad_conics, grad_colors, grad_weights);
  }
  return check_cuda(cudaGetLastError(), "finalize_conic_kernel");
}

int launch_adam_fit(const BinBuffers& bb, int64_t m, int height, int width, float* raw, float* m1,
                    float* m2, const AdamScalars& a, cudaStream_t s) {
  if (m == 0) return 0;
  adam_fit_kernel<<<grid_for(m), kThreads, 0, s>>>(m, bb.counts.as<int>(), bb.offsets.as<int>(),
                                                   bb.partials.as<float4>(), height, width, raw,
                                                   m1, m2, a);
  return check_cuda(cudaGetLastError(), "adam_fit_kernel");
}

}  // namespace rtgs2d
