// Shared definitions for the sm_100a Stage-1 2D gaussian splatting kernels.
//
// Conventions (identical to the reference renderer, src/rtgs/image2gs/renderer2d.py):
//   - pixel (px, py) has its centre at (px + 0.5, py + 0.5)
//   - q = i00*dx^2 + 2*i01*dx*dy + i11*dy^2 with (i00, i01, i11) = Sigma^-1 entries
//   - a pair contributes only if the pixel lies in the gaussian's support rectangle and q < cutoff
//   - out += exp(-q/2) * weight * color, density += exp(-q/2) * weight (accumulated, no alpha)
//
// Every quantity that decides WHICH pixels a gaussian touches (conic, covariance, rectangle, q)
// is computed with explicitly rounded float ops (__fmul_rn / __fadd_rn / __fdiv_rn / __fsqrt_rn)
// in the reference's operation order, so the support set is bit-identical to the reference's.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rtgs2d {

constexpr int kTile = 16;         // binning tile edge, pixels
constexpr float kCutoff = 12.0f;  // renderer2d.py:25 _CUTOFF
constexpr float kMinDiag = 0.3f;  // fit.py:25 _MIN_DIAG
constexpr int kAccum = 8;         // per (gaussian, tile) gradient moments

// Per-gaussian raster record, 48 bytes, read by the raster kernels through shared memory.
struct __align__(16) GaussRecord {
  float4 geo;  // mx, my, i00, 2*i01
  float4 app;  // i11, weight*r, weight*g, weight*b
  int4 rect;   // x0, y0, x1 - x0, y1 - y0 (inclusive support rectangle, clamped to the image)
};

// Per-gaussian tile span: tiles [tx0, tx0 + ntx) x [ty0, ty0 + count / ntx) of view `key_base / T`.
struct __align__(16) TileSpan {
  int tx0, ty0, ntx, key_base;
};

// ---------------------------------------------------------------------------------------------
// Bit-exact projection math.

// float -> int64 the way the reference's ``Tensor.long()`` behaves on x86 (NaN, +-inf and
// |v| >= 2^63 become INT64_MIN), followed by clamp(lo, hi).
__device__ __forceinline__ int to_index_clamped(float v, int hi) {
  if (!(fabsf(v) < 9.223372036854775808e18f)) return 0;  // INT64_MIN clamped to 0
  long long i = static_cast<long long>(v);
  i = i < 0 ? 0 : i;
  i = i > hi ? hi : i;
  return static_cast<int>(i);
}

// torch clamp_min(x, 0): NaN propagates.
__device__ __forceinline__ float clamp_min0(float x) { return x < 0.0f ? 0.0f : x; }

// Sigma^-1 entries (i00, i01, i11) and the entries (a, b, c) of L^-1 = [[a, 0], [b, c]] they are
// built from (zero when the conic was given directly).
struct Conic {
  float i00, i01, i11;
  float a = 0.f, b = 0.f, c = 0.f;
};

// Analytic Sigma^-1 from (l11, l21, l22), gaussians2d.py:34-44.
__device__ __forceinline__ Conic conic_from_chol(float l11, float l21, float l22) {
  Conic k;
  k.a = __frcp_rn(l11);
  k.b = __fdiv_rn(-l21, __fmul_rn(l11, l22));
  k.c = __frcp_rn(l22);
  k.i00 = __fadd_rn(__fmul_rn(k.a, k.a), __fmul_rn(k.b, k.b));
  k.i01 = __fmul_rn(k.b, k.c);
  k.i11 = __fmul_rn(k.c, k.c);
  return k;
}

struct Rect {
  int x0, x1, y0, y1;
  long long pixels;  // pixels in the rectangle, 0 when outside / empty
};

// Support rectangle, renderer2d.py:156-181, with Sigma = L L^T rounded as gaussians2d.py:28-31.
__device__ __forceinline__ Rect support_rect(float mx, float my, float l11, float l21, float l22,
                                             int height, int width) {
  const float s00 = __fmul_rn(l11, l11);
  const float s11 = __fadd_rn(__fmul_rn(l21, l21), __fmul_rn(l22, l22));
  const float rx = __fsqrt_rn(__fmul_rn(kCutoff, clamp_min0(s00)));
  const float ry = __fsqrt_rn(__fmul_rn(kCutoff, clamp_min0(s11)));
  Rect r;
  const float xm = __fsub_rn(mx, rx), xp = __fadd_rn(mx, rx);
  const float ym = __fsub_rn(my, ry), yp = __fadd_rn(my, ry);
  r.x0 = to_index_clamped(ceilf(__fsub_rn(xm, 0.5f)), width - 1);
  r.x1 = to_index_clamped(floorf(__fsub_rn(xp, 0.5f)), width - 1);
  r.y0 = to_index_clamped(ceilf(__fsub_rn(ym, 0.5f)), height - 1);
  r.y1 = to_index_clamped(floorf(__fsub_rn(yp, 0.5f)), height - 1);
  const bool outside = (xp < 0.5f) || (xm > static_cast<float>(width) - 0.5f) || (yp < 0.5f) ||
                       (ym > static_cast<float>(height) - 0.5f);
  const long long nx = r.x1 - r.x0 + 1 > 0 ? r.x1 - r.x0 + 1 : 0;
  const long long ny = r.y1 - r.y0 + 1 > 0 ? r.y1 - r.y0 + 1 : 0;
  r.pixels = outside ? 0 : nx * ny;
  return r;
}

// q for one pair, bit-identical to renderer2d.py:242-246:
//   ((dx*dx)*i00 + ((2*dx)*dy)*i01) + (dy*dy)*i11
// using i01x2 = 2*i01 (exact): round(round(dx*dy) * 2*i01) == round(round(2*dx*dy) * i01).
__device__ __forceinline__ float pair_q(float dx, float dy, float i00, float i01x2, float i11) {
  const float t0 = __fmul_rn(__fmul_rn(dx, dx), i00);
  const float t1 = __fmul_rn(__fmul_rn(dx, dy), i01x2);
  const float t2 = __fmul_rn(__fmul_rn(dy, dy), i11);
  return __fadd_rn(__fadd_rn(t0, t1), t2);
}

// Gaussian falloff exp(-q / 2) = 2^(q * (-log2(e) / 2)): one multiply and the hardware base-2
// exponential (ex2.approx, relative error ~2^-22, flushes denormal results to zero, which only
// happens for q > 250, far outside the q < 12 support).
__device__ __forceinline__ float falloff(float q) {
  constexpr float kNegHalfLog2e = -0.72134752044448170368f;  // -log2(e) / 2
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(q * kNegHalfLog2e));
  return r;
}

// ---------------------------------------------------------------------------------------------
// Raw-parameter transforms of the native fit, fit.py:402-417.

// The transforms only shape parameters and gradients (never the bit-exact support tests), so they
// use the hardware exponential (__expf, ~2 ulp) and fast division (__fdividef, ~2 ulp; 0 for a
// denominator above 2^126, where the exact quotient is below 2^-126 anyway): they sit on the
// latency-bound Adam kernel's critical path.
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// torch.nn.functional.softplus with beta = 1, threshold = 20.
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

// d softplus / dx (torch softplus_backward: z / (z + 1), z = exp(x); 1 above the threshold).
__device__ __forceinline__ float softplus_grad_f(float x) {
  if (x > 20.0f) return 1.0f;
  const float z = __expf(x);
  return __fdividef(z, z + 1.0f);
}
// Planar raw-parameter slots (each slot is an array of M floats).
enum RawSlot : int {
  kXr = 0, kYr = 1, kD0 = 2, kD1 = 3, kOff = 4, kCr = 5, kCg = 6, kCb = 7, kWr = 8, kRawSlots = 9
};

}  // namespace rtgs2d
