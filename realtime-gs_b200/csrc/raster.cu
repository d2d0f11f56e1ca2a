// Per-tile raster kernels for the accumulated 2D splatting renderer (sm_100a).
//
// One CTA per 16x16 tile, 16 / (4*PPT) * 2 warps (PPT pixels per lane: 4 in the renderer forward,
// 2 elsewhere, see kPPT). Each warp owns an 8 x (4*PPT) pixel sub-block and each lane PPT adjacent
// pixels of one column (rows PPT*r .. PPT*r + PPT-1, so that a small gaussian usually covers all
// of them). The tile's gaussian list (ascending gaussian index, from the binning step) is staged
// through shared memory in batches of one record per thread. In the fit loop's direct-placement
// iterations the fit raster sorts its own tile's list first (fused_tile_sort: warp 0, in
// registers, into shared memory), which replaces a separate tile-sort launch per iteration.
//
//   forward   per 32 staged records, 8 + 4*PPT ballots give every lane a 32-bit mask of the
//             records whose support rectangle covers each of its pixels (in the renderer forward
//             narrowed to the records whose ellipse can reach them: reach masks); the lane walks
//             exactly those, in list order, accumulating in registers (flat predicate for the
//             ellipse test q < cutoff, exp(-q/2) as one multiply + ex2). The list order is the
//             reference's summation order, so a render is deterministic and no atomics are used.
//   backward  the tile's upstream gradients are staged in shared memory; every (gaussian, tile)
//             entry's piece = support rectangle x tile is evaluated over exactly its pixels and
//             8 moments
//               Gx = sum dq*(i00 dx + i01 dy), Gy = sum dq*(i01 dx + i11 dy), Sxx = sum dq*dx^2,
//               Sxy = sum dq*dx*dy, Syy = sum dq*dy^2, Sr/Sg/Sb = sum e*g_rgb
//               (e = exp(-q/2), dq = e * g.A; Gx, Gy are the mean gradient's sums)
//             are written once per entry. Pieces are ordered by (orientation, step count) with a
//             stable counting sort; in the fused fit kernel a warp takes 4 pieces at a time, 8
//             lanes ("octet") per piece, each lane owning up to two columns (wide pieces, stepping
//             down the rows) or two rows (tall pieces, stepping across the columns), and an 8-lane
//             transpose butterfly leaves moment r in lane r of each octet: one 32-byte store per
//             entry. The renderer backward takes 8 pieces at a time, 4 lanes ("quad") per piece,
//             each lane owning up to four lines (backward_quad; the quad's transpose leaves moments
//             2q, 2q + 1 in lane q), and a lane steps only through the conservative span where its
//             lines can meet the support ellipse (line_span; the exact support test still runs on
//             every pixel); the step count that orders the pieces is the longest lane's. A per-gaussian pass
//             (optim.cu) sums a gaussian's entries in order and applies the chain rule:
//             deterministic, no global atomics.
//   fit       forward -> L2 loss gradient in registers -> backward, in one kernel: the rendered
//             image and dL/dout never leave the SM.
//
// Reference semantics: renderer2d_ext.cu:69-84 (forward), :142-171 (backward); parity of the
// support set with renderer2d.py:233-248.
#include "internal.h"
#include "kernels.cuh"

namespace rtgs2d {
namespace {

constexpr int kBuckets = 2 * kTile;  // backward work-list buckets: (orientation, steps)
// Row stride (in float4) of the tile's upstream gradients in shared memory: one float4 of padding
// per row puts the 8 rows that a column-wise octet reads at one step in 8 different bank groups
// (with a stride of 16 float4 = 64 words they all fall in the same 4 banks: an 8-way conflict).
constexpr int kGStride = kTile + 1;

template <int PPT>
struct Layout {
  static constexpr int kSubW = 8;
  static constexpr int kSubH = 4 * PPT;
  static constexpr int kSubX = kTile / kSubW;
  static constexpr int kSubY = kTile / kSubH;
  static constexpr int kWarps = kSubX * kSubY;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kBatch = kThreads;  // records staged per batch: one per thread
};

enum Mode : int { kFwd = 0, kBwd = 1, kFit = 2, kEval = 3 };

struct RasterArgs {
  const GaussRecord* records;
  const float* weights;       // density variants
  const TileSpan* spans;      // backward: entry index
  const int* offsets;         // backward: entry index
  const uint64_t* entries;    // radix path: sorted (tile key << 32 | gaussian id)
  const int2* ranges;         // per-tile [start, end) into list (or entries on the radix path)
  const uint32_t* list;       // list paths: gaussian ids grouped by tile, ascending in a tile
  int64_t cap;                // entry capacity (positions and entry indices at or past it are unused)
  int presorted;              // 1: radix path, 0: scatter path
  int height, width, tiles_x, tiles_per_view;
  float cutoff;
  // forward outputs
  float* out;  // (B,H,W,3)
  float* den;  // (B,H,W) or null
  // backward inputs / outputs
  const float* grad_out;  // (B,H,W,3) or null (zero)
  const float* grad_den;  // (B,H,W) or null (zero)
  float4* partials;       // (E, 2) float4
  float* partial_d;       // (E,) density moment
  // fit
  FitRasterArgs fit;
};

// Transpose butterfly inside each 8-lane octet: returns, in lane r of the octet, the octet-wide sum
// of v[r].
__device__ __forceinline__ float octet_transpose_reduce8(const float (&v)[8], int lane) {
  const bool u4 = lane & 4, u2 = lane & 2, u1 = lane & 1;
  float a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = u4 ? v[k] : v[k + 4];
    const float keep = u4 ? v[k + 4] : v[k];
    a[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  float b[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = u2 ? a[k] : a[k + 2];
    const float keep = u2 ? a[k + 2] : a[k];
    b[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  const float send = u1 ? b[0] : b[1];
  const float keep = u1 ? b[1] : b[0];
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// 32 x 32 bit-matrix transpose across the warp: lane i returns the word whose bit j is bit i of
// lane j's x (off-diagonal blocks swapped at every scale, 5 shuffle rounds).
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, int lane) {
  constexpr uint32_t kLow[5] = {0x0000ffffu, 0x00ff00ffu, 0x0f0f0f0fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int r = 0; r < 5; ++r) {
    const int s = 16 >> r;
    const uint32_t m = kLow[r];
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x, s);
    x = (lane & s) ? ((x & ~m) | ((y >> s) & m)) : ((x & m) | ((y << s) & ~m));
  }
  return x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ bool mask_bit(const uint8_t* bits, int64_t idx) {
  return (bits[idx >> 3] >> (idx & 7)) & 1;
}

// Backward piece = a gaussian's support rectangle clipped to the tile, packed as
// rx0 | ry0 << 4 | (pw - 1) << 8 | (ph - 1) << 12. Its bucket orders the backward's work list:
// row-wise pieces (pw >= ph) first, then column-wise ones, each by descending step count (the
// other side), so the 4 pieces of a warp task share an orientation and a step count.
__device__ __forceinline__ int piece_bucket(int pc) {
  const int pw = ((pc >> 8) & 15) + 1, ph = ((pc >> 12) & 15) + 1;
  return pw >= ph ? kTile - ph : 2 * kTile - pw;
}

// The same order with the step count of the longest lane's line spans (piece_quads).
__device__ __forceinline__ int piece_bucket_spans(int pc, int steps) {
  const int pw = ((pc >> 8) & 15) + 1, ph = ((pc >> 12) & 15) + 1;
  return (pw >= ph ? kTile : 2 * kTile) - max(steps, 1);
}

// Pieces whose step axis is shorter than this walk whole lines: their spans would save less than
// they cost. Measured on B200: the renderer backward of the 4K frame with 1M gaussians (median
// sigma 3 px) takes 7.6% less time with spans from 5 steps; the fused fit kernel, whose gaussians
// are small and nearly axis-aligned, is slower with spans at any threshold and walks whole lines.
constexpr int kSpanMinSteps = 5;

__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Coefficients of the support ellipse along one pixel line of a backward piece. With the
// fixed-axis offset d of the line and the varying-axis offset v, q(v) = A v^2 + (2 i01 d) v + F d^2
// (A = coefficient of the varying axis, F = of the fixed one) is a parabola in v with vertex
// vc = kappa d and q(v) - cutoff = A ((v - vc)^2 - h^2), h^2 = k0 - k1 d^2 (k0 = cutoff / A,
// k1 = det / A^2). Only positive definite conics get spans (others keep the whole line).
struct LineCoef {
  float kappa, k0, k1, base;  // base: mean minus the centre of step 0, along the varying axis
  float slack;                // absolute widening of every span (coordinate rounding)
  bool pd;
};

__device__ __forceinline__ LineCoef line_coef(float coef_fix, float coef_var, float i01x2, float mean_var,
                                              float v0, float cutoff) {
  LineCoef c;
  c.pd = coef_var > 0.f && coef_fix > 0.f && i01x2 * i01x2 < 4.f * coef_var * coef_fix;
  const float inv_a = 1.f / coef_var;
  c.kappa = -0.5f * i01x2 * inv_a;
  c.k0 = cutoff * inv_a;
  c.k1 = (coef_fix - 0.25f * i01x2 * i01x2 * inv_a) * inv_a;
  c.base = mean_var - v0;
  c.slack = 2e-6f * (fabsf(mean_var) + fabsf(v0)) + 1e-3f;
  return c;
}

// Steps [lo, hi] of a line (inside [0, steps)) that can hold pixels with q < cutoff; lo > hi when
// none. The span is conservative: the reference-rounded q (pair_q) differs from the exact
// quadratic by at most ~5 ulp of (|t0| + |t1| + |t2|) <= 2 (F d^2 + A v^2), and the widening
// m2 = 4e-6 (h^2 + k0 + 3 vc^2) of h^2 plus the relative and absolute slack of the half width
// exceed that bound (and the rounding of d, v, vc, h^2 and the coordinates) at least twofold, so
// every pixel outside the span has a rounded q >= cutoff. The exact support test still runs on
// every pixel inside it, which keeps the support set identical to the reference's.
__device__ __forceinline__ void line_span(const LineCoef& c, float d, float dsq, int steps, int& lo,
                                          int& hi) {
  if (!c.pd || hi < lo) return;  // not positive definite (whole line), or no pixel on this lane
  const float vc = c.kappa * d;
  const float h2 = fmaf(-c.k1, dsq, c.k0);
  const float r2 = h2 + 4e-6f * (fmaxf(h2, 0.f) + c.k0 + 3.f * vc * vc);
  if (r2 < 0.f) {
    lo = 0;
    hi = -1;
    return;
  }
  const float half = fmaf(sqrt_approx(r2), 1.00001f, fmaf(6e-6f, fabsf(vc), c.slack));
  const float ctr = c.base + vc;
  // NaN bounds (non-finite inputs) fall back to the whole line through fmaxf / fminf.
  lo = static_cast<int>(fminf(fmaxf(ceilf(ctr - half), 0.f), static_cast<float>(steps)));
  hi = static_cast<int>(fmaxf(fminf(floorf(ctr + half), static_cast<float>(steps - 1)), -1.f));
}

// One octet lane's part of a backward piece: up to two pixels per step along the lane axis
// (a = r8 and r8 + 8) and, along the other axis (rows when ROW, columns otherwise), the lane's
// steps start .. start + max(a_first + a_len, b_first + b_len) - 1 (pixel A on for a_len steps
// from start + a_first, B for b_len from start + b_first); the warp runs max_steps steps (the
// longest lane's count), and any_b is set when some lane of the warp has a pixel B.
// The fixed coordinate's terms are computed once; q keeps the reference's rounding order
// ((dx^2 i00 + dx dy 2 i01) + dy^2 i11), and pixel centres are exact (integers + 0.5).
// Moments: S0 = sum dq dx, S1 = sum dq dy (the Adam kernel applies Sigma^-1),
// S2 = sum dq dx^2, S3 = sum dq dx dy, S4 = sum dq dy^2,
// S5..S7 = sum e g_rgb, Sd = sum e g_den, with e = exp(-q/2) and dq = e (g . w c).
// A lane's pixel keeps its fixed-axis offset f for the whole piece, so the dq moments factor:
// per pixel only P0 = sum dq, P1 = sum dq v and P2 = sum dq v^2 (v = varying-axis offset) are
// accumulated, and f, f^2 are applied once at the end (S for dx-dy = f P1, for f^2 = f^2 P0, ...).
// This octet form serves the fused fit kernel, whose gaussians are small and nearly
// axis-aligned: its lanes walk whole lines and P1 sums dq v itself (the renderer backward's quad
// tasks centre each line on its ellipse centre, see backward_quad).
template <bool ROW, bool DEN>
__device__ __forceinline__ void backward_piece(const float4& geo, const float4& app, float wt,
                                               float pxc0, float pyc0, int sidx0, int r8,
                                               int start, unsigned a_first, unsigned a_len,
                                               unsigned b_first, unsigned b_len, bool any_b,
                                               int max_steps, float cutoff, const float4* s_g,
                                               float (&S)[8], float& Sd) {
  // Lane-axis (fixed) coordinate of pixels A and B, and its squared term.
  const float fix_a = (ROW ? pxc0 : pyc0) + static_cast<float>(r8);
  const float fix_b = fix_a + 8.f;
  const float da = __fsub_rn(fix_a, ROW ? geo.x : geo.y);
  const float db = __fsub_rn(fix_b, ROW ? geo.x : geo.y);
  const float sq_a = __fmul_rn(da, da), sq_b = __fmul_rn(db, db);
  const float coef_fix = ROW ? geo.z : app.x;  // i00 for x, i11 for y
  const float coef_var = ROW ? app.x : geo.z;
  const float t_a = __fmul_rn(sq_a, coef_fix), t_b = __fmul_rn(sq_b, coef_fix);
  constexpr int kStep = ROW ? kGStride : 1;        // shared-memory stride of one step
  constexpr int kLaneStride = ROW ? 1 : kGStride;  // and of one lane-axis pixel
  // The lane's steps [0, count) are the union of pixel A's span (from a_first, a_len steps) and
  // B's; a step inside the union but outside one pixel's own span is still inside the piece, where
  // that pixel's rounded q >= cutoff (line_span), so only the union bound is tested per step.
  const int count = static_cast<int>(max(a_first + a_len, b_first + b_len));
  const bool has_a = a_len > 0, has_b = b_len > 0;
  int sidx_a = sidx0 + r8 * kLaneStride + start * kStep;
  float fvar = (ROW ? pyc0 : pxc0) + static_cast<float>(start);  // integer + 0.5: exact
  float pa[3] = {0.f, 0.f, 0.f}, pb[3] = {0.f, 0.f, 0.f};
  // Only the shared-memory load, the falloff and the weighted upstream gradient sit under the
  // support predicate (short enough to be predicated rather than branched); the moment updates
  // run unconditionally with dq = e = 0 and g = 0 outside the support, which adds exact zeros
  // (the offsets and their products are finite), so a non-finite colour or gradient still only
  // reaches pixels inside the support.
  auto accumulate = [&](bool in, int sidx, float d_var, float sq_var, float q, float (&p)[3]) {
    float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
    float e = 0.f, dq = 0.f;
    if (in) {
      gv = s_g[sidx];
      e = falloff(q);
      float v = gv.x * app.y;
      v = fmaf(gv.y, app.z, v);
      v = fmaf(gv.z, app.w, v);
      if constexpr (DEN) v = fmaf(gv.w, wt, v);
      dq = e * v;
    }
    p[0] += dq;
    p[1] = fmaf(dq, d_var, p[1]);
    p[2] = fmaf(dq, sq_var, p[2]);
    S[5] = fmaf(e, gv.x, S[5]);
    S[6] = fmaf(e, gv.y, S[6]);
    S[7] = fmaf(e, gv.z, S[7]);
    if constexpr (DEN) Sd = fmaf(e, gv.w, Sd);
  };
  for (int st = 0; st < max_steps; ++st) {
    const float dv = __fsub_rn(fvar, ROW ? geo.y : geo.x);
    const float sq_v = __fmul_rn(dv, dv);
    const float t_v = __fmul_rn(sq_v, coef_var);
    const bool on = st < count;
    {
      const float t1 = __fmul_rn(__fmul_rn(da, dv), geo.w);  // dx dy (multiplication commutes)
      const float q = ROW ? __fadd_rn(__fadd_rn(t_a, t1), t_v) : __fadd_rn(__fadd_rn(t_v, t1), t_a);
      accumulate(on && has_a && q < cutoff, sidx_a, dv, sq_v, q, pa);
    }
    if (any_b) {
      const float t1 = __fmul_rn(__fmul_rn(db, dv), geo.w);
      const float q = ROW ? __fadd_rn(__fadd_rn(t_b, t1), t_v) : __fadd_rn(__fadd_rn(t_v, t1), t_b);
      accumulate(on && has_b && q < cutoff, sidx_a + 8 * kLaneStride, dv, sq_v, q, pb);
    }
    fvar += 1.f;
    sidx_a += kStep;
  }
  // Plain first moments S0 = sum dq dx, S1 = sum dq dy (the Adam kernel applies Sigma^-1; measured
  // 1.7 us per launch faster than applying it here at the 48-register cap).
  const float p1 = pa[1] + pb[1];
  const float m_f = fmaf(da, pa[0], db * pb[0]);
  S[0] = ROW ? m_f : p1;
  S[1] = ROW ? p1 : m_f;
  // Second moments: f^2 P0, f sum dq v and P2, over A and B.
  const float m_ff = fmaf(sq_a, pa[0], sq_b * pb[0]);
  const float m_fv = fmaf(da, pa[1], db * pb[1]);
  const float m_vv = pa[2] + pb[2];
  S[2] = ROW ? m_ff : m_vv;  // sum dq dx^2
  S[3] = m_fv;               // sum dq dx dy
  S[4] = ROW ? m_vv : m_ff;  // sum dq dy^2
}

// Renderer backward: quad tasks. A warp takes 8 pieces at a time, 4 lanes ("quad") per piece,
// each lane owning up to four lines of its piece (lines q, q + 4, q + 8, q + 12 of the lane axis):
// the per-piece work outside the pixel loop (work-list entry, piece decode, setup, reduction,
// store) is shared by twice as many pieces per warp as with octets, which at 4K is a third of the
// backward. Spans per quad lane, packed in two words: word 0 = start | first0 << 4 | len0 << 8 |
// first1 << 13 | len1 << 17, word 1 = first2 | len2 << 4 | first3 << 9 | len3 << 13 (first: the
// line's first step after start, len: its step count; line_span as for the octets).
__device__ __forceinline__ int piece_quads(const float4& geo, const float4& app, int pc, int ox,
                                           int oy, float cutoff, uint32_t* out) {
  const int rx0 = pc & 15, ry0 = (pc >> 4) & 15;
  const int pw = ((pc >> 8) & 15) + 1, ph = ((pc >> 12) & 15) + 1;
  const bool row = pw >= ph;
  const int lane_dim = row ? pw : ph, step_dim = row ? ph : pw;
  const float pxc0 = static_cast<float>(ox + rx0) + 0.5f;
  const float pyc0 = static_cast<float>(oy + ry0) + 0.5f;
  const float fix0 = row ? pxc0 : pyc0;
  const float mean_fix = row ? geo.x : geo.y;
  LineCoef lc = line_coef(row ? geo.z : app.x, row ? app.x : geo.z, geo.w, row ? geo.y : geo.x,
                          row ? pyc0 : pxc0, cutoff);
  lc.pd = lc.pd && step_dim >= kSpanMinSteps;
  int longest = 0;
  for (int q = 0; q < 4; ++q) {
    int lo[4], hi[4];
    int start = 16;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int line = q + 4 * m;
      lo[m] = 0;
      hi[m] = line < lane_dim ? step_dim - 1 : -1;
      const float d = __fsub_rn(fix0 + static_cast<float>(line), mean_fix);
      line_span(lc, d, __fmul_rn(d, d), step_dim, lo[m], hi[m]);
      if (lo[m] <= hi[m]) start = min(start, lo[m]);
    }
    if (start == 16) start = 0;
    uint32_t f[4], n[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const bool has = lo[m] <= hi[m];
      f[m] = has ? static_cast<uint32_t>(lo[m] - start) : 0u;
      n[m] = has ? static_cast<uint32_t>(hi[m] - lo[m] + 1) : 0u;
      longest = max(longest, static_cast<int>(f[m] + n[m]));
    }
    out[2 * q] = static_cast<uint32_t>(start) | f[0] << 4 | n[0] << 8 | f[1] << 13 | n[1] << 17;
    out[2 * q + 1] = f[2] | n[2] << 4 | f[3] << 9 | n[3] << 13;
  }
  return longest;
}

// One quad lane's part of a renderer-backward piece: the octet's backward_piece with four lines
// per lane (same rounding of q), each line's varying offset centred on the ellipse's centre along
// it, v' = v - vc with vc = -i01 f / coef_var, so that the mean gradient's sums
//   sum dq (c_fix f + c_var v) = (c_fix f + c_var vc) P0 + c_var P1'
// combine terms of the size of the result: for a rotated, elongated gaussian c_fix f and c_var v
// are large and nearly cancel along the line (by the factor i00 i11 / det, which grows with the
// aspect ratio squared), and accumulating sum dq v itself would carry that cancellation into
// float32 sums -- measured on the 4K frame's most elongated gaussians (aspect ratio 150-180) up to
// 6 times the error of the reference's per-pair sums, and no more than them with the centring.
// Every line has its own accumulators (sums of the same length as an octet lane's; with one
// centre and one second-moment sum shared by the four lines, the band test's worst Cholesky
// gradient error was 2.5 times the float32 reference's). Lines B, C, D run only when some lane of
// the warp has one (any_b, any_c, any_d).
template <bool ROW, bool DEN>
__device__ __forceinline__ void backward_quad(const float4& geo, const float4& app, float wt,
                                              float pxc0, float pyc0, int sidx0, int q4, int start,
                                              const unsigned (&first)[4], const unsigned (&len)[4],
                                              bool any_b, bool any_c, bool any_d, int max_steps,
                                              float cutoff, const float4* s_g, float (&S)[8],
                                              float& Sd) {
  const float fix_base = (ROW ? pxc0 : pyc0) + static_cast<float>(q4);
  const float mean_fix = ROW ? geo.x : geo.y;
  const float coef_fix = ROW ? geo.z : app.x;
  const float coef_var = ROW ? app.x : geo.z;
  float d[4], t[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    d[m] = __fsub_rn(fix_base + static_cast<float>(4 * m), mean_fix);
    t[m] = __fmul_rn(__fmul_rn(d[m], d[m]), coef_fix);
  }
  const float i01 = 0.5f * geo.w;
  float kappa = -__fdividef(i01, coef_var);
  kappa = isfinite(kappa) ? kappa : 0.f;
  constexpr int kStep = ROW ? kGStride : 1;
  constexpr int kLaneStride = ROW ? 1 : kGStride;
  unsigned count = 0;
  bool has[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    count = max(count, first[m] + len[m]);
    has[m] = len[m] > 0;
  }
  const bool any[4] = {true, any_b, any_c, any_d};
  int sidx = sidx0 + q4 * kLaneStride + start * kStep;
  float fvar = (ROW ? pyc0 : pxc0) + static_cast<float>(start);
  float P0[4] = {0.f, 0.f, 0.f, 0.f}, P1[4] = {0.f, 0.f, 0.f, 0.f}, P2[4] = {0.f, 0.f, 0.f, 0.f};
  for (int st = 0; st < max_steps; ++st) {
    const float dv = __fsub_rn(fvar, ROW ? geo.y : geo.x);
    const float sq_v = __fmul_rn(dv, dv);
    const float t_v = __fmul_rn(sq_v, coef_var);
    const bool on = static_cast<unsigned>(st) < count;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      if (!any[m]) continue;
      const float t1 = __fmul_rn(__fmul_rn(d[m], dv), geo.w);
      const float q = ROW ? __fadd_rn(__fadd_rn(t[m], t1), t_v) : __fadd_rn(__fadd_rn(t_v, t1), t[m]);
      const bool in = on && has[m] && q < cutoff;
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
      float e = 0.f, dq = 0.f;
      if (in) {
        gv = s_g[sidx + 4 * m * kLaneStride];
        e = falloff(q);
        float v = gv.x * app.y;
        v = fmaf(gv.y, app.z, v);
        v = fmaf(gv.z, app.w, v);
        if constexpr (DEN) v = fmaf(gv.w, wt, v);
        dq = e * v;
      }
      P0[m] += dq;
      P1[m] = fmaf(dq, fmaf(-kappa, d[m], dv), P1[m]);  // offset from the line's ellipse centre
      P2[m] = fmaf(dq, sq_v, P2[m]);
      S[5] = fmaf(e, gv.x, S[5]);
      S[6] = fmaf(e, gv.y, S[6]);
      S[7] = fmaf(e, gv.z, S[7]);
      if constexpr (DEN) Sd = fmaf(e, gv.w, Sd);
    }
    fvar += 1.f;
    sidx += kStep;
  }
  const float cx_fix = ROW ? geo.z : i01, cx_var = ROW ? i01 : geo.z;
  const float cy_fix = ROW ? i01 : app.x, cy_var = ROW ? app.x : i01;
  float s0 = 0.f, s1 = 0.f, p1 = 0.f, m_ff = 0.f, m_fv = 0.f, m_vv = 0.f;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float vc = kappa * d[m];  // the ellipse's centre along line m (varying-axis offset)
    s0 = fmaf(fmaf(cx_var, vc, cx_fix * d[m]), P0[m], s0);
    s1 = fmaf(fmaf(cy_var, vc, cy_fix * d[m]), P0[m], s1);
    p1 += P1[m];
    m_ff = fmaf(__fmul_rn(d[m], d[m]), P0[m], m_ff);
    m_fv = fmaf(d[m], fmaf(vc, P0[m], P1[m]), m_fv);
    m_vv += P2[m];
  }
  S[0] = fmaf(cx_var, p1, s0);
  S[1] = fmaf(cy_var, p1, s1);
  S[2] = ROW ? m_ff : m_vv;  // sum dq dx^2
  S[3] = m_fv;               // sum dq dx dy
  S[4] = ROW ? m_vv : m_ff;  // sum dq dy^2
}

// Sum of v[k] over the 4 lanes of a quad, transposed: lane q of the quad returns moments 2q and
// 2q + 1 (two shuffle rounds).
__device__ __forceinline__ float2 quad_transpose_reduce8(const float (&v)[8], int lane) {
  const bool u2 = lane & 2, u1 = lane & 1;
  float a[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = u2 ? v[k] : v[k + 4];
    const float keep = u2 ? v[k + 4] : v[k];
    a[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  float b[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = u1 ? a[k] : a[k + 2];
    const float keep = u1 ? a[k + 2] : a[k];
    b[k] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
  }
  return make_float2(b[0], b[1]);
}

// Fused tile sort of the fit raster (direct placement): warp 0 reads tile `tile`'s segment and
// cursor, flags a segment overrun (stats[kStatSegOverflow]) or a list above kFusedSortMax
// (stats[kStatFusedLong]: the chunk re-runs with the separate tile-sort kernel), sorts the list
// ascending in registers and leaves it in s_ids; block 0 retires the projection's stats (what the
// tile-sort kernel does otherwise). Called by every thread of the block; returns the list length
// (0 for a list that is not sorted here, whose results the engine discards).
template <int E>
__device__ __forceinline__ void sort_ids_to_shared(const uint32_t* src, int len, uint32_t* dst, int lane) {
  uint32_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    v[e] = i < len ? src[i] : 0xffffffffu;
  }
  warp_sort_striped<E>(v, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    if (i < len) dst[i] = v[e];
  }
}

__device__ __forceinline__ int fused_tile_sort(const FitRasterArgs& f, const uint32_t* list, int tile,
                                               int2 sg, uint32_t* s_ids, int* s_len) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    // The segment (sg, read before the wait) bounds the list, so the cursor and the segment's
    // first 128 slots are loaded in one round trip; slots past the count are ignored.
    const int sx = sg.x, sy = sg.y;
    constexpr int kPre = 4;
    uint32_t pre[kPre];
    const int cur = f.cursor[tile];
#pragma unroll
    for (int e = 0; e < kPre; ++e) {
      const int i = e * 32 + lane;
      pre[e] = i < sy ? list[sx + i] : 0xffffffffu;
    }
    const int filled = cur - sx;
    const int len = max(min(filled, sy), 0);
    if (lane == 0) {
      if (filled > sy) atomicMax(&f.stats[kStatSegOverflow], 1ull);  // ids spilled past the segment
      if (len > kFusedSortMax) atomicMax(&f.stats[kStatFusedLong], static_cast<unsigned long long>(len));
      *s_len = len <= kFusedSortMax ? len : 0;
    }
#pragma unroll
    for (int e = 0; e < kPre; ++e) {
      if (e * 32 + lane >= len) pre[e] = 0xffffffffu;
    }
    const uint32_t* src = list + sx;
    if (len <= 32) {
      uint32_t v[1] = {pre[0]};
      warp_sort_striped<1>(v, lane);
      if (lane < len) s_ids[lane] = v[0];
    } else if (len <= 64) {
      uint32_t v[2] = {pre[0], pre[1]};
      warp_sort_striped<2>(v, lane);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (e * 32 + lane < len) s_ids[e * 32 + lane] = v[e];
      }
    } else if (len <= 128) {
      warp_sort_striped<4>(pre, lane);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (e * 32 + lane < len) s_ids[e * 32 + lane] = pre[e];
      }
    } else if (len <= 256) {
      sort_ids_to_shared<8>(src, len, s_ids, lane);
    } else if (len <= kFusedSortMax) {
      // 257..512 ids (rare): bitonic network over 512 slots in shared memory, one
      // compare-exchange per pair and step (16 ids per lane in registers would spill).
      for (int i = lane; i < kFusedSortMax; i += 32) s_ids[i] = i < len ? src[i] : 0xffffffffu;
      __syncwarp();
      for (int k = 2; k <= kFusedSortMax; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
          for (int p = lane; p < kFusedSortMax / 2; p += 32) {
            const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));
            const uint32_t x = s_ids[i], y = s_ids[i | j];
            if ((x > y) == ((i & k) == 0)) {
              s_ids[i] = y;
              s_ids[i | j] = x;
            }
          }
          __syncwarp();
        }
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) retire_projection_stats(f.stats, true);
  __syncthreads();
  return *s_len;
}
static_assert(kFusedSortMax == 16 * 32, "the fused sort holds at most 16 ids per lane");

// Register caps (measured on B200): the renderer backward (quad tasks with line spans) is held to
// 64 registers, 8 blocks of 128 threads per SM (4K splat backward 2.56 ms; held to 56 registers,
// 9 blocks, it takes 2.99 ms); the fit kernel without the density channel to 48,
// 10 blocks (no spills; 76.7 -> 76.2 ms per 1024x768 / 50k-gaussian fit; 12 blocks spill and are
// slower); the renderer forward without density to 48, 20 blocks of 64 threads (the reach masks
// would take it to 64 registers; 1.73 -> 1.68 ms per 4K forward call with the cap).
template <int PPT, int MODE, bool DEN, bool FUSE = false>
__global__ void __launch_bounds__(Layout<PPT>::kThreads,
                                  MODE == kBwd ? 8 : (MODE == kFit && !DEN ? 10 : (MODE == kFwd && !DEN ? 20 : 0)))
raster_kernel(const RasterArgs a) {
  using L = Layout<PPT>;
  constexpr bool kDoFwd = MODE != kBwd;
  constexpr bool kDoBwd = MODE == kBwd || MODE == kFit;

  constexpr int kBatch = L::kBatch;
  __shared__ float4 s_geo[kBatch];
  __shared__ float4 s_app[kBatch];
  __shared__ int4 s_rect[kBatch];
  __shared__ float s_wt[DEN ? kBatch : 1];
  __shared__ int s_entry[kDoBwd ? kBatch : 1];
  __shared__ int s_piece[kDoBwd ? kBatch : 1];      // rx0 | ry0 << 4 | (pw-1) << 8 | (ph-1) << 12
  __shared__ float4 s_g[kDoBwd ? kTile * kGStride : 1];  // upstream gradient (r, g, b, density) per pixel
  __shared__ int s_list[kDoBwd ? kBatch : 1];   // batch records sorted by octet steps, descending
  // Line spans of the support ellipse: renderer backward only (see kSpanMinSteps).
  constexpr bool kSpans = MODE == kBwd;
  __shared__ uint32_t s_lanes[kSpans ? kBatch * 8 : 1];  // packed step ranges per (piece, octet lane)
  constexpr int kNB = kBuckets;
  __shared__ int s_wcount[kDoBwd ? L::kWarps : 1][kNB];  // per-warp bucket counts, then starts
  static_assert(kBatch == L::kThreads, "the backward work list assigns one piece per thread");
  static_assert(kNB % 32 == 0 && kNB <= 64, "warp 0 scans kNB / 32 consecutive buckets per lane");
  constexpr int kPerLane = kNB / 32;
  __shared__ int s_next;
  // Renderer forward: the walk is pruned to records whose support ellipse can reach a lane's
  // pixels (line spans along the sub-block's columns, in groups of 4 rows, one word per record,
  // transposed across the warp); the rectangle bit and the exact q test stay per pixel. 4K frame,
  // 1M gaussians (59% of rectangle pixels outside their ellipse): forward call 1.94 -> 1.68 ms.
  // With 2 pixels per lane the same masks cost as much as they saved.
  constexpr bool kEllMask = MODE == kFwd && PPT == 4;
  __shared__ double s_loss[L::kWarps][2];

  // The tile order is read from L2 (__ldcg): the fit raster may run before its predecessor ends
  // (programmatic dependent launch), and the order's buffer was read two iterations ago.
  const int tile = a.fit.tile_order ? __ldcg(&a.fit.tile_order[blockIdx.x]) : static_cast<int>(blockIdx.x);
  const int view = tile / a.tiles_per_view;
  const int tin = tile - view * a.tiles_per_view;
  const int tile_y = tin / a.tiles_x;
  const int tile_x = tin - tile_y * a.tiles_x;
  const int ox = tile_x * kTile, oy = tile_y * kTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sbx = warp % L::kSubX, sby = warp / L::kSubX;
  const int px = ox + sbx * L::kSubW + (lane & 7);
  const float pxc = static_cast<float>(px) + 0.5f;
  int py[PPT];
  float pyc[PPT];
  bool inimg[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    py[k] = oy + sby * L::kSubH + PPT * (lane >> 3) + k;
    pyc[k] = static_cast<float>(py[k]) + 0.5f;
    inimg[k] = px < a.width && py[k] < a.height;
  }
  const int sx0 = ox + sbx * L::kSubW, sy0 = oy + sby * L::kSubH;  // this warp's sub-block
  const int sub_col = lane & 7, sub_row0 = PPT * (lane >> 3);
  const int64_t view_base = static_cast<int64_t>(view) * a.height * a.width;
  // The tile's ids in ascending order: list[range) (tile sort) or the sorted entries (radix path).
  // The fit raster of a direct-placement iteration sorts its own tile's list into s_ids (then the
  // list is [0, len) of s_ids); otherwise the list is ranges[tile] of the tile sort (or of the
  // sorted entries on the radix path).
  static_assert(!FUSE || MODE == kFit, "only the fit raster sorts its own tile");
  __shared__ uint32_t s_ids[FUSE ? kFusedSortMax : 1];
  __shared__ int s_fused_len;
  int2 range;
  if constexpr (FUSE) {
    // Launched as a programmatic dependent of the Adam kernel before it (launch_raster_fit): the
    // block may start while that kernel still runs, and waits here for it to complete (records,
    // lists, cursors). Only after the wait does it let the next Adam kernel launch, so that the
    // next Adam's early loads never overlap the writes of the Adam kernel before this raster.
    // The tile's segment comes from the segment layout, which completed before the Adam kernel
    // started: read it before the wait (from L2: its buffer was read two iterations ago).
    int2 sg = make_int2(0, 0);
    if (threadIdx.x < 32) sg = __ldcg(&a.fit.seg[tile]);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    range = make_int2(0, fused_tile_sort(a.fit, a.list, tile, sg, s_ids, &s_fused_len));
  } else {
    range = a.ranges[tile];
  }
  // Stage records [base, base + n) of this tile's list into shared memory.
  auto stage = [&](int base, int n, bool with_entry) {
    for (int j = threadIdx.x; j < n; j += L::kThreads) {
      uint32_t gid;
      if constexpr (FUSE) {
        gid = s_ids[base + j];
      } else {
        gid = a.presorted ? static_cast<uint32_t>(a.entries[base + j]) : a.list[base + j];
      }
      const GaussRecord r = a.records[gid];
      s_geo[j] = r.geo;
      s_app[j] = r.app;
      s_rect[j] = r.rect;
      const int rx0 = r.rect.x - ox, rx1 = rx0 + r.rect.z;
      const int ry0 = r.rect.y - oy, ry1 = ry0 + r.rect.w;
      if constexpr (DEN) s_wt[j] = a.weights[gid];
      if constexpr (kDoBwd) {
        if (with_entry) {
          const TileSpan sp = a.spans[gid];
          s_entry[j] = a.offsets[gid] + (tile_y - sp.ty0) * sp.ntx + (tile_x - sp.tx0);
          const int px0 = max(rx0, 0), px1 = min(rx1, kTile - 1);
          const int py0 = max(ry0, 0), py1 = min(ry1, kTile - 1);
          s_piece[j] = px0 | (py0 << 4) | ((px1 - px0) << 8) | ((py1 - py0) << 12);
        }
      }
    }
  };

  // ------------------------------------------------------------------ forward
  float acc[PPT][3];
  float accd[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    acc[k][0] = acc[k][1] = acc[k][2] = 0.f;
    accd[k] = 0.f;
  }
  // A list that fits one batch is staged once, with the backward's fields, for both passes.
  const bool single_batch = range.y - range.x <= kBatch;
  if constexpr (kDoFwd) {
    for (int base = range.x; base < range.y; base += kBatch) {
      const int n = min(kBatch, range.y - base);
      __syncthreads();
      stage(base, n, kDoBwd && single_batch);
      __syncthreads();
      // 32 records at a time: each lane learns which of them cover each of its pixels (support
      // rectangle only; the ellipse test stays per pair) from 16 ballots, then walks exactly those,
      // in list order. Pixels outside the image are in no rectangle.
      for (int c = 0; c < n; c += 32) {
        unsigned cbits = 0, rbits = 0;  // record c + lane: covered columns / rows of this sub-block
        if (c + lane < n) {
          const int4 rc = s_rect[c + lane];
          const int clo = max(rc.x - sx0, 0), chi = min(rc.x + rc.z - sx0, L::kSubW - 1);
          const int rlo = max(rc.y - sy0, 0), rhi = min(rc.y + rc.w - sy0, L::kSubH - 1);
          if (clo <= chi && rlo <= rhi) {
            cbits = (0xffu >> (L::kSubW - 1 - chi)) & (0xffu << clo);
            rbits = ((2u << rhi) - 1u) & ~((1u << rlo) - 1u);
          }
        }
        // Bit g*8 + col of record c + lane: its ellipse's span along sub-block column col meets
        // rows 4g .. 4g+3 (a superset: line_span); with lane = g*8 + col that is lane g*8+col's
        // pixel column, so a bit transpose gives each lane its mask over the 32 records.
        uint32_t reach = 0xffffffffu;
        if constexpr (kEllMask) {
          static_assert(L::kSubW == 8 && L::kSubH == 16, "4 groups of 4 rows x 8 columns");
          if (cbits != 0) {
            const float4 geo = s_geo[c + lane];
            const float4 app = s_app[c + lane];
            const LineCoef lc = line_coef(geo.z, app.x, geo.w, geo.y, static_cast<float>(sy0) + 0.5f, a.cutoff);
            if (lc.pd) {
              reach = 0;
#pragma unroll
              for (int b = 0; b < L::kSubW; ++b) {
                const float d = __fsub_rn(static_cast<float>(sx0 + b) + 0.5f, geo.x);
                int lo = 0, hi = L::kSubH - 1;
                line_span(lc, d, __fmul_rn(d, d), L::kSubH, lo, hi);
                if (lo <= hi) {
                  const uint32_t groups = ((2u << (hi >> 2)) - 1u) & ~((1u << (lo >> 2)) - 1u);
                  reach |= ((groups * 0x00204081u) & 0x01010101u) << b;  // group g -> bit 8g
                }
              }
            }
          }
          reach = warp_transpose32(reach, lane);
        }
        unsigned mcol = 0;
#pragma unroll
        for (int b = 0; b < L::kSubW; ++b) {
          const unsigned v = __ballot_sync(0xffffffffu, (cbits >> b) & 1u);
          mcol = sub_col == b ? v : mcol;
        }
        unsigned mpix[PPT];
#pragma unroll
        for (int k = 0; k < PPT; ++k) mpix[k] = 0;
#pragma unroll
        for (int b = 0; b < L::kSubH; ++b) {
          const unsigned v = __ballot_sync(0xffffffffu, (rbits >> b) & 1u);
#pragma unroll
          for (int k = 0; k < PPT; ++k) mpix[k] = sub_row0 + k == b ? v : mpix[k];
        }
        unsigned walk = 0;
#pragma unroll
        for (int k = 0; k < PPT; ++k) {
          mpix[k] &= mcol;
          walk |= mpix[k];
        }
        if constexpr (kEllMask) walk &= reach;
        while (walk) {
          const int jb = __ffs(walk) - 1;
          walk &= walk - 1;
          const int jj = c + jb;
          const float4 geo = s_geo[jj];
          const float4 app = s_app[jj];
          const float dx = __fsub_rn(pxc, geo.x);
          float wt = 0.f;
          if constexpr (DEN) wt = s_wt[jj];
#pragma unroll
          for (int k = 0; k < PPT; ++k) {
            // One flat predicate (rectangle bit and ellipse), no nested branches. The sums are
            // guarded rather than multiplied by zero, so a non-finite colour outside the support
            // leaves a pixel untouched.
            const float dy = __fsub_rn(pyc[k], geo.y);
            const float q = pair_q(dx, dy, geo.z, geo.w, app.x);
            const bool in = ((mpix[k] >> jb) & 1u) && q < a.cutoff;
            if (in) {
              const float e = falloff(q);
              acc[k][0] = fmaf(e, app.y, acc[k][0]);
              acc[k][1] = fmaf(e, app.z, acc[k][1]);
              acc[k][2] = fmaf(e, app.w, acc[k][2]);
              if constexpr (DEN) accd[k] = fmaf(e, wt, accd[k]);
            }
          }
        }
      }
    }
  }

  if constexpr (MODE == kFwd) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      if (!inimg[k]) continue;
      const int64_t p = view_base + static_cast<int64_t>(py[k]) * a.width + px;
      a.out[3 * p] = acc[k][0];
      a.out[3 * p + 1] = acc[k][1];
      a.out[3 * p + 2] = acc[k][2];
      if constexpr (DEN) a.den[p] = accd[k];
    }
    return;
  }

  // ------------------------------------------------------------------ upstream gradient
  float g[PPT][3];
  float gd[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    g[k][0] = g[k][1] = g[k][2] = 0.f;
    gd[k] = 0.f;
  }
  if constexpr (MODE == kBwd) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      if (!inimg[k]) continue;
      const int64_t p = view_base + static_cast<int64_t>(py[k]) * a.width + px;
      if (a.grad_out) {
        g[k][0] = a.grad_out[3 * p];
        g[k][1] = a.grad_out[3 * p + 1];
        g[k][2] = a.grad_out[3 * p + 2];
      }
      if constexpr (DEN) {
        if (a.grad_den) gd[k] = a.grad_den[p];
      }
    }
  }
  if constexpr (MODE == kFit || MODE == kEval) {
    const FitRasterArgs& f = a.fit;
    const float scale = f.view_scale ? f.view_scale[view] : 0.f;
    float sse = 0.f, sse_c = 0.f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      if (!inimg[k]) continue;
      const int64_t p = view_base + static_cast<int64_t>(py[k]) * a.width + px;
      float wpix = 1.f, wpsnr = 1.f;
      if (f.loss_mode != kLossMse) {
        const bool mb = mask_bit(f.mask_bits + static_cast<int64_t>(view) * f.mask_bytes_per_view,
                                 static_cast<int64_t>(py[k]) * a.width + px);
        // Mask coverage penalty coef * mean(coverage * (1 - mask)), coverage = 1 - exp(-density):
        // its gradient reaches the backward as an upstream gradient on the density channel.
        if constexpr (MODE == kFit && DEN) gd[k] = mb ? 0.f : f.coverage_coef * __expf(-accd[k]);
        if (f.loss_mode == kLossMaskWeighted) {
          wpix = mb ? 1.0f : 0.1f;  // 0.1 + 0.9 * mask (fit.py:562)
        } else {
          wpix = mb ? 1.f : 0.f;
          wpsnr = wpix;
        }
      }
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        const float t = f.targets[3 * p + ch];
        const float r = acc[k][ch];
        const float res = __fsub_rn(r, t);
        const float rc = __fsub_rn(fminf(fmaxf(r, 0.f), 1.f), t);
        sse = fmaf(wpix * res, res, sse);
        sse_c = fmaf(wpsnr * rc, rc, sse_c);
        if constexpr (MODE == kFit) g[k][ch] = __fmul_rn(__fmul_rn(res, scale), wpix);
        if (f.render_out) f.render_out[3 * p + ch] = r;
      }
    }
    // Deterministic CTA reduction of the loss numerators.
    const double ws = static_cast<double>(warp_sum(sse));
    const double wc = static_cast<double>(warp_sum(sse_c));
    if (lane == 0) {
      s_loss[warp][0] = ws;
      s_loss[warp][1] = wc;
    }
    __syncthreads();
    if (threadIdx.x == 0 && f.tile_loss) {
      double t0 = 0.0, t1 = 0.0;
      for (int w = 0; w < L::kWarps; ++w) {
        t0 += s_loss[w][0];
        t1 += s_loss[w][1];
      }
      f.tile_loss[2 * tile] = t0;
      f.tile_loss[2 * tile + 1] = t1;
    }
  }

  if constexpr (kDoBwd) {
    // ---------------------------------------------------------------- backward
    // Upstream gradient of every tile pixel into shared memory (zeros outside the image).
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int lx = px - ox, ly = py[k] - oy;
      s_g[ly * kGStride + lx] = make_float4(g[k][0], g[k][1], g[k][2], gd[k]);
    }
    float* partials_f = reinterpret_cast<float*>(a.partials);
    const int r8 = lane & 7;
    for (int base = range.x; base < range.y; base += kBatch) {
      const int n = min(kBatch, range.y - base);
      __syncthreads();
      if (!single_batch || !kDoFwd) stage(base, n, true);
      // Work list: the batch's pieces ordered by bucket, stably (by index inside a bucket), so
      // the 4 pieces of every task -- and the orientation each is traversed in -- depend only on
      // the input. One piece per thread (kBatch == block size); ranks from match_any within a warp,
      // per-warp bucket counts for the order across warps.
      const int jb = threadIdx.x;
      int bucket = kNB;
      if (jb < n) {
        const int pc = s_piece[jb];
        if constexpr (kSpans) {
          bucket = piece_bucket_spans(pc, piece_quads(s_geo[jb], s_app[jb], pc, ox, oy, a.cutoff, &s_lanes[8 * jb]));
        } else {
          bucket = piece_bucket(pc);
        }
      }
      for (int i = threadIdx.x; i < L::kWarps * kNB; i += L::kThreads) (&s_wcount[0][0])[i] = 0;
      if (threadIdx.x == 0) s_next = 0;
      __syncthreads();
      const unsigned peers = __match_any_sync(0xffffffffu, bucket);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      if (bucket < kNB && rank == 0) s_wcount[warp][bucket] = __popc(peers);
      __syncthreads();
      if (warp == 0) {  // lane l owns buckets l * kPerLane ...: start of each (warp, bucket) run
        int total = 0;
#pragma unroll
        for (int u = 0; u < kPerLane; ++u) {
#pragma unroll
          for (int w = 0; w < L::kWarps; ++w) total += s_wcount[w][lane * kPerLane + u];
        }
        int x = total;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += y;
        }
        int run = x - total;
#pragma unroll
        for (int u = 0; u < kPerLane; ++u) {
#pragma unroll
          for (int w = 0; w < L::kWarps; ++w) {
            const int c = s_wcount[w][lane * kPerLane + u];
            s_wcount[w][lane * kPerLane + u] = run;
            run += c;
          }
        }
      }
      __syncthreads();
      if (bucket < kNB) s_list[s_wcount[warp][bucket] + rank] = jb;
      __syncthreads();

      if constexpr (MODE == kBwd) {
        // Quad tasks: 8 pieces per warp, 4 lanes each (backward_quad).
        const int q4 = lane & 3;
        const int n_tasks = (n + 7) >> 3;
        while (true) {
          int task = 0;
          if (lane == 0) task = atomicAdd(&s_next, 1);
          task = __shfl_sync(0xffffffffu, task, 0);
          if (task >= n_tasks) break;
          const int p = 8 * task + (lane >> 2);
          const bool valid = p < n;
          const int j = valid ? s_list[p] : s_list[0];
          const float4 geo = s_geo[j];
          const float4 app = s_app[j];
          const int pc = s_piece[j];
          const int rx0 = pc & 15, ry0 = (pc >> 4) & 15;
          const int pw = ((pc >> 8) & 15) + 1, ph = ((pc >> 12) & 15) + 1;
          // As for the octets: the task runs in its first piece's orientation; a piece of the
          // other orientation walks whole lines.
          const bool row = __shfl_sync(0xffffffffu, pw >= ph, 0);
          const int lane_dim = row ? pw : ph, step_dim = row ? ph : pw;
          int start = 0;
          unsigned first[4] = {0u, 0u, 0u, 0u}, len[4];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            len[m] = valid && q4 + 4 * m < lane_dim ? static_cast<unsigned>(step_dim) : 0u;
          }
          if (valid && (pw >= ph) == row) {
            const uint32_t w0 = s_lanes[8 * j + 2 * q4], w1 = s_lanes[8 * j + 2 * q4 + 1];
            start = w0 & 15;
            first[0] = (w0 >> 4) & 15;
            len[0] = (w0 >> 8) & 31;
            first[1] = (w0 >> 13) & 15;
            len[1] = (w0 >> 17) & 31;
            first[2] = w1 & 15;
            len[2] = (w1 >> 4) & 31;
            first[3] = (w1 >> 9) & 15;
            len[3] = (w1 >> 13) & 31;
          }
          unsigned count = 0;
#pragma unroll
          for (int m = 0; m < 4; ++m) count = max(count, first[m] + len[m]);
          const int max_steps = static_cast<int>(__reduce_max_sync(0xffffffffu, count));
          const bool any_b = __any_sync(0xffffffffu, len[1] > 0);
          const bool any_c = __any_sync(0xffffffffu, len[2] > 0);
          const bool any_d = __any_sync(0xffffffffu, len[3] > 0);
          const float pxc0 = static_cast<float>(ox + rx0) + 0.5f;
          const float pyc0 = static_cast<float>(oy + ry0) + 0.5f;
          float wt = 0.f;
          if constexpr (DEN) wt = s_wt[j];
          float S[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          float Sd = 0.f;
          if (row) {
            backward_quad<true, DEN>(geo, app, wt, pxc0, pyc0, ry0 * kGStride + rx0, q4, start, first, len,
                                     any_b, any_c, any_d, max_steps, a.cutoff, s_g, S, Sd);
          } else {
            backward_quad<false, DEN>(geo, app, wt, pxc0, pyc0, ry0 * kGStride + rx0, q4, start, first, len,
                                      any_b, any_c, any_d, max_steps, a.cutoff, s_g, S, Sd);
          }
          const float2 red = quad_transpose_reduce8(S, lane);
          const int64_t e = s_entry[j];
          // Entries outside [0, capacity) belong to a dropped binning.
          const bool store = valid && e >= 0 && e < a.cap;
          if (store) reinterpret_cast<float2*>(partials_f + 8 * e)[q4] = red;
          if constexpr (DEN) {
            Sd += __shfl_xor_sync(0xffffffffu, Sd, 2);
            Sd += __shfl_xor_sync(0xffffffffu, Sd, 1);
            if (store && q4 == 0) a.partial_d[e] = Sd;
          }
        }
      } else {
        const int n_tasks = (n + 3) >> 2;
        while (true) {
          int task = 0;
          if (lane == 0) task = atomicAdd(&s_next, 1);
          task = __shfl_sync(0xffffffffu, task, 0);
          if (task >= n_tasks) break;
          const int p = 4 * task + (lane >> 3);
          const bool valid = p < n;
          const int j = valid ? s_list[p] : s_list[0];
          const float4 geo = s_geo[j];
          const float4 app = s_app[j];
          const int pc = s_piece[j];
          const int rx0 = pc & 15, ry0 = (pc >> 4) & 15;
          const int pw = ((pc >> 8) & 15) + 1, ph = ((pc >> 12) & 15) + 1;
          // The task runs in the orientation of its first piece (the bucket order groups pieces of
          // one orientation): row-wise, each octet lane owns columns r8 and r8 + 8 of its piece and
          // steps down the rows; column-wise, rows r8 and r8 + 8, stepping across the columns. Any
          // piece is correct in either orientation: one of the other orientation (a task across the
          // boundary of the two bucket groups) walks whole lines.
          const bool row = __shfl_sync(0xffffffffu, pw >= ph, 0);
          const int lane_dim = row ? pw : ph, step_dim = row ? ph : pw;
          // Steps of the lane: whole lines (pixels on for the piece's step count).
          const int my_steps = valid ? step_dim : 0;
          const int start = 0;
          const unsigned a_first = 0, a_len = r8 < lane_dim ? my_steps : 0;
          const unsigned b_first = 0, b_len = r8 + 8 < lane_dim ? my_steps : 0;
          const int max_steps = static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(my_steps)));
          const bool any_b = __any_sync(0xffffffffu, b_len > 0);
          const float pxc0 = static_cast<float>(ox + rx0) + 0.5f;  // integer + 0.5 sums stay exact
          const float pyc0 = static_cast<float>(oy + ry0) + 0.5f;
          float wt = 0.f;
          if constexpr (DEN) wt = s_wt[j];
          float S[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          float Sd = 0.f;
  #define RTGS_PIECE(R)                                                                                  \
    backward_piece<R, DEN>(geo, app, wt, pxc0, pyc0, ry0 * kGStride + rx0, r8, start, a_first, a_len, \
                           b_first, b_len, any_b, max_steps, a.cutoff, s_g, S, Sd)
          if (row) RTGS_PIECE(true); else RTGS_PIECE(false);
  #undef RTGS_PIECE
          const float red = octet_transpose_reduce8(S, lane);
          const int64_t e = s_entry[j];
          // Entries outside [0, capacity) belong to a dropped binning.
          const bool store = valid && e >= 0 && e < a.cap;
          if (store) partials_f[8 * e + r8] = red;
          if constexpr (DEN) {
            Sd += __shfl_xor_sync(0xffffffffu, Sd, 4);
            Sd += __shfl_xor_sync(0xffffffffu, Sd, 2);
            Sd += __shfl_xor_sync(0xffffffffu, Sd, 1);
            if (store && r8 == 0) a.partial_d[e] = Sd;
          }
        }
      }
    }
  }
}

// Deterministic per-view reduction of tile loss numerators: one block per view.
__global__ void __launch_bounds__(kLossThreads)
loss_reduce_kernel(const double* __restrict__ tile_loss, int tiles_per_view, double* dst) {
  reduce_view_loss(tile_loss, tiles_per_view, blockIdx.x, dst);
}

// Pixels per lane: the renderer forward walks each record for a column of 4 pixels (2 warps per
// tile), which halves the per-record walk cost per pixel (4K frame, 1M gaussians: forward call
// 2.28 -> 1.94 ms); the backward variants and the fused fit kernel keep 2 (4 warps per tile: with 4
// they are slower, the backward's octet tasks having fewer warps per tile and the fit's small
// gaussians covering fewer of a lane's 4 rows).
template <int MODE>
constexpr int kPPT = MODE == kFwd ? 4 : 2;

RasterArgs base_args(const BinBuffers& bb, const Geometry& g, float cutoff) {
  RasterArgs a{};
  a.records = bb.records.as<GaussRecord>();
  a.weights = bb.weights.as<float>();
  a.spans = bb.spans.as<TileSpan>();
  a.offsets = bb.offsets.as<int>();
  a.entries = bb.entries[bb.sorted_sel].as<uint64_t>();
  a.ranges = bb.ranges.as<int2>();
  a.list = bb.list.as<uint32_t>();
  a.cap = bb.capacity;
  a.presorted = bb.presorted ? 1 : 0;
  a.height = g.height;
  a.width = g.width;
  a.tiles_x = g.tiles_x;
  a.tiles_per_view = g.tiles_per_view;
  a.cutoff = cutoff;
  return a;
}

template <int MODE, bool DEN, bool FUSE = false>
int launch(const RasterArgs& a, const Geometry& g, cudaStream_t s, const char* name) {
  const int64_t n_tiles = g.n_tiles();
  if (n_tiles == 0) return 0;
  if (n_tiles > INT32_MAX) return set_error(-1, "too many tiles");
  if (FUSE && a.fit.pdl) {
    // Programmatic dependent launch: the blocks are scheduled while the Adam kernel before them
    // finishes, which hides the launch gap between the two.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(n_tiles));
    cfg.blockDim = dim3(Layout<kPPT<MODE>>::kThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, raster_kernel<kPPT<MODE>, MODE, DEN, FUSE>, a), name);
  }
  raster_kernel<kPPT<MODE>, MODE, DEN, FUSE>
      <<<static_cast<unsigned>(n_tiles), Layout<kPPT<MODE>>::kThreads, 0, s>>>(a);
  return check_cuda(cudaGetLastError(), name);
}

int ensure_partials(BinBuffers& bb, bool den, cudaStream_t s) {
  // Entry-sized buffers already hold `capacity` entries; only a first density call allocates.
  if (bb.partials.ptr && (!den || bb.partial_d.ptr)) return 0;
  return ensure_entry_capacity(bb, bb.capacity > 0 ? bb.capacity : 1, den, s);
}

}  // namespace

int launch_raster_forward(const BinBuffers& bb, const Geometry& g, float cutoff, float* out,
                          float* den, cudaStream_t s) {
  RasterArgs a = base_args(bb, g, cutoff);
  a.out = out;
  a.den = den;
  if (den) return launch<kFwd, true>(a, g, s, "raster forward (density)");
  return launch<kFwd, false>(a, g, s, "raster forward");
}

int launch_raster_backward(BinBuffers& bb, const Geometry& g, float cutoff, const float* grad_out,
                           const float* grad_den, cudaStream_t s) {
  const bool den = grad_den != nullptr;
  RTGS_TRY(ensure_partials(bb, den, s));
  RasterArgs a = base_args(bb, g, cutoff);
  a.grad_out = grad_out;
  a.grad_den = grad_den;
  a.partials = bb.partials.as<float4>();
  a.partial_d = bb.partial_d.as<float>();
  if (den) return launch<kBwd, true>(a, g, s, "raster backward (density)");
  return launch<kBwd, false>(a, g, s, "raster backward");
}

int launch_raster_fit(BinBuffers& bb, const Geometry& g, float cutoff, const FitRasterArgs& fa,
                      bool backward, cudaStream_t s) {
  RTGS_TRY(ensure_partials(bb, backward && fa.coverage_coef > 0.f, s));
  RasterArgs a = base_args(bb, g, cutoff);
  a.partials = bb.partials.as<float4>();
  a.fit = fa;
  const bool fuse = fa.seg != nullptr;
  if (fuse && (!backward || !fa.cursor || !fa.stats)) return set_error(-1, "raster fit: incomplete own-sort arguments");
  if (backward && fa.coverage_coef > 0.f) {
    a.partial_d = bb.partial_d.as<float>();
    if (fuse) return launch<kFit, true, true>(a, g, s, "raster fit (coverage, own sort)");
    return launch<kFit, true>(a, g, s, "raster fit (coverage)");
  }
  if (backward && fuse) return launch<kFit, false, true>(a, g, s, "raster fit (own sort)");
  if (backward) return launch<kFit, false>(a, g, s, "raster fit");
  return launch<kEval, false>(a, g, s, "raster eval");
}

int launch_loss_reduce(const double* tile_loss, const Geometry& g, double* dst, cudaStream_t s) {
  if (g.n_views == 0) return 0;
  loss_reduce_kernel<<<g.n_views, kLossThreads, 0, s>>>(tile_loss, g.tiles_per_view, dst);
  return check_cuda(cudaGetLastError(), "loss_reduce_kernel");
}

}  // namespace rtgs2d
