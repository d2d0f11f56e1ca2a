// Device helpers shared by the projection, finalisation and Adam kernels.
#pragma once

#include "internal.h"

namespace rtgs2d {

constexpr int kSmallEntries = 32;  // gaussians with more entries are summed by the whole warp

constexpr int kSmallSpan = 16;  // tile spans above this are walked by the whole warp

// Threads per block of the per-gaussian kernels (projection, finalisation, Adam) and of the loss
// reduction: 128 spreads the latency-bound per-gaussian kernels over the SMs in smaller blocks.
constexpr int kProjThreads = 128;

struct ProjOut {
  GaussRecord* records;
  float* weights;  // nullable
  TileSpan* spans;
  int* counts;
  int* offsets;               // entry index of each gaussian's first tile
  int* tile_count;            // entries per tile (atomic; emitted entries only)
  uint64_t* entries;          // null: count every entry; else emit (tile key << 32 | id) at
  int64_t cap;                //   each entry index below cap and count only those
  const uint8_t* active;      // null: every gaussian is live; else 0 = parked (not rendered)
  uint32_t* list;             // non-null: direct placement; tile_count[t] is then tile t's cursor
  int64_t list_cap;           //   (next free list position) and ids go to list below list_cap
  unsigned long long* stats;  // kStat* slots
  int tiles_x;
};

// Call f(gaussian id, local tile index j, tile key, payload of that gaussian) for every tile of
// every active lane's span. Spans up to kSmallSpan tiles are walked by their own lane, longer ones
// by the whole warp (the owner's payload travels with its span); all lanes of the warp must call
// this.
template <typename F>
__device__ __forceinline__ void for_each_span_tile(int64_t gid, int cnt, const TileSpan& sp,
                                                   int payload, int tiles_x, F&& f) {
  if (cnt > 0 && cnt <= kSmallSpan) {
    int tx = sp.tx0, ty = sp.ty0;
    for (int j = 0; j < cnt; ++j) {
      f(gid, j, sp.key_base + ty * tiles_x + tx, payload);
      if (++tx == sp.tx0 + sp.ntx) {
        tx = sp.tx0;
        ++ty;
      }
    }
  }
  const int lane = threadIdx.x & 31;
  unsigned big = __ballot_sync(0xffffffffu, cnt > kSmallSpan);
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    const int c = __shfl_sync(0xffffffffu, cnt, src);
    const int tx0 = __shfl_sync(0xffffffffu, sp.tx0, src);
    const int ty0 = __shfl_sync(0xffffffffu, sp.ty0, src);
    const int ntx = __shfl_sync(0xffffffffu, sp.ntx, src);
    const int kb = __shfl_sync(0xffffffffu, sp.key_base, src);
    const int pl = __shfl_sync(0xffffffffu, payload, src);
    const long long g = __shfl_sync(0xffffffffu, static_cast<long long>(gid), src);
    for (int j = lane; j < c; j += 32) {
      const int ty = ty0 + j / ntx;
      const int tx = tx0 + j % ntx;
      f(g, j, kb + ty * tiles_x + tx, pl);
    }
  }
}

// Direct placement of gaussian gid into the segments of the tiles of its span: the tile's cursor
// (set to its segment's start by the layout) is advanced by one atomic, whose old value is the
// entry's list position. Nothing here checks the segment's end: the tile sort compares each
// cursor with its segment and flags an overrun in stats[kStatSegOverflow] (the chunk is then
// re-binned and re-run, so ids that an overrun wrote into a neighbouring segment are never used);
// positions past the list capacity are not written. Two halves, so the caller can overlap their
// round trips with its own: direct_reserve issues a small span's cursor atomics (nothing waits on
// them yet); direct_commit stores the ids, and walks spans longer than kSmallSpan with the whole
// warp (all lanes of the warp must call it).
struct DirectSlots {
  int pos[kSmallSpan];
};

__device__ __forceinline__ void direct_reserve(int cnt, const TileSpan& sp, const ProjOut& o,
                                               DirectSlots& d) {
  if (cnt <= 0 || cnt > kSmallSpan) return;
  int tx = sp.tx0, ty = sp.ty0;
#pragma unroll
  for (int j = 0; j < kSmallSpan; ++j) {
    if (j < cnt) {
      const int t = sp.key_base + ty * o.tiles_x + tx;
      d.pos[j] = atomicAdd(&o.tile_count[t], 1);
      if (++tx == sp.tx0 + sp.ntx) {
        tx = sp.tx0;
        ++ty;
      }
    }
  }
}

__device__ __forceinline__ void direct_commit(int64_t gid, int cnt, const TileSpan& sp,
                                              const ProjOut& o, const DirectSlots& d) {
  if (cnt > 0 && cnt <= kSmallSpan) {
#pragma unroll
    for (int j = 0; j < kSmallSpan; ++j) {
      if (j < cnt && d.pos[j] < o.list_cap) o.list[d.pos[j]] = static_cast<uint32_t>(gid);
    }
  }
  const int lane = threadIdx.x & 31;
  unsigned big = __ballot_sync(0xffffffffu, cnt > kSmallSpan);
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    const int c = __shfl_sync(0xffffffffu, cnt, src);
    const int tx0 = __shfl_sync(0xffffffffu, sp.tx0, src);
    const int ty0 = __shfl_sync(0xffffffffu, sp.ty0, src);
    const int ntx = __shfl_sync(0xffffffffu, sp.ntx, src);
    const int kb = __shfl_sync(0xffffffffu, sp.key_base, src);
    const uint32_t g = static_cast<uint32_t>(__shfl_sync(0xffffffffu, static_cast<long long>(gid), src));
    for (int j = lane; j < c; j += 32) {
      const int t = kb + (ty0 + j / ntx) * o.tiles_x + tx0 + j % ntx;
      const int p = atomicAdd(&o.tile_count[t], 1);
      if (p < o.list_cap) o.list[p] = g;
    }
  }
}

// Record, span, tile count and entry offset of gaussian i. Must be called by every thread of a
// block of kProjThreads threads (it synchronises the block).
//
// Entry offsets: a warp-wide exclusive scan of the tile counts, the warps' totals scanned in
// shared memory, and one atomic on stats[kStatEntries] per block for the block's base (the entry
// and pair counters are single addresses that every block updates, so one update per block
// instead of one per warp keeps them off the critical path). Blocks reserve in arrival order, so
// a gaussian's entry index varies from run to run; nothing reads entries in index order (the
// raster addresses its tile's entries through the gaussian, the gradient gather reads a
// gaussian's own entries), so no result depends on it.
__device__ __forceinline__ void project_tail(int64_t i, bool active, float mx, float my, Conic k,
                                             int x0, int x1, int y0, int y1, long long pixels,
                                             float w, float cr, float cg, float cb, int view,
                                             int tiles_x, int tiles_per_view, const ProjOut& o) {
  int cnt = 0;
  long long pairs = 0;
  TileSpan sp{0, 0, 1, 0};
  if (active) {
    if (pixels > 0 && isfinite(mx) && isfinite(my) && (!o.active || o.active[i])) {
      const int tx0 = x0 / kTile, tx1 = x1 / kTile;
      const int ty0 = y0 / kTile, ty1 = y1 / kTile;
      const int ntx = tx1 - tx0 + 1;
      cnt = ntx * (ty1 - ty0 + 1);
      pairs = pixels;
      sp.tx0 = tx0;
      sp.ty0 = ty0;
      sp.ntx = ntx;
      sp.key_base = view * tiles_per_view;
      o.spans[i] = sp;
      GaussRecord r;
      r.geo = make_float4(mx, my, k.i00, __fmul_rn(2.0f, k.i01));
      r.app = make_float4(k.i11, __fmul_rn(w, cr), __fmul_rn(w, cg), __fmul_rn(w, cb));
      r.rect = make_int4(x0, y0, x1 - x0, y1 - y0);
      o.records[i] = r;
    }
    if (o.weights) o.weights[i] = w;
    o.counts[i] = cnt;
  }
  DirectSlots dslots;  // with direct placement its round trips overlap the offset reservation's
  if (o.list) direct_reserve(cnt, sp, o, dslots);
  const int lane = threadIdx.x & 31;
  int incl = cnt;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  unsigned long long p = static_cast<unsigned long long>(pairs);
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) p += __shfl_xor_sync(0xffffffffu, p, d);
  constexpr int kWarps = kProjThreads / 32;
  __shared__ int s_warp_base[kWarps];
  __shared__ unsigned long long s_warp_pairs[kWarps];
  __shared__ int s_block_base;
  const int warp = threadIdx.x >> 5;
  if (lane == 31) s_warp_base[warp] = incl;
  if (lane == 0) s_warp_pairs[warp] = p;
  __syncthreads();
  if (threadIdx.x == 0) {
    int total = 0;
    unsigned long long block_pairs = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int c = s_warp_base[w];
      s_warp_base[w] = total;
      total += c;
      block_pairs += s_warp_pairs[w];
    }
    s_block_base = total ? static_cast<int>(atomicAdd(&o.stats[kStatEntries],
                                                      static_cast<unsigned long long>(total)))
                         : 0;
    if (block_pairs) {
      atomicAdd(&o.stats[kStatPairs], block_pairs);
      atomicAdd(&o.stats[kStatPairsTotal], block_pairs);
    }
  }
  __syncthreads();
  const int off = s_block_base + s_warp_base[warp] + incl - cnt;
  if (active) o.offsets[i] = off;
  if (o.list) {  // direct placement (warp-uniform choice; all lanes reach this point)
    direct_commit(i, cnt, sp, o, dslots);
    return;
  }
  // Tile counts, and with o.entries the entries themselves (all lanes reach this point). Emitted,
  // only entries that fit the capacity are emitted and counted: the binning stays consistent, and
  // stats[kStatEntries] (all entries) tells the caller it overflowed.
  for_each_span_tile(i, cnt, sp, off, o.tiles_x, [&](long long g, int j, int t, int g_off) {
    if (!o.entries) {
      atomicAdd(&o.tile_count[t], 1);  // result unused: a fire-and-forget reduction
      return;
    }
    const int64_t e = static_cast<int64_t>(g_off) + j;
    if (g_off >= 0 && e < o.cap) {
      atomicAdd(&o.tile_count[t], 1);
      o.entries[e] = (static_cast<uint64_t>(t) << 32) | static_cast<uint64_t>(g);
    }
  });
}

// Retire the projection's stats: the largest entry count so far, copies of the entry and pair
// counts (slots "last"), then slots 0-1 zeroed for the next projection (scatter path and direct
// placement, where nothing later reads them).
__device__ __forceinline__ void retire_projection_stats(unsigned long long* stats, bool zero) {
  const unsigned long long e = stats[kStatEntries];
  atomicMax(&stats[kStatMaxEntries], e);
  stats[kStatLastEntries] = e;
  stats[kStatLastPairs] = stats[kStatPairs];
  if (zero) {
    stats[kStatEntries] = 0;
    stats[kStatPairs] = 0;
  }
}

// Ascending bitonic sort of 32 * E values held by one warp in striped order (value e of lane l is
// element e * 32 + l): partner strides below 32 are shuffles, strides of 32 and more
// compare-exchanges inside the lane. Fully unrolled per E. Used by the tile sort (binning.cu) and
// by the fit raster that sorts its own tile (raster.cu).
template <int E>
__device__ __forceinline__ void warp_sort_striped(uint32_t (&v)[E], int lane) {
#pragma unroll
  for (int k = 2; k <= 32 * E; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int je = j >> 5;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & je) == 0) {
            const bool up = ((e * 32) & k) == 0;  // k >= 64 here: the lane bits do not matter
            const uint32_t x = v[e], y = v[e ^ je];
            v[e] = up ? min(x, y) : max(x, y);
            v[e ^ je] = up ? max(x, y) : min(x, y);
          }
        }
      } else {
        const bool lower = (lane & j) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const bool up = ((e * 32 + lane) & k) == 0;
          const uint32_t y = __shfl_xor_sync(0xffffffffu, v[e], j);
          v[e] = (lower == up) ? min(v[e], y) : max(v[e], y);
        }
      }
    }
  }
}

// Entries at or past the entry capacity were never written (an overflowed binning, whose results
// the caller discards); never read them. A negative offset (an entry count past 2^31, which the
// host rejects after the fact) reads nothing either.
__device__ __forceinline__ int clamp_to_capacity(int cnt, int off, int64_t cap) {
  if (off < 0) return 0;
  const int64_t room = cap - off;
  if (room <= 0) return 0;
  return cnt < room ? cnt : static_cast<int>(room);
}

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
    const float4* p = partials + 2 * static_cast<int64_t>(off);
    // Four entries' loads in flight at a time (predicated past the count, so a gaussian with 1..4
    // entries waits for one round trip); the additions keep the sequential entry order.
    for (int j = 0; j < cnt; j += 4) {
      float4 v[8];
      float vd[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool in = j + u < cnt;
        v[2 * u] = in ? p[2 * (j + u)] : make_float4(0.f, 0.f, 0.f, 0.f);
        v[2 * u + 1] = in ? p[2 * (j + u) + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (DEN) vd[u] = in ? partial_d[off + j + u] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j + u < cnt) {
          mo.s[0] += v[2 * u].x; mo.s[1] += v[2 * u].y; mo.s[2] += v[2 * u].z; mo.s[3] += v[2 * u].w;
          mo.s[4] += v[2 * u + 1].x; mo.s[5] += v[2 * u + 1].y; mo.s[6] += v[2 * u + 1].z;
          mo.s[7] += v[2 * u + 1].w;
          if constexpr (DEN) mo.sd += vd[u];
        }
      }
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

// Conic and Cholesky gradients from a gaussian's summed moments; the Cholesky chain rule uses the
// entries a, b, c of L^-1 that conic_from_chol computed (the same correctly rounded values as
// dividing again).
__device__ __forceinline__ GeoGrad geo_grad(const Moments& mo, const Conic& k, bool want_chol) {
  GeoGrad r;
  r.gmx = mo.s[0];  // the renderer backward applied Sigma^-1 per piece lane
  r.gmy = mo.s[1];
  r.gi00 = -0.5f * mo.s[2];
  r.gi01 = -mo.s[3];
  r.gi11 = -0.5f * mo.s[4];
  r.gl11 = r.gl21 = r.gl22 = 0.f;
  if (want_chol) {
    const float a = k.a, b = k.b, c = k.c;
    const float ga = 2.0f * a * r.gi00;
    const float gb = fmaf(2.0f * b, r.gi00, c * r.gi01);
    const float gc = fmaf(b, r.gi01, 2.0f * c * r.gi11);
    r.gl11 = -a * fmaf(ga, a, gb * b);
    r.gl21 = -gb * a * c;
    r.gl22 = -c * fmaf(gb, b, gc * c);
  }
  return r;
}

// One Adam update of a single float parameter, in the order of torch's single-tensor Adam
// (exp_avg.lerp_, exp_avg_sq.mul_.addcmul_, denom = sqrt(v)/bc2_sqrt + eps, p.addcdiv_). The
// moment updates are rounded as torch rounds them; the square root is the hardware approximation
// (sqrt.approx, relative error ~2^-23), the division by bc2_sqrt a multiplication by its
// reciprocal and the final quotient __fdividef (~2 ulp; denom >= eps, so never the > 2^126 case):
// correctly rounded square roots and divisions are tens of instructions each, 27 of them per
// gaussian on the Adam kernel's dependent chain, and the fit's tolerances are far above ulps.
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void adam_update(float& p, float& m1, float& m2, float g,
                                            const AdamScalars& a) {
  m1 = __fadd_rn(m1, __fmul_rn(a.one_minus_beta1, __fsub_rn(g, m1)));
  m2 = __fadd_rn(__fmul_rn(m2, a.beta2), __fmul_rn(__fmul_rn(a.one_minus_beta2, g), g));
  const float denom = fmaf(sqrt_approx(m2), a.inv_bc2_sqrt, a.eps);
  p = fmaf(a.neg_step_size, __fdividef(m1, denom), p);
}


// Loss numerators of one view: the per-tile (squared error, clamped squared error) pairs summed
// in a fixed order (strided per-thread sums, then a tree), so every caller gets the same bits.
// Called by all kLossThreads threads of a block (the per-gaussian kernels' block size, so that the
// Adam kernel's logging and the evaluation kernel reduce in the same order).
constexpr int kLossThreads = kProjThreads;

__device__ __forceinline__ void reduce_view_loss(const double* __restrict__ tile_loss,
                                                 int tiles_per_view, int view, double* dst) {
  __shared__ double s_loss[2][kLossThreads];
  double a0 = 0.0, a1 = 0.0;
  for (int t = threadIdx.x; t < tiles_per_view; t += kLossThreads) {
    const int64_t idx = static_cast<int64_t>(view) * tiles_per_view + t;
    a0 += tile_loss[2 * idx];
    a1 += tile_loss[2 * idx + 1];
  }
  s_loss[0][threadIdx.x] = a0;
  s_loss[1][threadIdx.x] = a1;
  __syncthreads();
  for (int stride = kLossThreads / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      s_loss[0][threadIdx.x] += s_loss[0][threadIdx.x + stride];
      s_loss[1][threadIdx.x] += s_loss[1][threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    dst[2 * view] = s_loss[0][0];
    dst[2 * view + 1] = s_loss[1][0];
  }
  __syncthreads();  // s_loss may be reused by a next call
}

}  // namespace rtgs2d
