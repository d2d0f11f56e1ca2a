// Tile binning: every gaussian with non-empty support is listed once in each 16x16 tile its
// support rectangle touches, and each tile's list must be read in ascending gaussian index -- the
// order in which the reference's index_add sums a pixel (renderer2d.py:228-253). The reference
// itself has no binning (one CUDA block per gaussian, renderer2d_ext.cu:26-85); this replaces its
// per-pair global atomics with per-tile gathers.
//
// Two ways to build the lists, both deterministic in what the raster kernels read:
//   tile scatter (default)  the projection counts entries per tile (and in the fit loop emits the
//                           (tile, id) entries); an inclusive scan of the tile counts gives every
//                           tile's [start, end); each entry claims a slot in its tile by counting
//                           that tile's count back down (so the counts are zero again for the next
//                           projection) -- emitted entries one thread each (scatter_kernel), else
//                           every gaussian its own tiles' slots (place_kernel) -- and one warp per
//                           tile then sorts the tile's ids (lists up to kSegSortMax).
//   radix                   entries emitted gaussian-major as (tile key << 32 | id), stable radix
//                           sort by key (sort.cu), per-tile ranges; used when some tile list is
//                           longer than kSegSortMax. Emission order must follow the gaussian
//                           index, so this path first recomputes the entry offsets as an ordered
//                           exclusive scan of the per-gaussian counts.
// Entry indices (offsets[g] + local tile index) address the backward's per-(gaussian, tile)
// gradient moments on both paths.
#include <cub/device/device_scan.cuh>

#include "internal.h"
#include "kernels.cuh"

namespace rtgs2d {
namespace {

constexpr int kThreads = 256;

// Entries of every gaussian, (tile key << 32 | id) at offsets[g] + j, up to the capacity. With
// `stats` (radix path) thread 0 also retires the projection's stats (slots 0-1 kept).
__global__ void __launch_bounds__(kThreads)
emit_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
            const TileSpan* __restrict__ spans, int tiles_x, int64_t cap,
            unsigned long long* __restrict__ stats, uint64_t* __restrict__ entries) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i == 0 && stats) retire_projection_stats(stats, false);
  int cnt = 0, off = 0;
  TileSpan sp{0, 0, 1, 0};
  if (i < m) {
    cnt = counts[i];
    if (cnt > 0) {
      off = offsets[i];
      sp = spans[i];
    }
  }
  for_each_span_tile(i, cnt, sp, off, tiles_x, [&](long long g, int j, int key, int g_off) {
    const int64_t e = static_cast<int64_t>(g_off) + j;
    if (g_off >= 0 && e < cap) {
      entries[e] = (static_cast<uint64_t>(key) << 32) | static_cast<uint64_t>(g);
    }
  });
}

// One thread per emitted entry: its slot in its tile is tile_end[t] minus the tile count before
// this entry counted it down, i.e. a unique slot of [end - count, end). The counts end at zero,
// ready for the next projection.
__global__ void __launch_bounds__(kThreads)
scatter_kernel(const uint64_t* __restrict__ entries, const unsigned long long* __restrict__ stats,
               int64_t cap, const int* __restrict__ tile_end, int* __restrict__ tile_count,
               uint32_t* __restrict__ list) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t n_all = static_cast<int64_t>(stats[kStatEntries]);
  const int64_t n = n_all < cap ? n_all : cap;
  if (e >= n) return;
  const uint64_t v = entries[e];
  const int t = static_cast<int>(v >> 32);
  const int pos = tile_end[t] - atomicSub(&tile_count[t], 1);
  if (pos >= 0 && pos < cap) list[pos] = static_cast<uint32_t>(v);
}

// The same slots without the entries in between (projections that only counted): each warp walks
// the entries of its 32 gaussians in gaussian-major order, 32 per round, lane k taking the round's
// k-th entry (its gaussian found by a binary search over the warp's inclusive count scan), and
// claims its slot as scatter_kernel does, tile_end[t] minus the tile count before it counted that
// count down. Consecutive lanes mostly hit one gaussian's consecutive tiles, so a round's atomics
// share cache lines, and the lanes stay busy whatever the spans' sizes. Only entries below the
// capacity are placed, as emit_kernel + scatter_kernel do.
__global__ void __launch_bounds__(kThreads)
place_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
             const TileSpan* __restrict__ spans, int tiles_x, int64_t cap,
             const int* __restrict__ tile_end, int* __restrict__ tile_count,
             uint32_t* __restrict__ list) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  int n_place = 0;
  TileSpan sp{0, 0, 1, 0};
  if (i < m) {
    const int cnt = counts[i];
    if (cnt > 0) {
      const int off = offsets[i];
      sp = spans[i];
      const int64_t room = off >= 0 ? cap - off : 0;  // entries off + j below the capacity
      n_place = static_cast<int>(room < cnt ? (room > 0 ? room : 0) : cnt);
    }
  }
  const int lane = threadIdx.x & 31;
  int incl = n_place;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  const int excl = incl - n_place;
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  for (int base = 0; base < total; base += 32) {
    const int q = base + lane;
    int o = 0;  // owner lane: the number of lanes whose inclusive count is <= q
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1) {
      if (__shfl_sync(0xffffffffu, incl, o + step - 1) <= q) o += step;
    }
    const int j = q - __shfl_sync(0xffffffffu, excl, o);
    const int tx0 = __shfl_sync(0xffffffffu, sp.tx0, o);
    const int ty0 = __shfl_sync(0xffffffffu, sp.ty0, o);
    const int ntx = __shfl_sync(0xffffffffu, sp.ntx, o);
    const int kb = __shfl_sync(0xffffffffu, sp.key_base, o);
    const uint32_t g = static_cast<uint32_t>(__shfl_sync(0xffffffffu, static_cast<int>(i), o));
    if (q < total) {
      const int t = kb + (ty0 + j / ntx) * tiles_x + tx0 + j % ntx;
      const int pos = __ldg(&tile_end[t]) - atomicSub(&tile_count[t], 1);
      if (pos >= 0 && pos < cap) list[pos] = g;
    }
  }
}

// One warp per tile: sort list[start, end) ascending (bitonic network over the length padded to a
// power of two >= 32, padding = 0xffffffff, which no gaussian id reaches).
//   len <= 512   in registers: E = n_pad / 32 values per lane in striped order (element
//                i = e * 32 + lane, coalesced loads and stores); partner strides < 32 are shuffles,
//                strides >= 32 compare-exchanges inside the lane. Fully unrolled per E.
//   len <= kSegSortMax  in shared memory (strides >= 32) plus shuffles per 32-element block.
// Lists longer than kSegSortMax are left as they are and flagged in stats[kStatLongTile] (the
// caller re-bins with the radix path).
constexpr int kTileSortWarps = 4;
constexpr int kRegSortMax = 512;

template <int E>
__device__ __forceinline__ void sort_tile_regs(uint32_t* seg, int len, int lane) {
  uint32_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    v[e] = i < len ? seg[i] : 0xffffffffu;
  }
  warp_sort_striped<E>(v, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    if (i < len) seg[i] = v[e];
  }
}

__device__ __forceinline__ uint32_t bitonic_shfl(uint32_t v, int i, int k, int j_top) {
  const bool up = (i & k) == 0;
#pragma unroll 1
  for (int j = j_top; j > 0; j >>= 1) {
    const uint32_t y = __shfl_xor_sync(0xffffffffu, v, j);
    const bool lower = (i & j) == 0;
    v = (lower == up) ? min(v, y) : max(v, y);
  }
  return v;
}

__global__ void __launch_bounds__(kTileSortWarps * 32)
tile_sort_kernel(const int* __restrict__ tile_end, const int2* __restrict__ tile_seg,
                 const int* __restrict__ cursor, int64_t n_tiles, int64_t cap,
                 unsigned long long* __restrict__ stats, uint32_t* __restrict__ list,
                 int2* __restrict__ ranges) {
  __shared__ uint32_t s_buf[kTileSortWarps][kSegSortMax];
  if (blockIdx.x == 0 && threadIdx.x == 0) retire_projection_stats(stats, true);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kTileSortWarps + warp;
  if (t >= n_tiles) return;
  int64_t start, end;
  if (tile_seg) {  // direct placement: the tile's segment and how far the projection moved its cursor
    const int2 sg = tile_seg[t];
    int cur = lane == 0 ? cursor[t] : 0;
    cur = __shfl_sync(0xffffffffu, cur, 0);
    const int filled = cur - sg.x;
    start = sg.x;
    end = start + (filled < sg.y ? filled : sg.y);
    if (lane == 0 && filled > sg.y) atomicMax(&stats[kStatSegOverflow], 1ull);  // ids spilled past the segment
  } else {    // scatter: inclusive scan of the tile counts
    start = t == 0 ? 0 : tile_end[t - 1];
    end = tile_end[t];
  }
  start = start < cap ? start : cap;
  end = end < cap ? end : cap;
  if (lane == 0) ranges[t] = make_int2(static_cast<int>(start), static_cast<int>(end));
  const int len = static_cast<int>(end - start);
  if (len <= 1) return;
  if (len > kSegSortMax) {
    if (lane == 0) atomicMax(&stats[kStatLongTile], static_cast<unsigned long long>(len));
    return;
  }
  uint32_t* seg = list + start;
  if (len <= 32) return sort_tile_regs<1>(seg, len, lane);
  if (len <= 64) return sort_tile_regs<2>(seg, len, lane);
  if (len <= 128) return sort_tile_regs<4>(seg, len, lane);
  if (len <= 256) return sort_tile_regs<8>(seg, len, lane);
  if (len <= kRegSortMax) return sort_tile_regs<16>(seg, len, lane);
  int n_pad = kRegSortMax * 2;
  while (n_pad < len) n_pad <<= 1;
  uint32_t* b = s_buf[warp];
  for (int c = 0; c < n_pad; c += 32) {  // load + first phase (k <= 32) per 32-element block
    const int i = c + lane;
    uint32_t v = i < len ? seg[i] : 0xffffffffu;
#pragma unroll 1
    for (int k = 2; k <= 32; k <<= 1) v = bitonic_shfl(v, i, k, k >> 1);
    b[i] = v;
  }
  __syncwarp();
  for (int k = 64; k <= n_pad; k <<= 1) {
    for (int j = k >> 1; j >= 32; j >>= 1) {
      for (int p = lane; p < (n_pad >> 1); p += 32) {  // one compare-exchange per pair
        const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));
        const int ixj = i | j;
        const uint32_t x = b[i], y = b[ixj];
        const bool up = (i & k) == 0;
        if ((x > y) == up) {
          b[i] = y;
          b[ixj] = x;
        }
      }
      __syncwarp();
    }
    for (int c = 0; c < n_pad; c += 32) {
      const int i = c + lane;
      b[i] = bitonic_shfl(b[i], i, k, 16);
    }
    __syncwarp();
  }
  for (int i = lane; i < len; i += 32) seg[i] = b[i];
}

// Flag tile lists longer than the raster's shared-memory sort (stats[kStatLongTile] = max length).
__global__ void __launch_bounds__(kThreads)
long_tile_kernel(const int* __restrict__ tile_count, int64_t n_tiles,
                 unsigned long long* __restrict__ stats) {
  int longest = 0;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; t < n_tiles;
       t += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = tile_count[t];
    longest = c > longest ? c : longest;
  }
  if (longest > kSegSortMax) atomicMax(&stats[kStatLongTile], static_cast<unsigned long long>(longest));
}

__global__ void __launch_bounds__(kThreads)
ranges_kernel(const uint64_t* __restrict__ entries, const unsigned long long* __restrict__ stats,
              int64_t cap, int2* __restrict__ ranges) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t n_all = static_cast<int64_t>(stats[kStatEntries]);
  const int64_t n = n_all < cap ? n_all : cap;
  if (i >= n) return;
  const uint32_t k = static_cast<uint32_t>(entries[i] >> 32);
  if (i == 0 || static_cast<uint32_t>(entries[i - 1] >> 32) != k) ranges[k].x = static_cast<int>(i);
  if (i == n - 1 || static_cast<uint32_t>(entries[i + 1] >> 32) != k) ranges[k].y = static_cast<int>(i + 1);
}

// Inclusive scan of up to kSmallScanMax ints by one block (tile counts -> tile ends): one launch
// instead of the device-wide scan's two for the tile counts of ordinary frames.
constexpr int kSmallScanThreads = 1024;
constexpr int kSmallScanMax = 8 * kSmallScanThreads;

__global__ void __launch_bounds__(kSmallScanThreads)
small_inclusive_scan_kernel(const int* __restrict__ in, int* __restrict__ out, int n) {
  __shared__ int s_warp[kSmallScanThreads / 32];
  const int per = (n + kSmallScanThreads - 1) / kSmallScanThreads;
  const int i0 = threadIdx.x * per;
  const int i1 = min(i0 + per, n);
  int sum = 0;
  for (int i = i0; i < i1; ++i) sum += in[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = sum;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = s_warp[lane];
    int x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    s_warp[lane] = x - v;  // exclusive prefix of the warp totals
  }
  __syncthreads();
  int run = s_warp[warp] + incl - sum;
  for (int i = i0; i < i1; ++i) {
    run += in[i];
    out[i] = run;
  }
}

// Exclusive prefix of v over the block (kSmallScanThreads threads); *total gets the block sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  __syncthreads();  // s_warp may still be read by a previous scan
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = s_warp[lane];
    int x = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    s_warp[lane] = x - w;
    if (lane == 31) s_warp[32] = x;
  }
  __syncthreads();
  if (total) *total = s_warp[32];
  return s_warp[warp] + incl - v;
}

// Direct placement layout for the next binning: tile t gets a segment of count + 8 + count / 4
// slots (count = this binning's entries of the tile; exactly count without slack), segments packed
// in tile order and clipped to the list capacity. Counts come from the scan (tile_end, after a
// scatter) or from the current placement (cursor_in - seg_in start: the ids the projection placed,
// including any that overran the segment). The segments and cursors (each set to its segment's
// start) go to seg_out / cursor_out, the other buffer of the pair, so a raster can still read the
// current ones. With `order`, the tiles are also counting-sorted by descending count (capped at
// 1023) into order[]: the next raster's block order. One block (it runs beside the raster, off the
// critical path); each thread owns a run of consecutive tiles.
__global__ void __launch_bounds__(kSmallScanThreads)
layout_kernel(const int* __restrict__ tile_end, const int2* __restrict__ seg_in,
              const int* __restrict__ cursor_in, int n_tiles, int list_cap, bool slack,
              int2* __restrict__ seg_out, int* __restrict__ cursor_out, int* __restrict__ order) {
  __shared__ int s_warp[kSmallScanThreads / 32 + 1];
  __shared__ int s_bin[kSmallScanThreads];
  const int per = (n_tiles + kSmallScanThreads - 1) / kSmallScanThreads;
  const int i0 = min(static_cast<int>(threadIdx.x) * per, n_tiles);
  const int i1 = min(i0 + per, n_tiles);
  auto count = [&](int t) {
    return tile_end ? tile_end[t] - (t > 0 ? tile_end[t - 1] : 0) : cursor_in[t] - seg_in[t].x;
  };
  auto seg_cap = [slack](int c) { return slack ? c + 8 + (c >> 2) : c; };
  auto bin = [](int c) { return kSmallScanThreads - 1 - min(c, kSmallScanThreads - 1); };
  if (order) s_bin[threadIdx.x] = 0;
  __syncthreads();
  int sum = 0;
  for (int t = i0; t < i1; ++t) {
    const int c = count(t);
    sum += seg_cap(c);
    if (order) atomicAdd(&s_bin[bin(c)], 1);
  }
  int start = block_exclusive_scan(sum, s_warp, nullptr);
  for (int t = i0; t < i1; ++t) {
    const int c = count(t);
    const int sc = seg_cap(c);
    const int room = list_cap - start;
    seg_out[t] = make_int2(start, sc < room ? sc : (room > 0 ? room : 0));
    cursor_out[t] = start;
    start += sc;
  }
  if (!order) return;
  const int first = block_exclusive_scan(s_bin[threadIdx.x], s_warp, nullptr);
  s_bin[threadIdx.x] = first;  // every thread read its own bin before the scan's barriers
  __syncthreads();
  for (int t = i0; t < i1; ++t) order[atomicAdd(&s_bin[bin(count(t))], 1)] = t;
}

template <bool INCLUSIVE>
int cub_scan(BinBuffers& bb, const int* in, int* out, int64_t n, cudaStream_t s) {
  size_t bytes = 0;
  if constexpr (INCLUSIVE) {
    RTGS_CUDA(cub::DeviceScan::InclusiveSum(nullptr, bytes, in, out, static_cast<int>(n), s), "scan size query");
  } else {
    RTGS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, bytes, in, out, static_cast<int>(n), s), "scan size query");
  }
  RTGS_TRY(bb.cub_temp.ensure(bytes, s));
  if constexpr (INCLUSIVE) {
    RTGS_CUDA(cub::DeviceScan::InclusiveSum(bb.cub_temp.ptr, bytes, in, out, static_cast<int>(n), s), "scan");
  } else {
    RTGS_CUDA(cub::DeviceScan::ExclusiveSum(bb.cub_temp.ptr, bytes, in, out, static_cast<int>(n), s), "scan");
  }
  return 0;
}

unsigned grid_for(int64_t m) { return static_cast<unsigned>((m + kThreads - 1) / kThreads); }

int bin_radix(BinBuffers& bb, const Geometry& g, int64_t m, int64_t launch_entries, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  RTGS_TRY(bb.ranges.ensure(static_cast<size_t>(n_tiles > 0 ? n_tiles : 1) * sizeof(int2), s));
  RTGS_CUDA(cudaMemsetAsync(bb.ranges.ptr, 0, static_cast<size_t>(n_tiles) * sizeof(int2), s),
            "memset ranges");
  bb.presorted = true;
  bb.counts_cleared = false;
  if (m == 0 || bb.capacity == 0 || launch_entries == 0) return 0;
  RTGS_TRY(cub_scan<false>(bb, bb.counts.as<int>(), bb.offsets.as<int>(), m, s));
  RTGS_TRY(bb.sort_counts.ensure(sort_counts_bytes(), s));
  emit_kernel<<<grid_for(m), kThreads, 0, s>>>(m, bb.counts.as<int>(), bb.offsets.as<int>(),
                                                bb.spans.as<TileSpan>(), g.tiles_x, bb.capacity,
                                                bb.stats.as<unsigned long long>(),
                                                bb.entries[0].as<uint64_t>());
  RTGS_CUDA(cudaGetLastError(), "emit_kernel");
  RTGS_TRY(radix_sort_entries(bb.entries[0].as<uint64_t>(), bb.entries[1].as<uint64_t>(),
                              bb.stats.as<unsigned long long>() + kStatEntries, bb.capacity,
                              key_bits_for(n_tiles), bb.sort_counts.as<int>(), s, &bb.sorted_sel));
  ranges_kernel<<<grid_for(launch_entries), kThreads, 0, s>>>(
      bb.entries[bb.sorted_sel].as<uint64_t>(), bb.stats.as<unsigned long long>(), bb.capacity,
      bb.ranges.as<int2>());
  return check_cuda(cudaGetLastError(), "ranges_kernel");
}

int bin_scatter(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  RTGS_TRY(bb.tile_end.ensure(static_cast<size_t>(n_tiles > 0 ? n_tiles : 1) * sizeof(int), s));
  bb.presorted = false;
  bb.counts_cleared = false;
  if (n_tiles == 0) return 0;
  if (n_tiles <= kSmallScanMax) {
    small_inclusive_scan_kernel<<<1, kSmallScanThreads, 0, s>>>(bb.tile_count.as<int>(),
                                                                bb.tile_end.as<int>(),
                                                                static_cast<int>(n_tiles));
    RTGS_CUDA(cudaGetLastError(), "small_inclusive_scan_kernel");
  } else {
    RTGS_TRY(cub_scan<true>(bb, bb.tile_count.as<int>(), bb.tile_end.as<int>(), n_tiles, s));
  }
  if (m > 0 && bb.capacity > 0 && bb.entries_emitted) {
    scatter_kernel<<<grid_for(bb.capacity), kThreads, 0, s>>>(
        bb.entries[0].as<uint64_t>(), bb.stats.as<unsigned long long>(), bb.capacity,
        bb.tile_end.as<int>(), bb.tile_count.as<int>(), bb.list.as<uint32_t>());
    RTGS_CUDA(cudaGetLastError(), "scatter_kernel");
  } else if (m > 0 && bb.capacity > 0) {
    place_kernel<<<grid_for(m), kThreads, 0, s>>>(m, bb.counts.as<int>(), bb.offsets.as<int>(),
                                                  bb.spans.as<TileSpan>(), g.tiles_x, bb.capacity,
                                                  bb.tile_end.as<int>(), bb.tile_count.as<int>(),
                                                  bb.list.as<uint32_t>());
    RTGS_CUDA(cudaGetLastError(), "place_kernel");
  }
  bb.counts_cleared = true;
  const unsigned blocks = static_cast<unsigned>((n_tiles + kTileSortWarps - 1) / kTileSortWarps);
  RTGS_TRY(bb.ranges.ensure(static_cast<size_t>(n_tiles) * sizeof(int2), s));
  tile_sort_kernel<<<blocks, kTileSortWarps * 32, 0, s>>>(
      bb.tile_end.as<int>(), nullptr, nullptr, n_tiles, bb.capacity,
      bb.stats.as<unsigned long long>(), bb.list.as<uint32_t>(), bb.ranges.as<int2>());
  return check_cuda(cudaGetLastError(), "tile_sort_kernel");
}

}  // namespace

bool direct_binning_supported(const Geometry& g) {
  return g.n_tiles() > 0 && g.n_tiles() <= kDirectMaxTiles;
}

int direct_layout(BinBuffers& bb, const Geometry& g, bool after_scatter, bool slack, int out,
                  int* order, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  if (!direct_binning_supported(g)) return set_error(-1, "direct binning: too many tiles");
  if (out != 0 && out != 1) return set_error(-1, "direct binning: segment buffer must be 0 or 1");
  RTGS_TRY(bb.seg.ensure(static_cast<size_t>(2 * n_tiles) * sizeof(int2), s));
  RTGS_TRY(bb.cursor.ensure(static_cast<size_t>(2 * n_tiles) * sizeof(int), s));
  const int64_t list_cap = static_cast<int64_t>(bb.list.bytes / sizeof(uint32_t));
  const int in = 1 - out;
  layout_kernel<<<1, kSmallScanThreads, 0, s>>>(
      after_scatter ? bb.tile_end.as<int>() : nullptr, bb.seg.as<int2>() + in * n_tiles,
      bb.cursor.as<int>() + in * n_tiles, static_cast<int>(n_tiles),
      static_cast<int>(list_cap < INT32_MAX ? list_cap : INT32_MAX), slack,
      bb.seg.as<int2>() + out * n_tiles, bb.cursor.as<int>() + out * n_tiles, order);
  return check_cuda(cudaGetLastError(), "layout_kernel");
}

int direct_sort(BinBuffers& bb, const Geometry& g, int in, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  if (in != 0 && in != 1) return set_error(-1, "direct binning: segment buffer must be 0 or 1");
  RTGS_TRY(bb.ranges.ensure(static_cast<size_t>(n_tiles) * sizeof(int2), s));
  bb.presorted = false;
  const unsigned blocks = static_cast<unsigned>((n_tiles + kTileSortWarps - 1) / kTileSortWarps);
  tile_sort_kernel<<<blocks, kTileSortWarps * 32, 0, s>>>(
      nullptr, bb.seg.as<int2>() + in * n_tiles, bb.cursor.as<int>() + in * n_tiles, n_tiles,
      static_cast<int64_t>(bb.list.bytes / sizeof(uint32_t)), bb.stats.as<unsigned long long>(),
      bb.list.as<uint32_t>(), bb.ranges.as<int2>());
  return check_cuda(cudaGetLastError(), "tile_sort_kernel");
}

int key_bits_for(int64_t n_tiles) {
  int b = 1;
  while ((int64_t{1} << b) < n_tiles) ++b;
  return b;
}

Geometry make_geometry(int n_views, int height, int width) {
  Geometry g;
  g.n_views = n_views;
  g.height = height;
  g.width = width;
  g.tiles_x = (width + kTile - 1) / kTile;
  g.tiles_y = (height + kTile - 1) / kTile;
  g.tiles_per_view = g.tiles_x * g.tiles_y;
  return g;
}

int reset_tile_counts(BinBuffers& bb, const Geometry& g, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  RTGS_TRY(bb.tile_count.ensure(static_cast<size_t>(n_tiles > 0 ? n_tiles : 1) * sizeof(int), s));
  RTGS_CUDA(cudaMemsetAsync(bb.tile_count.ptr, 0, static_cast<size_t>(n_tiles) * sizeof(int), s),
            "memset tile counts");
  return 0;
}

int ensure_entry_capacity(BinBuffers& bb, int64_t capacity, bool density, cudaStream_t s) {
  const size_t e = static_cast<size_t>(capacity > 0 ? capacity : 1);
  RTGS_TRY(bb.list.ensure(e * sizeof(uint32_t), s));
  RTGS_TRY(bb.entries[0].ensure(e * sizeof(uint64_t), s));
  RTGS_TRY(bb.entries[1].ensure(e * sizeof(uint64_t), s));
  RTGS_TRY(bb.partials.ensure(e * kAccum * sizeof(float), s));
  if (density) RTGS_TRY(bb.partial_d.ensure(e * sizeof(float), s));
  size_t cap = bb.list.bytes / sizeof(uint32_t);
  const size_t caps[3] = {bb.entries[0].bytes / sizeof(uint64_t), bb.entries[1].bytes / sizeof(uint64_t),
                          bb.partials.bytes / (kAccum * sizeof(float))};
  for (size_t c : caps) cap = cap < c ? cap : c;
  if (density) {
    const size_t cap_d = bb.partial_d.bytes / sizeof(float);
    cap = cap < cap_d ? cap : cap_d;
  }
  bb.capacity = static_cast<int64_t>(cap);
  return 0;
}

int check_long_tiles(BinBuffers& bb, const Geometry& g, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  if (n_tiles == 0) return 0;
  int64_t blocks = (n_tiles + kThreads - 1) / kThreads;
  blocks = blocks < 148 ? blocks : 148;
  long_tile_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
      bb.tile_count.as<int>(), n_tiles, bb.stats.as<unsigned long long>());
  return check_cuda(cudaGetLastError(), "long_tile_kernel");
}

int read_bin_stats(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  bb.n_entries = 0;
  bb.n_pairs = 0;
  bb.long_tile = false;
  if (m > INT32_MAX) return set_error(-1, "more than 2^31 gaussians in one call");
  RTGS_TRY(check_long_tiles(bb, g, s));
  if (!bb.host_stats) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&bb.host_stats),
                             kStatSlots * sizeof(unsigned long long)),
              "pinned stats");
  }
  RTGS_CUDA(cudaMemcpyAsync(bb.host_stats, bb.stats.ptr, kStatSlots * sizeof(unsigned long long),
                            cudaMemcpyDeviceToHost, s),
            "stats readback");
  RTGS_CUDA(cudaStreamSynchronize(s), "stats sync");
  const unsigned long long entries = bb.host_stats[kStatEntries];
  bb.n_pairs = static_cast<int64_t>(bb.host_stats[kStatPairs]);
  if (entries > static_cast<unsigned long long>(INT32_MAX)) {
    return set_error(-4, "more than 2^31 (gaussian, tile) entries in one call");
  }
  bb.n_entries = static_cast<int64_t>(entries);
  bb.long_tile = bb.host_stats[kStatLongTile] > 0;
  return 0;
}

int bin_known(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  const bool radix = bb.long_tile;
  const bool have = bb.entries[0].ptr != nullptr &&
                    (radix ? bb.entries[1].ptr != nullptr : bb.list.ptr != nullptr);
  if (bb.capacity < bb.n_entries || !have) {
    RTGS_TRY(ensure_entry_capacity(bb, bb.n_entries, bb.partial_d.ptr != nullptr, s));
  }
  if (radix) return bin_radix(bb, g, m, bb.n_entries, s);
  return bin_scatter(bb, g, m, s);
}

int bin_entries(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  RTGS_TRY(read_bin_stats(bb, g, m, s));
  return bin_known(bb, g, m, s);
}

int bin_entries_async(BinBuffers& bb, const Geometry& g, int64_t m, bool radix, cudaStream_t s) {
  if (m > INT32_MAX) return set_error(-1, "more than 2^31 gaussians in one call");
  if (radix) return bin_radix(bb, g, m, bb.capacity, s);
  return bin_scatter(bb, g, m, s);  // the tile sort flags a list too long for it
}

}  // namespace rtgs2d
