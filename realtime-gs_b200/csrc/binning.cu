// Tile binning: every gaussian with non-empty support is listed once in each 16x16 tile its
// support rectangle touches. Entries are emitted gaussian-major (exclusive scan of per-gaussian
// tile counts) as packed (tile key << 32 | gaussian id) words, then stably radix-sorted by key
// (sort.cu), so inside each tile the list is in ascending gaussian index -- the order in which
// the reference's index_add sums a pixel (renderer2d.py:228-253). The reference itself has no
// binning (one CUDA block per gaussian, renderer2d_ext.cu:26-85); this replaces its per-pair
// global atomics with per-tile gathers.
#include <cub/device/device_scan.cuh>

#include "internal.h"

namespace rtgs2d {
namespace {

constexpr int kThreads = 256;
constexpr int kSmallSpan = 16;  // spans above this are emitted by the whole warp

__global__ void __launch_bounds__(kThreads)
emit_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
            const TileSpan* __restrict__ spans, int tiles_x, int64_t cap,
            unsigned long long* __restrict__ stats, uint64_t* __restrict__ entries) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int lane = threadIdx.x & 31;
  if (i == 0) atomicMax(&stats[kStatMaxEntries], stats[kStatEntries]);
  int cnt = 0, off = 0;
  TileSpan sp{0, 0, 1, 0};
  if (i < m) {
    cnt = counts[i];
    if (cnt > 0) {
      off = offsets[i];
      sp = spans[i];
    }
  }
  if (cnt > 0 && cnt <= kSmallSpan) {
    for (int j = 0; j < cnt && off + j < cap; ++j) {
      const int ty = sp.ty0 + j / sp.ntx;
      const int tx = sp.tx0 + j % sp.ntx;
      const uint64_t key = static_cast<uint64_t>(sp.key_base + ty * tiles_x + tx);
      entries[off + j] = (key << 32) | static_cast<uint64_t>(i);
    }
  }
  unsigned big = __ballot_sync(0xffffffffu, cnt > kSmallSpan);
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    const int c = __shfl_sync(0xffffffffu, cnt, src);
    const int o = __shfl_sync(0xffffffffu, off, src);
    const int tx0 = __shfl_sync(0xffffffffu, sp.tx0, src);
    const int ty0 = __shfl_sync(0xffffffffu, sp.ty0, src);
    const int ntx = __shfl_sync(0xffffffffu, sp.ntx, src);
    const int kb = __shfl_sync(0xffffffffu, sp.key_base, src);
    const uint64_t gid = static_cast<uint64_t>(blockIdx.x) * kThreads + (threadIdx.x & ~31) + src;
    for (int j = lane; j < c && o + j < cap; j += 32) {
      const int ty = ty0 + j / ntx;
      const int tx = tx0 + j % ntx;
      const uint64_t key = static_cast<uint64_t>(kb + ty * tiles_x + tx);
      entries[o + j] = (key << 32) | gid;
    }
  }
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

int scan_counts(BinBuffers& bb, int64_t m, cudaStream_t s) {
  size_t scan_bytes = 0;
  RTGS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, bb.counts.as<int>(),
                                          bb.offsets.as<int>(), static_cast<int>(m), s),
            "scan size query");
  RTGS_TRY(bb.cub_temp.ensure(scan_bytes, s));
  RTGS_CUDA(cub::DeviceScan::ExclusiveSum(bb.cub_temp.ptr, scan_bytes, bb.counts.as<int>(),
                                          bb.offsets.as<int>(), static_cast<int>(m), s),
            "scan");
  return 0;
}

int emit_sort_ranges(BinBuffers& bb, const Geometry& g, int64_t m, int64_t launch_entries,
                     cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  RTGS_TRY(bb.ranges.ensure(static_cast<size_t>(n_tiles > 0 ? n_tiles : 1) * sizeof(int2), s));
  RTGS_CUDA(cudaMemsetAsync(bb.ranges.ptr, 0, static_cast<size_t>(n_tiles) * sizeof(int2), s),
            "memset ranges");
  if (m == 0 || bb.capacity == 0 || launch_entries == 0) return 0;
  RTGS_TRY(bb.sort_counts.ensure(sort_counts_bytes(), s));
  emit_kernel<<<static_cast<unsigned>((m + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.spans.as<TileSpan>(), g.tiles_x,
      bb.capacity, bb.stats.as<unsigned long long>(), bb.entries[0].as<uint64_t>());
  RTGS_CUDA(cudaGetLastError(), "emit_kernel");
  RTGS_TRY(radix_sort_entries(bb.entries[0].as<uint64_t>(), bb.entries[1].as<uint64_t>(),
                              bb.stats.as<unsigned long long>() + kStatEntries, bb.capacity,
                              key_bits_for(n_tiles), bb.sort_counts.as<int>(), s, &bb.sorted_sel));
  ranges_kernel<<<static_cast<unsigned>((launch_entries + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      bb.entries[bb.sorted_sel].as<uint64_t>(), bb.stats.as<unsigned long long>(), bb.capacity,
      bb.ranges.as<int2>());
  return check_cuda(cudaGetLastError(), "ranges_kernel");
}

}  // namespace

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

int ensure_entry_capacity(BinBuffers& bb, int64_t capacity, bool density, cudaStream_t s) {
  const size_t e = static_cast<size_t>(capacity > 0 ? capacity : 1);
  RTGS_TRY(bb.entries[0].ensure(e * sizeof(uint64_t), s));
  RTGS_TRY(bb.entries[1].ensure(e * sizeof(uint64_t), s));
  RTGS_TRY(bb.partials.ensure(e * kAccum * sizeof(float), s));
  if (density) RTGS_TRY(bb.partial_d.ensure(e * sizeof(float), s));
  const size_t cap_e = bb.entries[0].bytes / sizeof(uint64_t);
  const size_t cap_e1 = bb.entries[1].bytes / sizeof(uint64_t);
  const size_t cap_p = bb.partials.bytes / (kAccum * sizeof(float));
  size_t cap = cap_e < cap_e1 ? cap_e : cap_e1;
  cap = cap < cap_p ? cap : cap_p;
  if (density) {
    const size_t cap_d = bb.partial_d.bytes / sizeof(float);
    cap = cap < cap_d ? cap : cap_d;
  }
  bb.capacity = static_cast<int64_t>(cap);
  return 0;
}

int bin_entries(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  bb.n_entries = 0;
  bb.n_pairs = 0;
  if (m > INT32_MAX) return set_error(-1, "more than 2^31 gaussians in one call");
  if (m > 0) RTGS_TRY(scan_counts(bb, m, s));
  if (!bb.host_stats) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&bb.host_stats),
                             kStatSlots * sizeof(unsigned long long)),
              "pinned stats");
  }
  RTGS_CUDA(cudaMemcpyAsync(bb.host_stats, bb.stats.ptr, 2 * sizeof(unsigned long long),
                            cudaMemcpyDeviceToHost, s),
            "stats readback");
  RTGS_CUDA(cudaStreamSynchronize(s), "stats sync");
  const unsigned long long entries = bb.host_stats[kStatEntries];
  bb.n_pairs = static_cast<int64_t>(bb.host_stats[kStatPairs]);
  if (entries > static_cast<unsigned long long>(INT32_MAX)) {
    return set_error(-4, "more than 2^31 (gaussian, tile) entries in one call");
  }
  bb.n_entries = static_cast<int64_t>(entries);
  if (bb.capacity < bb.n_entries || bb.entries[0].ptr == nullptr) {
    RTGS_TRY(ensure_entry_capacity(bb, bb.n_entries, bb.partial_d.ptr != nullptr, s));
  }
  return emit_sort_ranges(bb, g, m, bb.n_entries, s);
}

int bin_entries_async(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  if (m > INT32_MAX) return set_error(-1, "more than 2^31 gaussians in one call");
  if (m > 0) RTGS_TRY(scan_counts(bb, m, s));
  return emit_sort_ranges(bb, g, m, bb.capacity, s);
}

}  // namespace rtgs2d
