// Tile binning: every gaussian with non-empty support is listed once in each 16x16 tile its
// support rectangle touches. Entries are emitted gaussian-major (exclusive scan of per-gaussian
// tile counts), then stably radix-sorted by tile key, so inside each tile the list is in
// ascending gaussian index -- the order in which the reference's index_add sums a pixel
// (renderer2d.py:228-253). The reference itself has no binning (one CUDA block per gaussian,
// renderer2d_ext.cu:26-85); this replaces its per-pair global atomics with per-tile gathers.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "internal.h"

namespace rtgs2d {
namespace {

constexpr int kThreads = 256;
constexpr int kSmallSpan = 16;  // spans above this are emitted by the whole warp

__global__ void __launch_bounds__(kThreads)
emit_kernel(int64_t m, const int* __restrict__ counts, const int* __restrict__ offsets,
            const TileSpan* __restrict__ spans, int tiles_x, uint32_t* __restrict__ keys,
            uint32_t* __restrict__ vals) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int lane = threadIdx.x & 31;
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
    for (int j = 0; j < cnt; ++j) {
      const int ty = sp.ty0 + j / sp.ntx;
      const int tx = sp.tx0 + j % sp.ntx;
      keys[off + j] = static_cast<uint32_t>(sp.key_base + ty * tiles_x + tx);
      vals[off + j] = static_cast<uint32_t>(i);
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
    const uint32_t gid = static_cast<uint32_t>(blockIdx.x * kThreads + (threadIdx.x & ~31) + src);
    for (int j = lane; j < c; j += 32) {
      const int ty = ty0 + j / ntx;
      const int tx = tx0 + j % ntx;
      keys[o + j] = static_cast<uint32_t>(kb + ty * tiles_x + tx);
      vals[o + j] = gid;
    }
  }
}

__global__ void __launch_bounds__(kThreads)
ranges_kernel(int64_t n, const uint32_t* __restrict__ keys, int2* __restrict__ ranges) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= n) return;
  const uint32_t k = keys[i];
  if (i == 0 || keys[i - 1] != k) ranges[k].x = static_cast<int>(i);
  if (i == n - 1 || keys[i + 1] != k) ranges[k].y = static_cast<int>(i + 1);
}

int bits_for(int64_t n_keys) {
  int b = 1;
  while ((int64_t{1} << b) < n_keys) ++b;
  return b;
}

}  // namespace

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

int bin_entries(BinBuffers& bb, const Geometry& g, int64_t m, cudaStream_t s) {
  const int64_t n_tiles = g.n_tiles();
  RTGS_TRY(bb.ranges.ensure(static_cast<size_t>(n_tiles > 0 ? n_tiles : 1) * sizeof(int2), s));
  RTGS_CUDA(cudaMemsetAsync(bb.ranges.ptr, 0, static_cast<size_t>(n_tiles) * sizeof(int2), s),
            "memset ranges");
  bb.n_entries = 0;
  bb.n_pairs = 0;
  if (m == 0) return 0;
  if (m > INT32_MAX) return set_error(-1, "more than 2^31 gaussians in one call");

  // 1. exclusive scan of per-gaussian tile counts -> entry offsets.
  size_t scan_bytes = 0;
  RTGS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, bb.counts.as<int>(),
                                          bb.offsets.as<int>(), static_cast<int>(m), s),
            "scan size query");
  RTGS_TRY(bb.cub_temp.ensure(scan_bytes, s));
  RTGS_CUDA(cub::DeviceScan::ExclusiveSum(bb.cub_temp.ptr, scan_bytes, bb.counts.as<int>(),
                                          bb.offsets.as<int>(), static_cast<int>(m), s),
            "scan");

  // 2. entry count -> host (the one host synchronisation of a render / fit iteration).
  if (!bb.host_stats) {
    RTGS_CUDA(cudaMallocHost(reinterpret_cast<void**>(&bb.host_stats), 2 * sizeof(unsigned long long)),
              "pinned stats");
  }
  RTGS_CUDA(cudaMemcpyAsync(bb.host_stats, bb.stats.ptr, 2 * sizeof(unsigned long long),
                            cudaMemcpyDeviceToHost, s),
            "stats readback");
  RTGS_CUDA(cudaStreamSynchronize(s), "stats sync");
  const unsigned long long entries = bb.host_stats[0];
  bb.n_pairs = static_cast<int64_t>(bb.host_stats[1]);
  if (entries > static_cast<unsigned long long>(INT32_MAX)) {
    return set_error(-4, "more than 2^31 (gaussian, tile) entries in one call");
  }
  bb.n_entries = static_cast<int64_t>(entries);
  if (entries == 0) return 0;
  const size_t e = static_cast<size_t>(entries);

  for (int k = 0; k < 2; ++k) {
    RTGS_TRY(bb.keys[k].ensure(e * sizeof(uint32_t), s));
    RTGS_TRY(bb.vals[k].ensure(e * sizeof(uint32_t), s));
  }

  // 3. emit (tile key, gaussian id), gaussian-major.
  emit_kernel<<<static_cast<unsigned>((m + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      m, bb.counts.as<int>(), bb.offsets.as<int>(), bb.spans.as<TileSpan>(), g.tiles_x,
      bb.keys[0].as<uint32_t>(), bb.vals[0].as<uint32_t>());
  RTGS_CUDA(cudaGetLastError(), "emit_kernel");

  // 4. stable LSD radix sort on the significant key bits only.
  cub::DoubleBuffer<uint32_t> dk(bb.keys[0].as<uint32_t>(), bb.keys[1].as<uint32_t>());
  cub::DoubleBuffer<uint32_t> dv(bb.vals[0].as<uint32_t>(), bb.vals[1].as<uint32_t>());
  const int end_bit = bits_for(n_tiles);
  size_t sort_bytes = 0;
  RTGS_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, dk, dv, static_cast<int>(e), 0,
                                            end_bit, s),
            "sort size query");
  RTGS_TRY(bb.cub_temp.ensure(sort_bytes, s));
  RTGS_CUDA(cub::DeviceRadixSort::SortPairs(bb.cub_temp.ptr, sort_bytes, dk, dv,
                                            static_cast<int>(e), 0, end_bit, s),
            "sort");
  bb.sorted_sel = dk.selector;

  // 5. per-tile [start, end) ranges.
  ranges_kernel<<<static_cast<unsigned>((e + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      static_cast<int64_t>(e), bb.keys[bb.sorted_sel].as<uint32_t>(), bb.ranges.as<int2>());
  return check_cuda(cudaGetLastError(), "ranges_kernel");
}

}  // namespace rtgs2d
