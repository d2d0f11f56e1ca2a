// Stable LSD radix sort of packed 64-bit tile entries (tile key << 32 | gaussian id) by the key.
//
// The item count is read from device memory (the projection's atomic entry counter), clamped to
// the buffer capacity, so a sort can be enqueued without the host knowing the count: no host
// synchronisation per fit iteration. Each pass is reduce-then-scan with a fixed grid:
//   hist     per-block digit counts of a contiguous chunk            counts[digit][block]
//   scan     one block per digit: exclusive scan of its per-block counts, and the digit total
//   scatter  per block: digit starts (scan of the digit totals), per-warp digit counts and bases,
//            then an ordered walk of the chunk
//            32 items at a time; __match_any_sync gives each item its rank among equal digits
//            of the step, so the order of equal keys is preserved (stable).
// Digit width adapts to the key width: ceil(bits / 8) passes of ceil(bits / passes) bits.
#include "internal.h"

namespace rtgs2d {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;

__device__ __forceinline__ void chunk_of(const unsigned long long* d_n, int64_t cap, int64_t& b0,
                                         int64_t& b1) {
  const int64_t n_all = static_cast<int64_t>(*d_n);
  const int64_t n = n_all < cap ? n_all : cap;
  const int64_t g = gridDim.x;
  const int64_t chunk = (n + g - 1) / g;
  b0 = static_cast<int64_t>(blockIdx.x) * chunk;
  if (b0 > n) b0 = n;
  b1 = b0 + chunk < n ? b0 + chunk : n;
}

template <int DBITS>
__device__ __forceinline__ uint32_t digit_of(uint64_t item, int shift) {
  return static_cast<uint32_t>(item >> (32 + shift)) & ((1u << DBITS) - 1u);
}

template <int DBITS>
__global__ void __launch_bounds__(kSortThreads)
sort_hist_kernel(const uint64_t* __restrict__ in, const unsigned long long* __restrict__ d_n,
                 int64_t cap, int shift, int* __restrict__ counts) {
  constexpr int R = 1 << DBITS;
  __shared__ int h[R];
  for (int i = threadIdx.x; i < R; i += kSortThreads) h[i] = 0;
  __syncthreads();
  int64_t b0, b1;
  chunk_of(d_n, cap, b0, b1);
  for (int64_t i = b0 + threadIdx.x; i < b1; i += kSortThreads) {
    atomicAdd(&h[digit_of<DBITS>(in[i], shift)], 1);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < R; d += kSortThreads) counts[d * gridDim.x + blockIdx.x] = h[d];
}

// One block per digit: exclusive scan of that digit's per-block counts (row d of the digit-major
// count matrix) in place, and the digit's total into totals[d].
__global__ void __launch_bounds__(kSortThreads)
sort_digit_scan_kernel(int* __restrict__ counts, int grid, int* __restrict__ totals) {
  __shared__ int s_warp[kSortWarps];
  __shared__ int s_carry;
  const int d = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int* row = counts + static_cast<int64_t>(d) * grid;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < grid; base += kSortThreads) {
    const int i = base + tid;
    const int v = i < grid ? row[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    int before = s_carry;
    for (int ww = 0; ww < warp; ++ww) before += s_warp[ww];
    if (i < grid) row[i] = before + x - v;
    __syncthreads();
    if (tid == kSortThreads - 1) s_carry = before + x;
    __syncthreads();
  }
  if (tid == 0) totals[d] = s_carry;
}

template <int DBITS>
__global__ void __launch_bounds__(kSortThreads)
sort_scatter_kernel(const uint64_t* __restrict__ in, uint64_t* __restrict__ out,
                    const unsigned long long* __restrict__ d_n, int64_t cap, int shift,
                    const int* __restrict__ offsets, const int* __restrict__ totals) {
  constexpr int R = 1 << DBITS;
  __shared__ int s_base[kSortWarps][R];
  __shared__ int s_start[R];
  int64_t b0, b1;
  chunk_of(d_n, cap, b0, b1);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t wlen = (b1 - b0 + kSortWarps - 1) / kSortWarps;
  int64_t w0 = b0 + w * wlen;
  if (w0 > b1) w0 = b1;
  const int64_t w1 = w0 + wlen < b1 ? w0 + wlen : b1;
  for (int i = threadIdx.x; i < kSortWarps * R; i += kSortThreads) (&s_base[0][0])[i] = 0;
  // Global start of every digit: exclusive scan of the digit totals (R <= blockDim).
  const int tid = threadIdx.x;
  const int own = tid < R ? totals[tid] : 0;
  if (tid < R) s_start[tid] = own;
  __syncthreads();
  for (int off = 1; off < R; off <<= 1) {
    const int t = (tid < R && tid >= off) ? s_start[tid - off] : 0;
    __syncthreads();
    if (tid < R) s_start[tid] += t;
    __syncthreads();
  }
  if (tid < R) s_start[tid] -= own;
  __syncthreads();
  for (int64_t i = w0 + lane; i < w1; i += 32) atomicAdd(&s_base[w][digit_of<DBITS>(in[i], shift)], 1);
  __syncthreads();
  for (int d = threadIdx.x; d < R; d += kSortThreads) {
    int run = s_start[d] + offsets[d * gridDim.x + blockIdx.x];
    for (int ww = 0; ww < kSortWarps; ++ww) {
      const int c = s_base[ww][d];
      s_base[ww][d] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t s0 = w0; s0 < w1; s0 += 32) {
    const int64_t i = s0 + lane;
    const bool valid = i < w1;
    const uint64_t item = valid ? in[i] : 0ull;
    const uint32_t d = valid ? digit_of<DBITS>(item, shift) : static_cast<uint32_t>(R);
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    int pos = 0;
    if (valid) pos = s_base[w][d] + __popc(peers & lt);
    __syncwarp();
    if (valid && (peers & lt) == 0) s_base[w][d] += __popc(peers);
    __syncwarp();
    if (valid) out[pos] = item;
  }
}

template <int DBITS>
int launch_pass(const uint64_t* in, uint64_t* out, const unsigned long long* d_n, int64_t cap,
                int shift, int grid, int* counts, cudaStream_t s) {
  sort_hist_kernel<DBITS><<<grid, kSortThreads, 0, s>>>(in, d_n, cap, shift, counts);
  RTGS_CUDA(cudaGetLastError(), "sort_hist_kernel");
  int* totals = counts + static_cast<int64_t>(256) * kSortGrid;
  sort_digit_scan_kernel<<<1 << DBITS, kSortThreads, 0, s>>>(counts, grid, totals);
  RTGS_CUDA(cudaGetLastError(), "sort_digit_scan_kernel");
  sort_scatter_kernel<DBITS><<<grid, kSortThreads, 0, s>>>(in, out, d_n, cap, shift, counts, totals);
  return check_cuda(cudaGetLastError(), "sort_scatter_kernel");
}

}  // namespace

int sort_plan_passes(int key_bits) { return (key_bits + 7) / 8; }

size_t sort_counts_bytes() { return (static_cast<size_t>(256) * kSortGrid + 256) * sizeof(int); }

int radix_sort_entries(uint64_t* buf0, uint64_t* buf1, const unsigned long long* d_n, int64_t cap,
                       int key_bits, int* counts, cudaStream_t s, int* result_sel) {
  const int passes = sort_plan_passes(key_bits);
  const int dbits = (key_bits + passes - 1) / passes;
  // About 4k items per block, at most kSortGrid blocks (the digit-count array is sized for that).
  int64_t want = (cap + 4095) / 4096;
  const int grid = static_cast<int>(want < 1 ? 1 : (want > kSortGrid ? kSortGrid : want));
  uint64_t* bufs[2] = {buf0, buf1};
  int cur = 0;
  for (int p = 0; p < passes; ++p) {
    const int shift = p * dbits;
    uint64_t* in = bufs[cur];
    uint64_t* out = bufs[cur ^ 1];
    int rc = 0;
    switch (dbits) {
      case 1: rc = launch_pass<1>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 2: rc = launch_pass<2>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 3: rc = launch_pass<3>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 4: rc = launch_pass<4>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 5: rc = launch_pass<5>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 6: rc = launch_pass<6>(in, out, d_n, cap, shift, grid, counts, s); break;
      case 7: rc = launch_pass<7>(in, out, d_n, cap, shift, grid, counts, s); break;
      default: rc = launch_pass<8>(in, out, d_n, cap, shift, grid, counts, s); break;
    }
    if (rc) return rc;
    cur ^= 1;
  }
  *result_sel = cur;
  return 0;
}

}  // namespace rtgs2d
