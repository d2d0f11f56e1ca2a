// C ABI: error handling, device buffers, scratch arena and the render entry points.
#include <cmath>
#include <cstdio>
#include <new>
#include <string>
#include <algorithm>
#include <vector>

#include "../../include/rtgs2d.h"
#include "internal.h"

namespace rtgs2d {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return 0;
  // Clear the runtime's last-error slot so a later, unrelated launch check does not report it.
  cudaGetLastError();
  const int code = (err == cudaErrorMemoryAllocation) ? RTGS2D_ERR_ALLOC : RTGS2D_ERR_CUDA;
  return set_error(code, std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                             cudaGetErrorString(err) + ")");
}

int DevBuf::ensure(size_t need, cudaStream_t stream) {
  if (need <= bytes && ptr != nullptr) return 0;
  if (ptr != nullptr) {
    // Queued kernels may still read the old allocation.
    RTGS_CUDA(cudaStreamSynchronize(stream), "sync before buffer growth");
    cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
  }
  size_t grow = need + need / 4;  // headroom so slowly growing workloads do not reallocate often
  grow = (grow + 255) & ~static_cast<size_t>(255);
  if (grow == 0) grow = 256;
  RTGS_CUDA(cudaMalloc(&ptr, grow), "cudaMalloc");
  bytes = grow;
  return 0;
}

void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

void BinBuffers::release() {
  for (DevBuf* b : {&records, &weights, &spans, &counts, &offsets, &list, &tile_count, &tile_end,
                    &entries[0], &entries[1], &ranges, &seg, &cursor, &tile_order, &partials, &partial_d, &cub_temp,
                    &sort_counts, &stats}) {
    b->release();
  }
  if (host_stats) cudaFreeHost(host_stats);
  host_stats = nullptr;
}

BinBuffers::~BinBuffers() { release(); }

}  // namespace rtgs2d

using namespace rtgs2d;

struct rtgs2d_arena {
  int device = 0;
  BinBuffers bb;
  int64_t n_tiles = 0;  // tiles of the last binning
  // Inputs of the last binning if it came from rtgs2d_render_forward (valid = true); any other
  // binning on the arena clears it. rtgs2d_render_backward_after_forward reuses that binning.
  struct ForwardKey {
    const float *xy, *chol, *color, *weight;
    int64_t n_views, n, height, width;
    bool weights_written;
  } last_forward{};
  bool last_forward_valid = false;
  // Stream ordering: every call that touches the arena's buffers first makes its stream wait for
  // the event recorded at the end of the previous such call, then records it again on its own
  // stream. Calls issued on different streams therefore run one after another on the device, so
  // one call's kernels never overwrite records, entries or moments another call's kernels still
  // read (the reference allocated fresh outputs per call, renderer2d_ext.cu:198-199).
  cudaEvent_t done = nullptr;
  bool done_recorded = false;
  ~rtgs2d_arena() {
    if (done) cudaEventDestroy(done);
  }
};

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int check_arena(const rtgs2d_arena* a) {
  if (!a) return set_error(RTGS2D_ERR_INVALID, "arena is NULL");
  int dev = -1;
  RTGS_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != a->device) {
    return set_error(RTGS2D_ERR_INVALID, "arena was created on device " + std::to_string(a->device) +
                                             " but the current device is " + std::to_string(dev));
  }
  return 0;
}

// Orders a call's work on `s` after the previous arena user's (see rtgs2d_arena::done) and, on
// scope exit (error paths included), marks the end of this call's work for the next user.
class ArenaUse {
 public:
  ArenaUse(rtgs2d_arena* a, cudaStream_t s) : a_(a), s_(s) {}
  int begin() {
    if (!a_->done) {
      RTGS_CUDA(cudaEventCreateWithFlags(&a_->done, cudaEventDisableTiming), "cudaEventCreate");
    }
    if (a_->done_recorded) RTGS_CUDA(cudaStreamWaitEvent(s_, a_->done, 0), "cudaStreamWaitEvent");
    active_ = true;
    return 0;
  }
  ~ArenaUse() {
    if (active_ && cudaEventRecord(a_->done, s_) == cudaSuccess) a_->done_recorded = true;
  }

 private:
  rtgs2d_arena* a_;
  cudaStream_t s_;
  bool active_ = false;
};

int check_dims(int64_t m, int64_t n_views, int64_t height, int64_t width) {
  if (m < 0) return set_error(RTGS2D_ERR_INVALID, "number of gaussians must be non-negative");
  if (n_views <= 0) return set_error(RTGS2D_ERR_INVALID, "n_views must be positive");
  if (height <= 0 || width <= 0) {
    return set_error(RTGS2D_ERR_INVALID, "height and width must be positive");
  }
  if (height > 32768 || width > 32768) {
    return set_error(RTGS2D_ERR_CAPACITY, "height and width must be at most 32768");
  }
  const int64_t tiles = n_views * ((height + kTile - 1) / kTile) * ((width + kTile - 1) / kTile);
  if (tiles > INT32_MAX) return set_error(RTGS2D_ERR_CAPACITY, "too many tiles (views x tiles)");
  if (m > INT32_MAX) return set_error(RTGS2D_ERR_CAPACITY, "more than 2^31 gaussians");
  return 0;
}

int require(const void* p, const char* name) {
  if (p == nullptr) return set_error(RTGS2D_ERR_INVALID, std::string(name) + " is NULL");
  return 0;
}

}  // namespace

namespace {

int render_backward(rtgs2d_arena* arena, const float* grad_out, const float* grad_den,
                    const float* xy, const float* chol, const float* color, const float* weight,
                    int64_t n_views, int64_t n, int64_t height, int64_t width, float* grad_xy,
                    float* grad_chol, float* grad_color, float* grad_weight, bool reuse,
                    void* stream) {
  RTGS_TRY(check_arena(arena));
  if (n < 0) return set_error(RTGS2D_ERR_INVALID, "n must be non-negative");
  const int64_t m = n_views * n;
  RTGS_TRY(check_dims(m, n_views, height, width));
  if (m == 0) return RTGS2D_OK;
  RTGS_TRY(require(xy, "xy"));
  RTGS_TRY(require(chol, "chol"));
  RTGS_TRY(require(color, "color"));
  RTGS_TRY(require(weight, "weight"));
  cudaStream_t s = as_stream(stream);
  const Geometry g = make_geometry(static_cast<int>(n_views), static_cast<int>(height),
                                   static_cast<int>(width));
  BinBuffers& bb = arena->bb;
  const bool den = grad_den != nullptr;
  ArenaUse use(arena, s);
  RTGS_TRY(use.begin());
  const rtgs2d_arena::ForwardKey& k = arena->last_forward;
  const bool same = reuse && arena->last_forward_valid && k.xy == xy && k.chol == chol &&
                    k.color == color && k.weight == weight && k.n_views == n_views && k.n == n &&
                    k.height == height && k.width == width && (k.weights_written || !den);
  if (!same) {
    arena->last_forward_valid = false;
    RTGS_TRY(launch_project_chol(bb, g, xy, chol, color, weight, m, n, den, s));
    RTGS_TRY(bin_entries(bb, g, m, s));
    arena->n_tiles = g.n_tiles();
  }
  RTGS_TRY(launch_raster_backward(bb, g, kCutoff, grad_out, grad_den, s));
  return launch_finalize_chol(bb, m, chol, color, weight, den, grad_xy, grad_chol, grad_color,
                              grad_weight, s);
}

}  // namespace

extern "C" {

int rtgs2d_abi_version(void) { return RTGS2D_ABI_VERSION; }

const char* rtgs2d_last_error(void) { return rtgs2d::g_last_error.c_str(); }

int rtgs2d_arena_create(rtgs2d_arena** out) {
  if (!out) return set_error(RTGS2D_ERR_INVALID, "out is NULL");
  *out = nullptr;
  int dev = 0;
  RTGS_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  rtgs2d_arena* a = new (std::nothrow) rtgs2d_arena();
  if (!a) return set_error(RTGS2D_ERR_ALLOC, "host allocation failed");
  a->device = dev;
  *out = a;
  return RTGS2D_OK;
}

int rtgs2d_arena_destroy(rtgs2d_arena* arena) {
  if (!arena) return RTGS2D_OK;
  const int dev = arena->device;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  delete arena;
  if (prev != dev) cudaSetDevice(prev);
  return RTGS2D_OK;
}

int rtgs2d_arena_last_stats(const rtgs2d_arena* arena, int64_t* entries, int64_t* pairs) {
  if (!arena) return set_error(RTGS2D_ERR_INVALID, "arena is NULL");
  if (entries) *entries = arena->bb.n_entries;
  if (pairs) *pairs = arena->bb.n_pairs;
  return RTGS2D_OK;
}

int rtgs2d_forward(rtgs2d_arena* arena, const float* xy, const float* conics, const float* colors,
                   const float* weights, const int32_t* rects, const int32_t* view_index,
                   int64_t m, int64_t n_views, int64_t height, int64_t width, double cutoff,
                   float* out, float* den, void* stream) {
  RTGS_TRY(check_arena(arena));
  arena->last_forward_valid = false;
  RTGS_TRY(check_dims(m, n_views, height, width));
  RTGS_TRY(require(out, "out"));
  if (m > 0) {
    RTGS_TRY(require(xy, "xy"));
    RTGS_TRY(require(conics, "conics"));
    RTGS_TRY(require(colors, "colors"));
    RTGS_TRY(require(weights, "weights"));
    RTGS_TRY(require(rects, "rects"));
    RTGS_TRY(require(view_index, "view_index"));
  }
  cudaStream_t s = as_stream(stream);
  const Geometry g = make_geometry(static_cast<int>(n_views), static_cast<int>(height),
                                   static_cast<int>(width));
  BinBuffers& bb = arena->bb;
  ArenaUse use(arena, s);
  RTGS_TRY(use.begin());
  RTGS_TRY(launch_project_conic(bb, g, xy, conics, colors, weights, rects, view_index, m,
                                den != nullptr, s));
  RTGS_TRY(bin_entries(bb, g, m, s));
  arena->n_tiles = g.n_tiles();
  return launch_raster_forward(bb, g, static_cast<float>(cutoff), out, den, s);
}

int rtgs2d_backward(rtgs2d_arena* arena, const float* grad_out, const float* grad_den,
                    const float* xy, const float* conics, const float* colors,
                    const float* weights, const int32_t* rects, const int32_t* view_index,
                    int64_t m, int64_t n_views, int64_t height, int64_t width, double cutoff,
                    float* grad_xy, float* grad_conics, float* grad_colors, float* grad_weights,
                    void* stream) {
  RTGS_TRY(check_arena(arena));
  arena->last_forward_valid = false;
  RTGS_TRY(check_dims(m, n_views, height, width));
  if (m == 0) return RTGS2D_OK;
  RTGS_TRY(require(xy, "xy"));
  RTGS_TRY(require(conics, "conics"));
  RTGS_TRY(require(colors, "colors"));
  RTGS_TRY(require(weights, "weights"));
  RTGS_TRY(require(rects, "rects"));
  RTGS_TRY(require(view_index, "view_index"));
  RTGS_TRY(require(grad_xy, "grad_xy"));
  RTGS_TRY(require(grad_conics, "grad_conics"));
  RTGS_TRY(require(grad_colors, "grad_colors"));
  RTGS_TRY(require(grad_weights, "grad_weights"));
  cudaStream_t s = as_stream(stream);
  const Geometry g = make_geometry(static_cast<int>(n_views), static_cast<int>(height),
                                   static_cast<int>(width));
  BinBuffers& bb = arena->bb;
  const bool den = grad_den != nullptr;
  ArenaUse use(arena, s);
  RTGS_TRY(use.begin());
  RTGS_TRY(launch_project_conic(bb, g, xy, conics, colors, weights, rects, view_index, m, den, s));
  RTGS_TRY(bin_entries(bb, g, m, s));
  arena->n_tiles = g.n_tiles();
  RTGS_TRY(launch_raster_backward(bb, g, static_cast<float>(cutoff), grad_out, grad_den, s));
  return launch_finalize_conic(bb, m, conics, colors, weights, den, grad_xy, grad_conics,
                               grad_colors, grad_weights, s);
}

int rtgs2d_render_forward(rtgs2d_arena* arena, const float* xy, const float* chol,
                          const float* color, const float* weight, int64_t n_views, int64_t n,
                          int64_t height, int64_t width, float* out, float* den, void* stream) {
  RTGS_TRY(check_arena(arena));
  if (n < 0) return set_error(RTGS2D_ERR_INVALID, "n must be non-negative");
  const int64_t m = n_views * n;
  RTGS_TRY(check_dims(m, n_views, height, width));
  RTGS_TRY(require(out, "out"));
  if (m > 0) {
    RTGS_TRY(require(xy, "xy"));
    RTGS_TRY(require(chol, "chol"));
    RTGS_TRY(require(color, "color"));
    RTGS_TRY(require(weight, "weight"));
  }
  cudaStream_t s = as_stream(stream);
  const Geometry g = make_geometry(static_cast<int>(n_views), static_cast<int>(height),
                                   static_cast<int>(width));
  BinBuffers& bb = arena->bb;
  arena->last_forward_valid = false;
  ArenaUse use(arena, s);
  RTGS_TRY(use.begin());
  RTGS_TRY(launch_project_chol(bb, g, xy, chol, color, weight, m, n > 0 ? n : 1, den != nullptr, s));
  RTGS_TRY(bin_entries(bb, g, m, s));
  arena->n_tiles = g.n_tiles();
  arena->last_forward = {xy, chol, color, weight, n_views, n, height, width, den != nullptr};
  arena->last_forward_valid = true;
  return launch_raster_forward(bb, g, kCutoff, out, den, s);
}

int rtgs2d_render_backward(rtgs2d_arena* arena, const float* grad_out, const float* grad_den,
                           const float* xy, const float* chol, const float* color,
                           const float* weight, int64_t n_views, int64_t n, int64_t height,
                           int64_t width, float* grad_xy, float* grad_chol, float* grad_color,
                           float* grad_weight, void* stream) {
  return render_backward(arena, grad_out, grad_den, xy, chol, color, weight, n_views, n, height,
                         width, grad_xy, grad_chol, grad_color, grad_weight, false, stream);
}

int rtgs2d_render_backward_after_forward(rtgs2d_arena* arena, const float* grad_out,
                                         const float* grad_den, const float* xy,
                                         const float* chol, const float* color,
                                         const float* weight, int64_t n_views, int64_t n,
                                         int64_t height, int64_t width, float* grad_xy,
                                         float* grad_chol, float* grad_color, float* grad_weight,
                                         void* stream) {
  return render_backward(arena, grad_out, grad_den, xy, chol, color, weight, n_views, n, height,
                         width, grad_xy, grad_chol, grad_color, grad_weight, true, stream);
}


int rtgs2d_support_rects(const float* xy, const float* chol, int64_t m, int64_t height,
                         int64_t width, int32_t* rects, int64_t* counts, void* stream) {
  RTGS_TRY(check_dims(m, 1, height, width));
  if (m == 0) return RTGS2D_OK;
  RTGS_TRY(require(xy, "xy"));
  RTGS_TRY(require(chol, "chol"));
  return launch_support_rects(xy, chol, m, static_cast<int>(height), static_cast<int>(width), rects,
                              counts, as_stream(stream));
}

int rtgs2d_arena_copy_binning(const rtgs2d_arena* arena, int64_t max_entries, uint32_t* gids,
                              int64_t max_tiles, int32_t* ranges, int64_t* n_entries,
                              int64_t* n_tiles, void* stream) {
  RTGS_TRY(check_arena(arena));
  const BinBuffers& bb = arena->bb;
  const int64_t ne = bb.n_entries < bb.capacity ? bb.n_entries : bb.capacity;
  const int64_t nt = arena->n_tiles;
  if (n_entries) *n_entries = ne;
  if (n_tiles) *n_tiles = nt;
  cudaStream_t s = as_stream(stream);
  ArenaUse use(const_cast<rtgs2d_arena*>(arena), s);
  RTGS_TRY(use.begin());
  // Per-tile ranges and the ids in read order (ascending inside each tile), on the host.
  std::vector<int32_t> rng(static_cast<size_t>(2 * nt), 0);
  std::vector<uint32_t> ids(static_cast<size_t>(ne), 0);
  if (bb.presorted) {
    std::vector<uint64_t> packed(static_cast<size_t>(ne));
    if (ne > 0) {
      RTGS_CUDA(cudaMemcpyAsync(packed.data(), bb.entries[bb.sorted_sel].ptr, ne * sizeof(uint64_t),
                                cudaMemcpyDeviceToHost, s), "copy entries");
    }
    if (nt > 0) {
      RTGS_CUDA(cudaMemcpyAsync(rng.data(), bb.ranges.ptr, nt * 2 * sizeof(int32_t),
                                cudaMemcpyDeviceToHost, s), "copy ranges");
    }
    RTGS_CUDA(cudaStreamSynchronize(s), "copy binning sync");
    for (int64_t i = 0; i < ne; ++i) ids[static_cast<size_t>(i)] = static_cast<uint32_t>(packed[static_cast<size_t>(i)]);
  } else {
    // List path: each tile's ids sit in list[ranges[t]) in ascending order (the tile sort).
    std::vector<uint32_t> list(static_cast<size_t>(ne), 0);
    if (ne > 0) {
      RTGS_CUDA(cudaMemcpyAsync(list.data(), bb.list.ptr, ne * sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
                "copy list");
    }
    std::vector<int32_t> r(static_cast<size_t>(2 * nt), 0);
    if (nt > 0) {
      RTGS_CUDA(cudaMemcpyAsync(r.data(), bb.ranges.ptr, nt * 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, s),
                "copy ranges");
    }
    RTGS_CUDA(cudaStreamSynchronize(s), "copy binning sync");
    int64_t at = 0;  // repack tile by tile, so ranges index the returned ids
    for (int64_t t = 0; t < nt; ++t) {
      int32_t a0 = r[static_cast<size_t>(2 * t)], a1 = r[static_cast<size_t>(2 * t + 1)];
      a0 = a0 < ne ? a0 : static_cast<int32_t>(ne);
      a1 = a1 < ne ? a1 : static_cast<int32_t>(ne);
      rng[static_cast<size_t>(2 * t)] = static_cast<int32_t>(at);
      for (int32_t k = a0; k < a1 && at < ne; ++k) ids[static_cast<size_t>(at++)] = list[static_cast<size_t>(k)];
      rng[static_cast<size_t>(2 * t + 1)] = static_cast<int32_t>(at);
    }
  }
  if (gids) {
    const int64_t c = ne < max_entries ? ne : max_entries;
    for (int64_t i = 0; i < c; ++i) gids[i] = ids[static_cast<size_t>(i)];
  }
  if (ranges) {
    const int64_t c = nt < max_tiles ? nt : max_tiles;
    for (int64_t i = 0; i < 2 * c; ++i) ranges[i] = rng[static_cast<size_t>(i)];
  }
  return RTGS2D_OK;
}

}  // extern "C"
