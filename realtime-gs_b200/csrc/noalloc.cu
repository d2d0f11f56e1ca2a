// rtgs2d_forward_noalloc: the reference-ABI forward render for callers that must not allocate.
//
// Some callers cannot call cudaMalloc: a plugin whose host application owns every byte of device
// memory and forbids the plugin from allocating behind its back, a latency-critical loop in which
// cudaMalloc / cudaFree would implicitly synchronise the device and stall its other streams, or a
// process whose free device memory is already fully reserved by another allocator. For them this
// entry point takes all of its scratch (gaussian records, tile spans, per-gaussian tile counts and
// offsets, tile entries and their sort buffers, per-tile ranges, radix-sort and scan temporaries)
// from one file-scope static device array of kScratchBytes per device, loaded with the library.
// The caller still passes inputs and outputs; the host side allocates nothing either (the entry
// count is read back into static host memory).
//
// Behaviour is that of rtgs2d_forward (same kernels, same results); the differences are:
//   - problems whose scratch does not fit kScratchBytes are rejected with RTGS2D_ERR_CAPACITY
//     and a message giving the bytes needed, before the entries that do not fit are written;
//   - all calls on one device share the one array and it keeps the last call's contents, so calls
//     whose GPU work overlaps (two host threads, or two streams without ordering between them)
//     race and corrupt each other; calls ordered on one stream are safe;
//   - the first call on each device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current. With lazy module loading (the CUDA 12 default) that lookup is
//     also what commits the array's 32 MiB on the device, so the first call can fail with
//     RTGS2D_ERR_CUDA (out of memory) when another allocator already holds the device's memory:
//     make the first call on each device at start-up, before other allocators reserve memory and
//     before any stream capture;
//   - the device statistics are read back into a static host row per device, so calls on
//     different devices (from different host threads) share nothing.
#include <cub/device/device_scan.cuh>

#include <mutex>
#include <string>

#include "../../include/rtgs2d.h"
#include "internal.h"

namespace {

constexpr size_t kScratchBytes = size_t{32} << 20;  // 32 MiB per device
constexpr int kMaxDevices = 64;

// The scratch itself. In host code `g_scratch` is only a host-side stand-in for the symbol, never
// a device address: the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
// Readback of the device statistics (entry count, long-tile flag), one row per device like the
// scratch itself: calls on different devices never share it. Pageable static memory, so the host
// side allocates nothing either.
unsigned long long g_host_stats[kMaxDevices][rtgs2d::kStatSlots];

// Device address of this device's scratch and its host readback row (with the device current).
int scratch_base(unsigned char** out, unsigned long long** host_stats) {
  int dev = -1;
  RTGS_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    return rtgs2d::set_error(RTGS2D_ERR_INVALID, "device index out of range for the static scratch table");
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    RTGS_CUDA(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress(static scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  *host_stats = g_host_stats[dev];
  return 0;
}

size_t align256(size_t v) { return (v + 255) & ~size_t{255}; }

// Bins whose buffers are views into the static array: every view is sized to what the launchers
// ask for, so DevBuf::ensure never reallocates, and the views are detached before the BinBuffers
// destructor runs, so nothing is ever freed.
struct BorrowedBins {
  rtgs2d::BinBuffers bb;
  ~BorrowedBins() {
    for (rtgs2d::DevBuf* b : {&bb.records, &bb.weights, &bb.spans, &bb.counts, &bb.offsets,
                              &bb.list, &bb.tile_count, &bb.tile_end,
                              &bb.entries[0], &bb.entries[1], &bb.ranges, &bb.partials,
                              &bb.partial_d, &bb.cub_temp, &bb.sort_counts, &bb.stats}) {
      b->ptr = nullptr;
      b->bytes = 0;
    }
    bb.host_stats = nullptr;
  }
};

struct Carver {
  unsigned char* base;
  size_t used = 0;
  bool take(rtgs2d::DevBuf& buf, size_t bytes) {
    bytes = bytes ? bytes : 1;
    const size_t at = align256(used);
    if (at + bytes > kScratchBytes) return false;
    buf.ptr = base + at;
    buf.bytes = bytes;
    used = at + bytes;
    return true;
  }
};

int too_big(size_t need_hint) {
  return rtgs2d::set_error(RTGS2D_ERR_CAPACITY,
                           "rtgs2d_forward_noalloc: problem needs more than the " +
                               std::to_string(kScratchBytes >> 20) +
                               " MiB static scratch (at least " + std::to_string(need_hint) +
                               " bytes); use rtgs2d_forward with an arena");
}

}  // namespace

extern "C" int rtgs2d_forward_noalloc(const float* xy, const float* conics, const float* colors,
                                      const float* weights, const int32_t* rects,
                                      const int32_t* view_index, int64_t m, int64_t n_views,
                                      int64_t height, int64_t width, double cutoff, float* out,
                                      float* den, void* stream) {
  using namespace rtgs2d;
  if (m < 0 || n_views <= 0 || height <= 0 || width <= 0) {
    return set_error(RTGS2D_ERR_INVALID, "m >= 0 and positive n_views, height, width are required");
  }
  if (height > 32768 || width > 32768 || m > INT32_MAX) {
    return set_error(RTGS2D_ERR_CAPACITY, "height/width at most 32768 and m below 2^31");
  }
  if (!out) return set_error(RTGS2D_ERR_INVALID, "out is NULL");
  if (m > 0 && (!xy || !conics || !colors || !weights || !rects || !view_index)) {
    return set_error(RTGS2D_ERR_INVALID, "an input pointer is NULL");
  }
  const Geometry g = make_geometry(static_cast<int>(n_views), static_cast<int>(height),
                                   static_cast<int>(width));
  if (g.n_tiles() > INT32_MAX) return set_error(RTGS2D_ERR_CAPACITY, "too many tiles");
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  unsigned char* base = nullptr;
  unsigned long long* host_stats = nullptr;
  RTGS_TRY(scratch_base(&base, &host_stats));
  BorrowedBins holder;
  BinBuffers& bb = holder.bb;
  bb.host_stats = host_stats;

  // Per-gaussian and per-tile buffers (the sizes the projection and binning launchers request).
  const size_t mm = static_cast<size_t>(m > 0 ? m : 1);
  const size_t tiles = static_cast<size_t>(g.n_tiles() > 0 ? g.n_tiles() : 1);
  size_t scan_bytes = 0, tile_scan_bytes = 0;
  RTGS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int*>(nullptr),
                                          static_cast<int*>(nullptr), static_cast<int>(m), s),
            "scan size query");
  RTGS_CUDA(cub::DeviceScan::InclusiveSum(nullptr, tile_scan_bytes, static_cast<int*>(nullptr),
                                          static_cast<int*>(nullptr),
                                          static_cast<int>(g.n_tiles()), s),
            "tile scan size query");
  if (tile_scan_bytes > scan_bytes) scan_bytes = tile_scan_bytes;
  Carver c{base};
  const size_t need_m = mm * (sizeof(GaussRecord) + sizeof(TileSpan) + 3 * sizeof(int)) +
                        tiles * (sizeof(int2) + 2 * sizeof(int)) + scan_bytes + sort_counts_bytes();
  if (!c.take(bb.records, mm * sizeof(GaussRecord)) || !c.take(bb.spans, mm * sizeof(TileSpan)) ||
      !c.take(bb.counts, mm * sizeof(int)) || !c.take(bb.offsets, mm * sizeof(int)) ||
      !c.take(bb.stats, kStatSlots * sizeof(unsigned long long)) ||
      !c.take(bb.ranges, tiles * sizeof(int2)) || !c.take(bb.cub_temp, scan_bytes) ||
      !c.take(bb.tile_count, tiles * sizeof(int)) || !c.take(bb.tile_end, tiles * sizeof(int)) ||
      !c.take(bb.sort_counts, sort_counts_bytes()) ||
      (den != nullptr && !c.take(bb.weights, mm * sizeof(float)))) {
    return too_big(need_m);
  }

  RTGS_TRY(launch_project_conic(bb, g, xy, conics, colors, weights, rects, view_index, m,
                                den != nullptr, s));
  // Entry count and long-tile flag (one check, one readback, one synchronisation), to size the
  // entry buffers before the binning writes any entry.
  const int rc = read_bin_stats(bb, g, m, s);
  if (rc == RTGS2D_ERR_CAPACITY) return too_big(static_cast<size_t>(bb.host_stats[kStatEntries]) * 16);
  RTGS_TRY(rc);
  const size_t e = static_cast<size_t>(bb.n_entries > 0 ? bb.n_entries : 1);
  // Both binnings need the entries; the tile scatter also the id list, the radix fallback (a
  // tile list longer than the tile sort) the entry double buffer.
  const bool radix = bb.long_tile;
  const bool fits = c.take(bb.entries[0], e * sizeof(uint64_t)) &&
                    (radix ? c.take(bb.entries[1], e * sizeof(uint64_t))
                           : c.take(bb.list, e * sizeof(uint32_t)));
  if (!fits) return too_big(c.used + (radix ? 16 : 12) * e);
  bb.capacity = static_cast<int64_t>(e);  // so bin_known grows no buffer
  RTGS_TRY(bin_known(bb, g, m, s));
  return launch_raster_forward(bb, g, static_cast<float>(cutoff), out, den, s);
}
