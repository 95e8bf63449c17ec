// gs_rasterize_noalloc: the tile binning + sort + blend of gs_rasterize for callers that
// cannot allocate device memory at the time they render.
//
// Who needs it: code that runs inside a memory budget it does not own — an engine plugin
// handed only input and output buffers by its host application, a process whose CUDA memory
// is reserved up front by another allocator (so a cudaMalloc would fail or fragment that
// pool), or a render path that must not call into an allocator on every frame because
// cudaMalloc/cudaFree synchronise the device. Such callers still own their inputs and outputs;
// what they cannot do is provide the binning/sort scratch that gs_rasterize takes as a
// workspace. This entry point uses a fixed scratch array compiled into the library instead.
//
// The array is file-scope device memory of kNoAllocScratchBytes (16 MiB); every GPU on which
// the library is loaded holds it until the process exits. A call whose workspace layout for
// (N, H, W, pair_capacity) does not fit is rejected with GS_ERR_CAPACITY before any GPU work;
// for example 65,536 Gaussians at 1024 x 1024 with up to 600,000 (tile, Gaussian) pairs fit.
//
// Host code cannot use the array's name as a device address, so the first call on each device
// (with that device current) looks the address up with cudaGetSymbolAddress and caches it;
// that first call should therefore be made before any stream capture begins. All calls share
// the one array and it keeps the previous call's contents: the call clears the counters,
// histograms and look-back words it relies on at the start (an asynchronous memset, not an
// allocation). Calls whose GPU work overlaps — on different streams, or from different host
// threads — race on the array and must be serialised by the caller.
//
// The pair count M is always written to *pair_count_dev (required here, unlike gs_rasterize,
// because this entry point has no host-side path to report it). When M exceeds
// pair_capacity the sort, range and blend kernels skip their work, so img, final_T,
// n_contrib, tile_ranges and sorted_ids are NOT written by that call; the caller must read M
// and call again with pair_capacity >= M. The cached array address belongs to the device's
// primary context: after cudaDeviceReset in the same process, do not call this entry point
// again (the cached address would be stale).
#include <mutex>

#include "capi_internal.h"
#include "raster_layout.h"

namespace gs {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_addr[kNoAllocMaxDevices] = {};

}  // namespace gs

using namespace gs;

extern "C" int gs_rasterize_noalloc(int N, int H, int W, const float* depths,
                                    const float* mean2d, const float* cov2d,
                                    const float* colors, const float* alpha,
                                    long long pair_capacity, float* img, int* sorted_ids,
                                    int* tile_ranges, float* final_T, int* n_contrib,
                                    int* pair_count_dev, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  GS_REQUIRE((W + 15) / 16 < 65536 && (H + 15) / 16 < 65536, "image too large");
  GS_REQUIRE(pair_capacity >= 0 && pair_capacity < (1ll << 30),
             "pair capacity must be in [0, 2^30)");
  GS_REQUIRE(img && tile_ranges && final_T && n_contrib, "null output pointer");
  GS_REQUIRE(N == 0 || (depths && mean2d && cov2d && colors && alpha), "null input pointer");
  GS_REQUIRE(pair_capacity == 0 || sorted_ids, "null sorted_ids with a non-zero capacity");
  GS_REQUIRE(pair_count_dev, "pair_count_dev is required: it reports M, and M > pair_capacity "
             "leaves the outputs unwritten");
  const RasterLayout L = make_raster_layout(N, W, H, pair_capacity);
  if (L.total > kNoAllocScratchBytes)
    return set_error(GS_ERR_CAPACITY,
                     "gs_rasterize_noalloc: this call needs " + std::to_string(L.total) +
                         " bytes of scratch but the fixed scratch holds " +
                         std::to_string(kNoAllocScratchBytes) +
                         " bytes; reduce N, the image size or pair_capacity, or use "
                         "gs_rasterize with a caller-provided workspace");
  int dev = 0;
  GS_CUDA(cudaGetDevice(&dev));
  GS_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "device ordinal out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
      void* addr = nullptr;
      GS_CUDA(cudaGetSymbolAddress(&addr, g_noalloc_scratch));
      g_noalloc_addr[dev] = addr;
    }
    scratch = g_noalloc_addr[dev];
  }
  return launch_rasterize(L, N, H, W, depths, mean2d, cov2d, colors, alpha,
                          static_cast<char*>(scratch), pair_capacity, img, sorted_ids,
                          tile_ranges, final_T, n_contrib, pair_count_dev, nullptr, nullptr,
                          (cudaStream_t)stream);
  GS_API_END();
}
