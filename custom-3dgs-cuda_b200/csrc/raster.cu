// Host orchestration of binning, sorting and blending (gs_rasterize) and of the blend
// backward (gs_rasterize_backward), with the caller-provided workspace layout.
#include <algorithm>
#include <atomic>

#include "binning.cuh"
#include "blend.cuh"
#include "capi_internal.h"
#include "onesweep.cuh"
#include "raster_internal.h"

namespace gs {

// Blend records of every Gaussian for the backward of the stand-alone API, where the
// forward's records are not available (conic from the covariance as at forward load).
__global__ void __launch_bounds__(256) build_records_kernel(int N, const float* __restrict__ mean2d,
                                                           const float* __restrict__ cov2d,
                                                           const float* __restrict__ colors,
                                                           const float* __restrict__ alpha,
                                                           float4* __restrict__ records) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const float a = cov2d[3 * i], b = cov2d[3 * i + 1], c = cov2d[3 * i + 2];
  const float3 conic = conic_from_cov(a, b, c);
  const float op = alpha[i];
  const float2 ext = splat_extent(conic, op);
  records[3 * i + 0] = make_float4(mean2d[2 * i], mean2d[2 * i + 1], ext.x, ext.y);
  records[3 * i + 1] = make_float4(conic.x, conic.y, conic.z, op);
  records[3 * i + 2] = make_float4(colors[3 * i], colors[3 * i + 1], colors[3 * i + 2],
                                   __int_as_float(i));
}

static int tile_id_bits(long long T) {
  int bits = 0;
  while (bits < 32 && ((T - 1) >> bits) > 0) ++bits;
  return bits;
}

RasterLayout make_raster_layout(int N, int W, int H, long long capacity) {
  RasterLayout L;
  L.tiles_x = (W + kTileSide - 1) / kTileSide;
  L.tiles_y = (H + kTileSide - 1) / kTileSide;
  L.T = (long long)L.tiles_x * L.tiles_y;
  const int bits = tile_id_bits(L.T);
  L.tile_passes = (bits + 7) / 8;
  for (int p = 0, shift = 0; p < L.tile_passes; ++p) {
    const int w = std::min(8, bits - shift);  // 8-bit digits, the remainder last
    L.tile_shift[p] = shift;
    L.tile_mask[p] = (1u << w) - 1u;
    shift += w;
  }
  const long long nb = ((long long)N + kBinThreads - 1) / kBinThreads;
  const long long nd = ((long long)N + kSortTileItems - 1) / kSortTileItems;
  const long long nt = (capacity + kSortTileItems - 1) / kSortTileItems;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += (bytes + 255) / 256 * 256;
    return at;
  };
  // zero-initialised region
  L.header = take(sizeof(RasterHeader));
  L.depth_hist = take(4 * 256 * sizeof(unsigned));
  L.tile_hist = take(4 * 256 * sizeof(unsigned));
  L.status_dup = take(nb * sizeof(unsigned));
  L.status_depth = take(4 * nd * 256 * sizeof(unsigned));
  L.status_tile = take((size_t)std::max(L.tile_passes, 1) * nt * 256 * sizeof(unsigned));
  L.zero_bytes = off;
  // scratch arrays
  L.rects = take((size_t)N * sizeof(uint2));
  L.records = take((size_t)N * 3 * sizeof(float4));
  L.depth_keys[0] = take((size_t)N * sizeof(unsigned));
  L.depth_keys[1] = take((size_t)N * sizeof(unsigned));
  L.depth_vals[0] = take((size_t)N * sizeof(unsigned));
  L.depth_vals[1] = take((size_t)N * sizeof(unsigned));
  L.tile_keys[0] = take((size_t)capacity * sizeof(unsigned));
  L.tile_keys[1] = take((size_t)capacity * sizeof(unsigned));
  L.tile_vals_tmp = take((size_t)capacity * sizeof(unsigned));
  L.tile_order = take((size_t)L.T * sizeof(int));
  L.total = off;
  L.nb = nb;
  L.nd = nd;
  L.nt = nt;
  return L;
}

// SM count of the current device, looked up once per device ordinal (devices of different
// models in one process each get their own figure; a racing first lookup stores the same value).
static int sm_count() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> counts[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  int count = counts[dev].load(std::memory_order_relaxed);
  if (count == 0) {
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
    counts[dev].store(count, std::memory_order_relaxed);
  }
  return count;
}

void fill_bin_params(BinParams& bp, const RasterLayout& L, char* ws, int N, int H, int W,
                     const float* depths, const float* mean2d, const float* cov2d,
                     const float* colors, const float* alpha, long long capacity) {
  RasterHeader* hdr = reinterpret_cast<RasterHeader*>(ws + L.header);
  bp.N = N;
  bp.W = W;
  bp.H = H;
  bp.tiles_x = L.tiles_x;
  bp.tiles_y = L.tiles_y;
  bp.depths = depths;
  bp.mean2d = mean2d;
  bp.cov2d = cov2d;
  bp.colors = colors;
  bp.alpha = alpha;
  bp.rects = reinterpret_cast<uint2*>(ws + L.rects);
  bp.records = reinterpret_cast<float4*>(ws + L.records);
  bp.depth_keys = reinterpret_cast<unsigned*>(ws + L.depth_keys[0]);
  bp.depth_vals = reinterpret_cast<unsigned*>(ws + L.depth_vals[0]);
  bp.done_counter = &hdr->done_bin;
  bp.depth_hist = reinterpret_cast<unsigned*>(ws + L.depth_hist);
  bp.pair_acc = &hdr->pair_acc;
  bp.n_visible = &hdr->n_visible;
  bp.pair_count = &hdr->pair_count;
  bp.pair_capacity = capacity;
  bp.tight = 0;
}

int launch_sort_and_blend(const RasterLayout& L, int N, int H, int W, char* ws,
                          long long capacity, float* img, int* sorted_ids, int* tile_ranges,
                          float* final_T, int* n_contrib, bool throughput,
                          cudaStream_t stream) {
  RasterHeader* hdr = reinterpret_cast<RasterHeader*>(ws + L.header);
  float4* records = reinterpret_cast<float4*>(ws + L.records);
  unsigned* dk[2] = {reinterpret_cast<unsigned*>(ws + L.depth_keys[0]),
                     reinterpret_cast<unsigned*>(ws + L.depth_keys[1])};
  unsigned* dv[2] = {reinterpret_cast<unsigned*>(ws + L.depth_vals[0]),
                     reinterpret_cast<unsigned*>(ws + L.depth_vals[1])};
  const int P = L.tile_passes;
  unsigned* tk[2] = {reinterpret_cast<unsigned*>(ws + L.tile_keys[0]),
                     reinterpret_cast<unsigned*>(ws + L.tile_keys[1])};
  unsigned* tv[2];
  tv[P % 2] = reinterpret_cast<unsigned*>(sorted_ids);
  tv[(P + 1) % 2] = reinterpret_cast<unsigned*>(ws + L.tile_vals_tmp);

  if (N > 0) {
    // depth sort of the visible Gaussians: 4 passes, result back in buffer 0
    for (int pass = 0; pass < 4; ++pass) {
      SortPass sp;
      sp.keys_in = dk[pass & 1];
      sp.vals_in = dv[pass & 1];
      sp.keys_out = pass < 3 ? dk[(pass + 1) & 1] : nullptr;  // the duplication reads ids only
      sp.vals_out = dv[(pass + 1) & 1];
      sp.n_items = &hdr->n_visible;
      sp.overflow_count = &hdr->pair_count;
      sp.overflow_limit = capacity;
      sp.digit_hist = reinterpret_cast<unsigned*>(ws + L.depth_hist) + pass * 256;
      sp.status = reinterpret_cast<unsigned*>(ws + L.status_depth) + (size_t)pass * L.nd * 256;
      sp.ticket = &hdr->ticket_depth[pass];
      sp.shift = 8 * pass;
      sp.mask = 255u;
      onesweep_pass_kernel<<<(unsigned)L.nd, kSortThreads, 0, stream>>>(sp);
      GS_CHECK_LAUNCH();
    }
    mark_stage(2, stream);
    DupParams dp;
    dp.tiles_x = L.tiles_x;
    dp.n_tile_passes = P;
    for (int k = 0; k < 4; ++k) {
      dp.tile_shift[k] = L.tile_shift[k];
      dp.tile_mask[k] = L.tile_mask[k];
    }
    dp.n_visible = &hdr->n_visible;
    dp.pair_count = &hdr->pair_count;
    dp.pair_capacity = capacity;
    dp.sorted_gids = dv[0];
    dp.rects = reinterpret_cast<uint2*>(ws + L.rects);
    dp.status = reinterpret_cast<unsigned*>(ws + L.status_dup);
    dp.ticket = &hdr->ticket_dup;
    dp.tile_keys = tk[0];
    dp.tile_vals = tv[0];
    dp.tile_hist = reinterpret_cast<unsigned*>(ws + L.tile_hist);
    dp.runs = dup_runs(N, sm_count());
    const long long dup_items = (long long)kBinThreads * dp.runs;
    const unsigned dup_blocks = (unsigned)(((long long)N + dup_items - 1) / dup_items);
    scan_duplicate_kernel<<<dup_blocks, kBinThreads, 0, stream>>>(dp);
    GS_CHECK_LAUNCH();
    mark_stage(3, stream);
    for (int pass = 0; pass < P; ++pass) {
      SortPass sp;
      sp.keys_in = tk[pass & 1];
      sp.vals_in = tv[pass & 1];
      sp.keys_out = tk[(pass + 1) & 1];
      sp.vals_out = tv[(pass + 1) & 1];
      sp.n_items = &hdr->pair_count;
      sp.overflow_count = &hdr->pair_count;
      sp.overflow_limit = capacity;
      sp.digit_hist = reinterpret_cast<unsigned*>(ws + L.tile_hist) + pass * 256;
      sp.status = reinterpret_cast<unsigned*>(ws + L.status_tile) + (size_t)pass * L.nt * 256;
      sp.ticket = &hdr->ticket_tile[pass];
      sp.shift = L.tile_shift[pass];
      sp.mask = L.tile_mask[pass];
      const bool last = pass == P - 1;
      sp.ranges = last ? reinterpret_cast<int2*>(tile_ranges) : nullptr;
      sp.num_tiles = (unsigned)L.T;
      if (last) sp.keys_out = nullptr;  // the ranges are written in this pass
      if (L.nt > 0) {
        onesweep_pass_kernel<<<(unsigned)L.nt, kSortThreads, 0, stream>>>(sp);
        GS_CHECK_LAUNCH();
      }
    }
    mark_stage(4, stream);
  }
  int* tile_order = reinterpret_cast<int*>(ws + L.tile_order);
  tile_order_kernel<<<1, kOrderThreads, 0, stream>>>(reinterpret_cast<int2*>(tile_ranges),
                                                      &hdr->pair_count, capacity, (int)L.T,
                                                      tile_order);
  GS_CHECK_LAUNCH();
  mark_stage(5, stream);
  BlendFwdParams fp;
  fp.W = W;
  fp.H = H;
  fp.tiles_x = L.tiles_x;
  fp.num_tiles = (int)L.T;
  fp.ranges = reinterpret_cast<const int2*>(tile_ranges);
  fp.tile_order = tile_order;
  fp.sorted_ids = sorted_ids;
  fp.records = records;
  fp.pair_count = &hdr->pair_count;
  fp.pair_capacity = capacity;
  fp.img = img;
  fp.final_T = final_T;
  fp.n_contrib = n_contrib;
  if (throughput) {
    blend_forward_kernel<kBlendFwdPixThroughput>
        <<<(unsigned)L.T, kTilePixels / kBlendFwdPixThroughput, 0, stream>>>(fp);
  } else {
    blend_forward_kernel<kBlendFwdPix>
        <<<(unsigned)L.T, kTilePixels / kBlendFwdPix, 0, stream>>>(fp);
  }
  GS_CHECK_LAUNCH();
  mark_stage(6, stream);
  return GS_OK;
}

int launch_rasterize(const RasterLayout& L, int N, int H, int W, const float* depths,
                     const float* mean2d, const float* cov2d, const float* colors,
                     const float* alpha, char* ws, long long capacity, float* img,
                     int* sorted_ids, int* tile_ranges, float* final_T, int* n_contrib,
                     int* pair_count_dev, int* pair_count_host, cudaEvent_t m_ready,
                     cudaStream_t stream) {
  RasterHeader* hdr = reinterpret_cast<RasterHeader*>(ws + L.header);
  GS_CUDA(cudaMemsetAsync(ws, 0, L.zero_bytes, stream));
  GS_CUDA(cudaMemsetAsync(tile_ranges, 0x7f, (size_t)L.T * 2 * sizeof(int), stream));  // kRangeUnset
  if (N > 0) {
    BinParams bp;
    fill_bin_params(bp, L, ws, N, H, W, depths, mean2d, cov2d, colors, alpha, capacity);
    bin_prepare_kernel<<<(unsigned)L.nb, kBinThreads, 0, stream>>>(bp);
    GS_CHECK_LAUNCH();
  }
  if (pair_count_dev)
    GS_CUDA(cudaMemcpyAsync(pair_count_dev, &hdr->pair_count, sizeof(int),
                            cudaMemcpyDeviceToDevice, stream));
  if (pair_count_host)
    GS_CUDA(cudaMemcpyAsync(pair_count_host, &hdr->pair_count, sizeof(int),
                            cudaMemcpyDeviceToHost, stream));
  if (m_ready) GS_CUDA(cudaEventRecord(m_ready, stream));
  return launch_sort_and_blend(L, N, H, W, ws, capacity, img, sorted_ids, tile_ranges, final_T,
                               n_contrib, false, stream);
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_rasterize_workspace_size(int N, int H, int W, long long pair_capacity) {
  if (N < 0 || H <= 0 || W <= 0 || pair_capacity < 0) return 0;
  return make_raster_layout(N, W, H, pair_capacity).total;
}

extern "C" int gs_rasterize(int N, int H, int W, const float* depths, const float* mean2d,
                            const float* cov2d, const float* colors, const float* alpha,
                            void* workspace, size_t workspace_bytes, long long pair_capacity,
                            float* img, int* sorted_ids, int* tile_ranges, float* final_T,
                            int* n_contrib, int* pair_count_dev, int* pair_count_host,
                            void* m_ready_event, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  GS_REQUIRE((W + 15) / 16 < 65536 && (H + 15) / 16 < 65536, "image too large");
  GS_REQUIRE(pair_capacity >= 0 && pair_capacity < (1ll << 30),
             "pair capacity must be in [0, 2^30)");
  GS_REQUIRE(img && tile_ranges && final_T && n_contrib && workspace, "null pointer");
  GS_REQUIRE(N == 0 || (depths && mean2d && cov2d && colors && alpha), "null input pointer");
  GS_REQUIRE(pair_capacity == 0 || sorted_ids, "null sorted_ids with a non-zero capacity");
  const RasterLayout L = make_raster_layout(N, W, H, pair_capacity);
  GS_REQUIRE(workspace_bytes >= L.total, "workspace too small");
  GS_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0u,
             "workspace must be 256-byte aligned");
  return launch_rasterize(L, N, H, W, depths, mean2d, cov2d, colors, alpha,
                          static_cast<char*>(workspace), pair_capacity, img, sorted_ids,
                          tile_ranges, final_T, n_contrib, pair_count_dev, pair_count_host,
                          (cudaEvent_t)m_ready_event, (cudaStream_t)stream);
  GS_API_END();
}

extern "C" size_t gs_rasterize_backward_workspace_size(int N) {
  if (N < 0) return 0;
  return (size_t)N * 3 * sizeof(float4) + 256;
}

extern "C" int gs_rasterize_backward(int N, int H, int W, const float* grad_img,
                                     const float* mean2d, const float* cov2d,
                                     const float* colors, const float* alpha,
                                     const int* sorted_ids, const int* tile_ranges,
                                     const float* final_T, const int* n_contrib,
                                     void* workspace, size_t workspace_bytes, float* g_mean2d,
                                     float* g_cov2d, float* g_colors, float* g_alpha,
                                     void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  if (N == 0) return GS_OK;
  GS_REQUIRE(grad_img && mean2d && cov2d && colors && alpha && tile_ranges && final_T &&
                 n_contrib && workspace && g_mean2d && g_cov2d && g_colors && g_alpha,
             "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_rasterize_backward_workspace_size(N), "workspace too small");
  float4* records = reinterpret_cast<float4*>(
      (reinterpret_cast<uintptr_t>(workspace) + 255u) & ~uintptr_t(255u));
  cudaStream_t st = (cudaStream_t)stream;
  build_records_kernel<<<(N + 255) / 256, 256, 0, st>>>(N, mean2d, cov2d, colors, alpha,
                                                         records);
  GS_CHECK_LAUNCH();
  const int tiles_x = (W + kTileSide - 1) / kTileSide;
  const int tiles_y = (H + kTileSide - 1) / kTileSide;
  BlendBwdParams bp;
  bp.N = N;
  bp.W = W;
  bp.H = H;
  bp.tiles_x = tiles_x;
  bp.num_tiles = tiles_x * tiles_y;
  bp.pair_count = nullptr;  // the caller's tile ranges are valid
  bp.pair_capacity = 0;
  bp.grad_img = grad_img;
  bp.ranges = reinterpret_cast<const int2*>(tile_ranges);
  bp.tile_order = nullptr;  // raster order: this entry point has no forward workspace
  bp.sorted_ids = sorted_ids;
  bp.records = records;
  bp.final_T = final_T;
  bp.n_contrib = n_contrib;
  bp.g_mean2d = g_mean2d;
  bp.g_cov2d = g_cov2d;
  bp.g_colors = g_colors;
  bp.g_alpha = g_alpha;
  bp.g_accum = nullptr;
  blend_backward_kernel<false, kBlendBwdPix>
      <<<(unsigned)(tiles_x * tiles_y), kTilePixels / kBlendBwdPix, 0, st>>>(bp);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
