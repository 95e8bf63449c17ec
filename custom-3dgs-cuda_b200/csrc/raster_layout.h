// Byte layout of the gs_rasterize workspace. The first `zero_bytes` (counters, digit
// histograms and look-back status words) are cleared at the start of every call.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace gs {

struct RasterHeader {
  unsigned long long pair_acc;  // running total of (tile, Gaussian) pairs
  unsigned done_bin, ticket_dup;
  unsigned ticket_depth[4];
  unsigned ticket_tile[4];
  int n_visible;   // Gaussians with at least one tile
  int pair_count;  // M
};

struct RasterLayout {
  int tiles_x = 0, tiles_y = 0, tile_passes = 0;
  // digit of each tile-sort pass: 8 bits, the remainder of the tile-id bits in the last pass
  // (an even split, 7 + 6 at 1080p, measured slower: fewer histogram bins contend more)
  int tile_shift[4] = {0, 0, 0, 0};
  unsigned tile_mask[4] = {0u, 0u, 0u, 0u};
  long long T = 0, nb = 0, nd = 0, nt = 0;
  size_t header = 0, depth_hist = 0, tile_hist = 0, status_dup = 0,
         status_depth = 0, status_tile = 0, zero_bytes = 0;
  size_t rects = 0, records = 0, depth_keys[2] = {0, 0}, depth_vals[2] = {0, 0},
         tile_keys[2] = {0, 0}, tile_vals_tmp = 0, tile_order = 0;
  size_t total = 0;
};

RasterLayout make_raster_layout(int N, int W, int H, long long capacity);

// Enqueues binning, sorting and blending with `ws` laid out as `L` (defined in raster.cu).
int launch_rasterize(const RasterLayout& L, int N, int H, int W, const float* depths,
                     const float* mean2d, const float* cov2d, const float* colors,
                     const float* alpha, char* ws, long long capacity, float* img,
                     int* sorted_ids, int* tile_ranges, float* final_T, int* n_contrib,
                     int* pair_count_dev, int* pair_count_host, cudaEvent_t m_ready,
                     cudaStream_t stream);

}  // namespace gs
