// Launch helpers shared by the rasterize and render entry points (raster.cu, render.cu).
#pragma once

#include "binning.cuh"
#include "raster_layout.h"

namespace gs {

// Points the binning parameters at the workspace buffers of layout L.
void fill_bin_params(BinParams& bp, const RasterLayout& L, char* ws, int N, int H, int W,
                     const float* depths, const float* mean2d, const float* cov2d,
                     const float* colors, const float* alpha, long long capacity);

// Enqueues everything after binning prep: depth sort, pair duplication, tile sort, tile
// ranges and the forward blend (the throughput variant when `throughput`, see blend.cuh).
int launch_sort_and_blend(const RasterLayout& L, int N, int H, int W, char* ws,
                          long long capacity, float* img, int* sorted_ids, int* tile_ranges,
                          float* final_T, int* n_contrib, bool throughput,
                          cudaStream_t stream);

}  // namespace gs
