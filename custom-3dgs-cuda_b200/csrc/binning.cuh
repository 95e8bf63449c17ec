// Tile binning: per-Gaussian tile rectangles, order-preserving compaction of the visible
// Gaussians into depth-sort input, the pair-count total, the depth-ordered pair
// duplication and the tile ranges.
//
// Sort strategy. The reference sorts 64-bit keys (tile << 32 | depth bits) with a stable
// radix sort over all 64 bits (csrc/forward/rasterize.cu:416-435). An LSD radix sort
// processes the 32 depth bits before the tile bits, and pair duplication copies a
// Gaussian's depth bits unchanged into each of its pairs without reordering Gaussians, so
// the four depth passes can run on the visible Gaussians (N_v items) before duplication
// instead of on the M pairs after it. Only ceil(log2(T) / 8) passes over the M pairs
// remain. Ties (equal tile and bit-identical depth) keep Gaussian-index order in both
// schemes, so the sorted order is identical to the reference's.
#pragma once

#include "gs_common.cuh"

namespace gs {

constexpr int kBinThreads = 256;

// Packed tile rectangle: x = x0 | x1 << 16, y = y0 | y1 << 16.
__device__ __forceinline__ uint2 pack_rect(const TileRect& r) {
  return make_uint2((unsigned)r.x0 | ((unsigned)r.x1 << 16),
                    (unsigned)r.y0 | ((unsigned)r.y1 << 16));
}

__device__ __forceinline__ TileRect unpack_rect(uint2 p) {
  TileRect r;
  r.x0 = (int)(p.x & 0xffffu);
  r.x1 = (int)(p.x >> 16);
  r.y0 = (int)(p.y & 0xffffu);
  r.y1 = (int)(p.y >> 16);
  return r;
}

// Per-Gaussian blend record, 3 x float4:
//   [0] = (mean.x, mean.y, extent.x, extent.y)   (extent: splat_extent)
//   [1] = (conic.x, conic.y, conic.z, opacity)
//   [2] = (r, g, b, gaussian index as bits)
struct BinParams {
  int N, W, H, tiles_x, tiles_y;
  const float* depths;
  const float* mean2d;
  const float* cov2d;
  const float* colors;
  const float* alpha;
  uint2* rects;
  float4* records;
  unsigned* depth_keys;
  unsigned* depth_vals;
  unsigned* done_counter;
  unsigned* depth_hist;         // [4][256]
  unsigned long long* pair_acc; // running pair total
  int* n_visible;
  int* pair_count;              // M, clamped to INT_MAX
  long long pair_capacity;
  int tight;                    // 1: intersect each rectangle with the opacity-test extent
};

// Per-Gaussian part of binning: tile rectangle and count of a projected splat; for a splat
// covering at least one tile it also writes the packed rectangle and the blend record and
// returns the depth key. Shared by bin_prepare_kernel and the fused render preprocess. With
// p.tight the reference's rectangle is intersected with the tiles that hold a pixel of the
// splat's opacity-test extent box: the image, transmittance and gradients are unchanged (the
// dropped pairs fail the opacity test at every pixel of their tile), the tile lists shorter.
__device__ __forceinline__ unsigned bin_gaussian(const BinParams& p, int i, float2 mean,
                                                 float a, float b, float c, float depth,
                                                 float3 color, float opacity,
                                                 unsigned& depth_bits) {
  TileRect r;
  unsigned count = 0;
  depth_bits = 0;
  if (splat_tile_rect(mean, a, b, c, p.W, p.H, p.tiles_x, p.tiles_y, r)) {
    count = (unsigned)rect_count(r);
    float3 conic;
    float2 ext;
    if (count > 0) {
      conic = conic_from_cov(a, b, c);
      ext = splat_extent(conic, opacity);
      if (p.tight) {
        // keep only the tiles that hold a pixel inside the extent box: every other pair of the
        // reference's rectangle fails the opacity test at all of its tile's pixels
        if (ext.x == -INFINITY) {
          count = 0;
        } else if (ext.x != INFINITY) {
          const float lo_x = fmaxf(mean.x - ext.x, 0.0f);
          const float hi_x = fminf(mean.x + ext.x, (float)(p.W - 1));
          const float lo_y = fmaxf(mean.y - ext.y, 0.0f);
          const float hi_y = fminf(mean.y + ext.y, (float)(p.H - 1));
          if (hi_x < lo_x || hi_y < lo_y) {
            count = 0;
          } else {
            r.x0 = max(r.x0, (int)ceilf(lo_x) / kTileSide);
            r.x1 = min(r.x1, (int)floorf(hi_x) / kTileSide + 1);
            r.y0 = max(r.y0, (int)ceilf(lo_y) / kTileSide);
            r.y1 = min(r.y1, (int)floorf(hi_y) / kTileSide + 1);
            count = (unsigned)rect_count(r);
          }
        }
      }
    }
    if (count > 0) {
      p.rects[i] = pack_rect(r);
      p.records[3 * i + 0] = make_float4(mean.x, mean.y, ext.x, ext.y);
      p.records[3 * i + 1] = make_float4(conic.x, conic.y, conic.z, opacity);
      p.records[3 * i + 2] = make_float4(color.x, color.y, color.z, __int_as_float(i));
      depth_bits = __float_as_uint(depth);
    }
  }
  return count;
}

// Block part of binning, called by all kBinThreads threads of a CTA that holds Gaussians
// [tile * kBinThreads, ...): the depth-sort input for every Gaussian (key = depth bits, or
// 0xffffffff for a splat that covers no tile; value = index), the digit histograms of the four
// depth passes, the running pair total and, in the last CTA to finish, M. Sorting all N keeps
// the order the reference's stable 64-bit sort gives: splats without pairs are skipped by the
// duplication, and ties on the key keep index order whatever their value.
__device__ __forceinline__ void bin_block(const BinParams& p, int tile, int i, unsigned count,
                                          unsigned depth_bits, unsigned* s_scan,
                                          unsigned (*s_hist)[256], bool& s_last) {
  const int tid = threadIdx.x;
  if (i < p.N) {
    const unsigned key = count > 0 ? depth_bits : 0xffffffffu;
    if (count == 0) p.rects[i] = make_uint2(0u, 0u);
    p.depth_keys[i] = key;
    p.depth_vals[i] = (unsigned)i;
    atomicAdd(&s_hist[0][key & 255u], 1u);
    atomicAdd(&s_hist[1][(key >> 8) & 255u], 1u);
    atomicAdd(&s_hist[2][(key >> 16) & 255u], 1u);
    atomicAdd(&s_hist[3][key >> 24], 1u);
  }
  unsigned tile_pairs;
  block_exclusive_scan(count, s_scan, &tile_pairs);  // also orders the histogram updates
  for (int k = tid; k < 4 * 256; k += kBinThreads) {
    const unsigned h = (&s_hist[0][0])[k];
    if (h) atomicAdd(p.depth_hist + k, h);
  }
  const int num_tiles = (p.N + kBinThreads - 1) / kBinThreads;
  if (tid == 0) {
    if (tile_pairs) atomicAdd(p.pair_acc, (unsigned long long)tile_pairs);
    __threadfence();
    s_last = atomicAdd(p.done_counter, 1u) == (unsigned)(num_tiles - 1);
  }
  __syncthreads();
  if (s_last && tid == 0) {
    // every other CTA's pair total is visible after its fence + done_counter increment
    __threadfence();
    const unsigned long long m = atomicAdd(p.pair_acc, 0ull);
    const unsigned long long clamped = m > 0x7fffffffull ? 0x7fffffffull : m;
    *p.pair_count = (int)clamped;
    *p.n_visible = p.N;
    if (m > 0x7fffffffull) raise_device_error(kErrCapacity);
  }
}

static __global__ void __launch_bounds__(kBinThreads) bin_prepare_kernel(BinParams p) {
  __shared__ unsigned s_scan[33];
  __shared__ unsigned s_hist[4][256];
  __shared__ bool s_last;
  const int tid = threadIdx.x;
  for (int i = tid; i < 4 * 256; i += kBinThreads) (&s_hist[0][0])[i] = 0u;
  __syncthreads();
  const int tile = (int)blockIdx.x;
  const int i = tile * kBinThreads + tid;
  unsigned count = 0, depth_bits = 0;
  if (i < p.N) {
    const float2 mean = make_float2(__ldg(p.mean2d + 2 * i), __ldg(p.mean2d + 2 * i + 1));
    const float a = __ldg(p.cov2d + 3 * i), b = __ldg(p.cov2d + 3 * i + 1),
                c = __ldg(p.cov2d + 3 * i + 2);
    // colours and opacity are only read for splats that cover a tile
    TileRect r;
    if (splat_tile_rect(mean, a, b, c, p.W, p.H, p.tiles_x, p.tiles_y, r) && rect_count(r) > 0) {
      const float3 col = make_float3(__ldg(p.colors + 3 * i), __ldg(p.colors + 3 * i + 1),
                                     __ldg(p.colors + 3 * i + 2));
      count = bin_gaussian(p, i, mean, a, b, c, __ldg(p.depths + i), col, __ldg(p.alpha + i),
                           depth_bits);
    }
  }
  bin_block(p, tile, i, count, depth_bits, s_scan, s_hist, s_last);
}

struct DupParams {
  int tiles_x;
  int n_tile_passes;
  int runs;               // runs of kBinThreads Gaussians per CTA, 1..kDupRuns
  int tile_shift[4];      // digit bit offset of each tile-sort pass
  unsigned tile_mask[4];  // digit mask of each tile-sort pass
  const int* n_visible;
  const int* pair_count;
  long long pair_capacity;
  const unsigned* sorted_gids;  // depth-sorted Gaussians
  const uint2* rects;
  unsigned* status;
  unsigned* ticket;
  unsigned* tile_keys;
  unsigned* tile_vals;
  unsigned* tile_hist;  // [n_tile_passes][256]
};

// Exclusive scan of the tile counts in depth order and duplication of each Gaussian into
// one (tile id, Gaussian index) pair per covered tile, row-major over its rectangle
// (the order of csrc/forward/rasterize.cu:124-135). A CTA takes p.runs (1 to kDupRuns)
// consecutive runs of kBinThreads Gaussians: one look-back per CTA over fewer CTAs keeps the
// decoupled look-back chain short (with one run per CTA at 1M Gaussians the other warps spent
// most of the kernel waiting at the barrier behind warp 0's walk), and the runs' rectangle loads
// are in flight together. The host picks the runs so that the grid keeps at least four CTAs per
// SM (dup_runs): few Gaussians with many pairs each need the CTAs more than a short chain. Within a run a warp's 32 Gaussians own a contiguous run of pairs, which the
// warp writes 32 at a time: lanes where a Gaussian's pairs start in the current window record
// their lane in a per-warp table and the window's start positions are OR-reduced into one
// mask; pair lane q takes the Gaussian of the highest start at or below q (or the one carried
// from the previous window) and fetches its rectangle by shuffle.
constexpr int kDupRuns = 4;  // most runs per CTA

// Runs per duplication CTA for N Gaussians on `sms` SMs: as many as keep >= 4 CTAs per SM.
inline int dup_runs(long long N, int sms) {
  const long long r = N / ((long long)kBinThreads * 4 * sms);
  return (int)(r < 1 ? 1 : (r > kDupRuns ? kDupRuns : r));
}

// Five CTAs per SM (48 registers, 8 bytes of spill) rather than the four that 56 registers
// allowed: 53.7 -> 50.3 us per config-4 view; the sort passes at five CTAs per SM spilled
// 116 bytes and were slower.
static __global__ void __launch_bounds__(kBinThreads, 5) scan_duplicate_kernel(DupParams p) {
  __shared__ unsigned s_tile, s_prefix;
  __shared__ unsigned s_scan[33];
  __shared__ unsigned s_owner[kBinThreads / 32][32];
  __shared__ unsigned s_hist[4][256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr unsigned kFull = 0xffffffffu;
  if ((long long)(*p.pair_count) > p.pair_capacity) return;
  const int nv = *p.n_visible;
  const int items = kBinThreads * p.runs;  // Gaussians per CTA
  const int num_tiles = (nv + items - 1) / items;
  if (tid == 0) s_tile = atomicAdd(p.ticket, 1u);
  for (int k = tid; k < 4 * 256; k += kBinThreads) (&s_hist[0][0])[k] = 0u;
  __syncthreads();
  const int tile = (int)s_tile;
  if (tile >= num_tiles) return;
  unsigned count[kDupRuns], gid[kDupRuns];
  uint2 pr[kDupRuns];
#pragma unroll
  for (int r = 0; r < kDupRuns; ++r) {
    const int j = tile * items + r * kBinThreads + tid;
    gid[r] = r < p.runs && j < nv ? p.sorted_gids[j] : 0u;
  }
#pragma unroll
  for (int r = 0; r < kDupRuns; ++r) {
    const int j = tile * items + r * kBinThreads + tid;
    const bool ok = r < p.runs && j < nv;
    pr[r] = ok ? p.rects[gid[r]] : make_uint2(0u, 0u);
    count[r] = ok ? rect_count(unpack_rect(pr[r])) : 0u;
  }
  // per run: each thread's exclusive offset within its run, and the run's total
  unsigned excl[kDupRuns], run_pairs[kDupRuns], tile_pairs = 0;
#pragma unroll
  for (int r = 0; r < kDupRuns; ++r) {
    excl[r] = 0u;
    run_pairs[r] = 0u;
    if (r < p.runs) {  // uniform over the CTA
      excl[r] = block_exclusive_scan(count[r], s_scan, &run_pairs[r]);
      tile_pairs += run_pairs[r];
    }
  }
  if (tid == 0)
    st_relaxed(p.status + tile, (tile == 0 ? kFlagPrefix : kFlagAggregate) | tile_pairs);
  if (tid < 32) {
    unsigned prefix = 0;
    if (tile > 0) prefix = lookback_warp(p.status, tile);
    if (tid == 0) {
      if (tile > 0) st_relaxed(p.status + tile, kFlagPrefix | (prefix + tile_pairs));
      s_prefix = prefix;
    }
  }
  __syncthreads();
  const unsigned M = (unsigned)*p.pair_count;
  if (s_prefix + tile_pairs > M) {  // only reachable after a look-back timeout
    if (tid == 0) raise_device_error(kErrBadIndex);
    return;
  }
  const unsigned le = lane == 31 ? kFull : ((2u << lane) - 1u);  // lanes 0..lane
  unsigned* table = s_owner[warp];
  unsigned base = s_prefix;  // first pair of the current run
#pragma unroll
  for (int r = 0; r < kDupRuns; ++r) {
    if (r >= p.runs) break;  // uniform over the CTA
    // this warp's run of pairs: [w_first, w_first + w_total) of the run's
    const unsigned w_first = __shfl_sync(kFull, excl[r], 0);
    const unsigned w_total = __shfl_sync(kFull, excl[r] + count[r], 31) - w_first;
    const unsigned my_o = excl[r] - w_first;
    const TileRect mine = unpack_rect(pr[r]);
    const unsigned my_w = count[r] > 0 ? (unsigned)(mine.x1 - mine.x0) : 1u;
    const float my_inv_w = 1.0f / (float)my_w;
    const bool has = count[r] > 0;
    const unsigned prx = pr[r].x, pry = pr[r].y, my_gid = gid[r];
    int carried = 0;
    for (unsigned wb = 0; wb < w_total; wb += 32) {
      const bool starts_here = has && my_o >= wb && my_o < wb + 32;
      if (starts_here) table[my_o - wb] = (unsigned)lane;
      const unsigned starts = __reduce_or_sync(kFull, starts_here ? 1u << (my_o - wb) : 0u);
      __syncwarp();
      const unsigned m = starts & le;
      const int owner = m ? (int)table[31 - __clz(m)] : carried;
      const unsigned o_own = __shfl_sync(kFull, my_o, owner);
      const unsigned rx = __shfl_sync(kFull, prx, owner), ry = __shfl_sync(kFull, pry, owner);
      const unsigned g_own = __shfl_sync(kFull, my_gid, owner);
      const float inv_w = __shfl_sync(kFull, my_inv_w, owner);
      const unsigned q = wb + (unsigned)lane;
      if (q < w_total) {
        const TileRect rc = unpack_rect(make_uint2(rx, ry));
        const unsigned w = (unsigned)(rc.x1 - rc.x0);
        const unsigned lp = q - o_own;
        // row = lp / w from the float reciprocal, then made exact
        unsigned row = (unsigned)(((float)lp + 0.5f) * inv_w);
        if (row * w > lp) --row;
        if ((row + 1) * w <= lp) ++row;
        const unsigned col = lp - row * w;
        const unsigned tile_id =
            (unsigned)(rc.y0 + (int)row) * (unsigned)p.tiles_x + (unsigned)rc.x0 + col;
        p.tile_keys[base + w_first + q] = tile_id;
        p.tile_vals[base + w_first + q] = g_own;
#pragma unroll
        for (int pass = 0; pass < 4; ++pass)  // constant indices keep the parameters in registers
          if (pass < p.n_tile_passes)
            atomicAdd(&s_hist[pass][(tile_id >> p.tile_shift[pass]) & p.tile_mask[pass]], 1u);
      }
      carried = __shfl_sync(kFull, owner, 31);
      __syncwarp();  // the next window rewrites the table
    }
    base += run_pairs[r];
  }
  __syncthreads();
  for (int k = tid; k < p.n_tile_passes * 256; k += kBinThreads) {
    const unsigned h = (&s_hist[0][0])[k];
    if (h) atomicAdd(p.tile_hist + k, h);
  }
}

// Launch order of the blend CTAs: tiles by decreasing list length, so the long serial
// walks of crowded tiles start first and the short ones fill in behind them (with raster
// order a crowded tile that starts late sets the kernel's end). Lengths are bucketed by
// their leading bit and the two bits below it (129 buckets, descending); order within a
// bucket is arbitrary. The outputs do not depend on the order. One CTA.
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 129;

__device__ __forceinline__ int tile_order_bucket(int K) {
  if (K <= 0) return 0;
  const int lead = 31 - __clz(K);
  const int next2 = lead >= 2 ? (K >> (lead - 2)) & 3 : (K << (2 - lead)) & 3;
  return 1 + 4 * lead + next2;
}

// It also finishes the tile ranges (csrc/forward/rasterize.cu:146-165: [start, end) of each
// tile in the sorted pairs, empty tiles (0, 0)): with one tile the range is (0, M); otherwise the
// final tile-sort pass left (start, -end) for every tile with pairs and kRangeUnset for the
// others.
static __global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(
    int2* __restrict__ ranges, const int* pair_count, long long pair_capacity, int num_tiles,
    int* __restrict__ order) {
  __shared__ unsigned s_hist[kOrderBuckets];
  if ((long long)(*pair_count) > pair_capacity) return;  // the blend kernels return too
  const int tid = threadIdx.x;
  for (int b = tid; b < kOrderBuckets; b += kOrderThreads) s_hist[b] = 0u;
  __syncthreads();
  const int M = *pair_count;
  for (int t = tid; t < num_tiles; t += kOrderThreads) {
    int2 r = ranges[t];
    if (num_tiles == 1)
      r = make_int2(0, M);
    else
      r = r.x == kRangeUnset ? make_int2(0, 0) : make_int2(r.x, -r.y);
    ranges[t] = r;
    atomicAdd(&s_hist[tile_order_bucket(r.y - r.x)], 1u);
  }
  __syncthreads();
  if (tid == 0) {  // exclusive scan from the heaviest bucket down
    unsigned run = 0;
    for (int b = kOrderBuckets - 1; b >= 0; --b) {
      const unsigned h = s_hist[b];
      s_hist[b] = run;
      run += h;
    }
  }
  __syncthreads();
  for (int t = tid; t < num_tiles; t += kOrderThreads) {
    const int2 r = ranges[t];
    order[atomicAdd(&s_hist[tile_order_bucket(r.y - r.x)], 1u)] = t;
  }
}

}  // namespace gs
