// One pass of a stable least-significant-digit radix sort of (u32 key, u32 value) pairs
// with digits of up to 8 bits, after Adinets & Merrill, "Onesweep: A Faster Least Significant Digit
// Radix Sort for GPUs" (2022): a single kernel per digit that ranks a tile of items with
// warp-level multi-split, publishes per-digit tile counts and resolves each tile's global
// offset with a decoupled look-back over its predecessors, then scatters through shared
// memory so that every digit run is written contiguously.
#pragma once

#include "gs_common.cuh"

namespace gs {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
#ifndef GS_SORT_ITEMS
#define GS_SORT_ITEMS 12
#endif
constexpr int kSortItems = GS_SORT_ITEMS;               // items per thread
constexpr int kSortTileItems = kSortThreads * kSortItems;  // 3072 items per tile
constexpr int kRadix = 256;

struct SortPass {
  const unsigned* keys_in;
  const unsigned* vals_in;
  unsigned* keys_out;        // may be null when the sorted keys are not needed
  unsigned* vals_out;
  const int* n_items;        // device-side item count
  const int* overflow_count; // when non-null and *overflow_count > overflow_limit: no work
  long long overflow_limit;
  const unsigned* digit_hist;  // global histogram of this pass's digit [256]
  unsigned* status;            // look-back words [tiles][256], zeroed before the sort
  unsigned* ticket;            // tile ticket counter, zeroed before the sort
  int shift;                   // bit offset of this pass's digit
  unsigned mask;               // digit mask: (1 << digit bits) - 1, at most 255
  // Final pass of the tile sort only (else null): the keys are tile ids, this pass's digit is
  // their top digit, and each tile's [start, end) in the sorted order is written here as
  // (start, -end), both initialised to kRangeUnset (see tile_order_kernel, which decodes them).
  int2* ranges = nullptr;
  unsigned num_tiles = 0;
};

// Four CTAs per SM (64 registers, 48 bytes of spill): against three (80 registers, none), the
// tile sort 109.0 -> 107.3 us per config-4 view and the config-4 step 743.9 -> 751.7 views/s,
// the passes' latency hidden by more warps while other views' kernels share the SMs.
static __global__ void __launch_bounds__(kSortThreads, 4) onesweep_pass_kernel(SortPass a) {
  __shared__ unsigned s_tile;
  __shared__ unsigned s_warp_hist[kSortWarps][kRadix];
  __shared__ unsigned s_local_start[kRadix];
  __shared__ unsigned s_global_off[kRadix];
  __shared__ unsigned s_scan[33];
  __shared__ unsigned s_keys[kSortTileItems];
  __shared__ unsigned s_vals[kSortTileItems];

  if (a.overflow_count && (long long)(*a.overflow_count) > a.overflow_limit) return;
  const int n = *a.n_items;
  const int num_tiles = (n + kSortTileItems - 1) / kSortTileItems;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) s_tile = atomicAdd(a.ticket, 1u);
  for (int i = tid; i < kSortWarps * kRadix; i += kSortThreads) (&s_warp_hist[0][0])[i] = 0u;
  __syncthreads();
  const int tile = (int)s_tile;
  if (tile >= num_tiles) return;

  // ---- load a warp-striped tile: warp w owns items [w * 32 * kSortItems, ...) ------------
  const int warp_base = tile * kSortTileItems + warp * (32 * kSortItems);
  unsigned keys[kSortItems], vals[kSortItems], rank[kSortItems];
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    const int idx = warp_base + j * 32 + lane;
    const bool valid = idx < n;
    keys[j] = valid ? __ldcs(a.keys_in + idx) : 0u;
    vals[j] = valid ? __ldcs(a.vals_in + idx) : 0u;
  }

  // ---- warp-level multi-split ranking, in item order ------------------------------------
  unsigned* wh = s_warp_hist[warp];
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    const int idx = warp_base + j * 32 + lane;
    const bool valid = idx < n;
    const unsigned d = valid ? ((keys[j] >> a.shift) & a.mask) : (unsigned)kRadix;
    // lanes holding the same digit, one ballot per digit bit (bit 8 marks the invalid items);
    // measured against __match_any_sync at 1M Gaussians and 1080p: depth sort 95.0 -> 86.3 us,
    // tile sort 114.9 -> 109.3 us per view
    unsigned peers = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < 9; ++b) {
      const bool bit = (d >> b) & 1u;
      const unsigned ones = __ballot_sync(0xffffffffu, bit);
      peers &= bit ? ones : ~ones;
    }
    const unsigned lower = __popc(peers & lt);
    const unsigned cnt = valid ? wh[d] : 0u;
    rank[j] = cnt + lower;
    __syncwarp();
    if (valid && lower == 0) wh[d] = cnt + __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // ---- per digit (thread d): tile count, warp offsets, publish, look-back ----------------
  const int d = tid;
  unsigned tile_count = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) {
    const unsigned c = s_warp_hist[w][d];
    s_warp_hist[w][d] = tile_count;
    tile_count += c;
  }
  // a digit absent from the whole input has prefix 0 in every tile: published as final at
  // once, and no look-back runs for it
  const unsigned digit_total = __ldg(a.digit_hist + d);
  unsigned* my_status = a.status + (size_t)tile * kRadix + d;
  st_relaxed(my_status,
             (tile == 0 || digit_total == 0u ? kFlagPrefix : kFlagAggregate) | tile_count);

  unsigned tile_total;
  const unsigned local_start = block_exclusive_scan(tile_count, s_scan, &tile_total);
  unsigned hist_total;
  const unsigned digit_base = block_exclusive_scan(digit_total, s_scan, &hist_total);
  unsigned excl = 0;
  if (tile > 0 && digit_total != 0u) {
    excl = lookback_serial(a.status + d, tile, kRadix);
    st_relaxed(my_status, kFlagPrefix | (excl + tile_count));
  }
  s_local_start[d] = local_start;
  s_global_off[d] = digit_base + excl - local_start;
  __syncthreads();

  // ---- scatter into shared memory in digit order, then write digit runs -----------------
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    const int idx = warp_base + j * 32 + lane;
    if (idx < n) {
      const unsigned dj = (keys[j] >> a.shift) & a.mask;
      const unsigned pos = s_local_start[dj] + wh[dj] + rank[j];
      s_keys[pos] = keys[j];
      s_vals[pos] = vals[j];
    }
  }
  __syncthreads();
  const int count = min(kSortTileItems, n - tile * kSortTileItems);
  for (int i = tid; i < count; i += kSortThreads) {
    const unsigned k = s_keys[i];
    const unsigned dg = (k >> a.shift) & a.mask;
    const unsigned gpos = s_global_off[dg] + i;
    if (gpos >= (unsigned)n) {  // only reachable after a look-back timeout
      raise_device_error(kErrBadIndex);
      continue;
    }
    if (a.keys_out) a.keys_out[gpos] = k;
    a.vals_out[gpos] = s_vals[i];
    if (a.ranges) {
      // Tile ranges. Within this tile of items each digit run lands contiguously in the
      // output, and within a run the keys are sorted (the earlier passes left the lower digits
      // in order and this one is stable), so a key change inside a run is exactly a tile's
      // start and its predecessor's end. At a run's ends the neighbour in the output belongs
      // to another tile of items: those candidates go through atomics (min of the starts, max
      // of the ends), which any exact store also written for that tile agrees with.
      if (k >= a.num_tiles) {
        raise_device_error(kErrBadIndex);
        continue;
      }
      const bool run_start = i == 0 || ((s_keys[i - 1] >> a.shift) & a.mask) != dg;
      const bool run_end = i == count - 1 || ((s_keys[i + 1] >> a.shift) & a.mask) != dg;
      if (run_start) {
        atomicMin(&a.ranges[k].x, (int)gpos);
      } else {
        const unsigned prev = s_keys[i - 1];
        if (prev != k) {
          a.ranges[k].x = (int)gpos;
          a.ranges[prev].y = -(int)gpos;
        }
      }
      if (run_end) atomicMin(&a.ranges[k].y, -(int)(gpos + 1));
    }
  }
}

}  // namespace gs
