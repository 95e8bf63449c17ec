// Front-to-back alpha blending of 16x16 tiles and its backward.
//
// One CTA per tile with 256 / kPix threads; each thread owns kPix pixels of one column,
// 4 rows apart, so warp w covers the 8 x (4 kPix) pixel block at ((w & 1) * 8, (w >> 1) * 4 kPix)
// of the tile. Pixels of a thread share each splat-record load, the warp's cull test and, in
// the backward, one warp reduction. The tile's depth-sorted splats are consumed in batches of
// blend records (48 bytes each; 256 per batch forward, 128 or 64 backward) gathered with cp.async
// into a double-buffered shared-memory ring: batch b + 1 is in flight while batch b is blended.
#pragma once

#include "gs_common.cuh"

namespace gs {

constexpr int kBlendBatch = 256;  // records per shared-memory batch, forward

// Pixels per thread. A thread's pixels share each record load, the warp's cull test and (in
// the backward) one warp reduction per splat, so more pixels per thread means fewer
// instructions per pixel, but fewer threads per tile and a longer kernel when it runs alone.
// The latency variants serve one view at a time; the throughput variants are for views that
// overlap on several streams (GS_RENDER_CONCURRENT), where the SMs are shared with other
// kernels and the instruction count sets the pace (config-4 step on one B200: 565 -> 584
// views/s, although each blend kernel alone is 3% / 26% slower).
constexpr int kBlendFwdPix = 1;            // forward, one view at a time
constexpr int kBlendFwdPixThroughput = 2;  // forward, overlapped views
constexpr int kBlendBwdPix = 2;            // backward, one view at a time
constexpr int kBlendBwdPixThroughput = 4;  // backward, overlapped views

// Backward shared-memory batch (records) and resident CTAs per SM: 128 records and 10 CTAs of
// 128 threads (43 registers) at two pixels per thread; 64 records and 16 CTAs of 64 threads
// (56 registers) at four.
template <int kPix>
struct BlendBwdShape {
  static constexpr int kBatch = kPix >= 4 ? 64 : 128;
  static constexpr int kMinBlocks = kPix >= 4 ? 16 : 10;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Pixel block of this thread's warp and the column / first row of the thread's pixels.
template <int kPix>
struct BlendGeometry {
  float wx0, wy0;  // warp block origin
  int px, py0;     // thread column, first row; pixel q is at (px, py0 + 4 q)
  __device__ __forceinline__ BlendGeometry(int tile_x, int tile_y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bx = tile_x * kTileSide + (warp & 1) * 8;
    const int by = tile_y * kTileSide + (warp >> 1) * 4 * kPix;
    wx0 = (float)bx;
    wy0 = (float)by;
    px = bx + (lane & 7);
    py0 = by + (lane >> 3);
  }
};

// Can splat record (r0 = (mean, extent), r1 = (conic, opacity)) reach the warp's pixel block
// (pixel centres [wx0, wx0 + 7] x [wy0, wy0 + 4 kPix - 1])? First its extent box, then its
// opacity ellipse: a pixel passes the opacity test only where Q(d) = d^T conic d <=
// tau = 2 ln(255 o), so the block is reachable only if the minimum of Q over the block's
// rectangle (offsets d from the mean) is at most tau. Q is convex with its minimum at d = 0,
// so the rectangle's minimum lies on an edge that faces the mean (or is 0 when the mean is
// inside): one candidate per axis, the clamped line minimum on the edge nearest the mean,
// and the smaller of the two is the minimum. The test is conservative: tau is inflated as the
// extent is (1% + 1e-3) and a degenerate conic falls back to the box.
template <int kPix>
__device__ __forceinline__ bool warp_block_hit(float4 r0, float4 r1, float wx0, float wy0) {
  constexpr float kSpanY = 4.0f * kPix - 1.0f;
  if (!(r0.x + r0.z >= wx0 && r0.x - r0.z <= wx0 + 7.0f && r0.y + r0.w >= wy0 &&
        r0.y - r0.w <= wy0 + kSpanY))
    return false;
  const float a = r1.x, b = r1.y, c = r1.z;
  if (!(a > 0.0f && c > 0.0f && a * c > b * b)) return true;
  const float x0 = wx0 - r0.x, x1 = x0 + 7.0f, y0 = wy0 - r0.y, y1 = y0 + kSpanY;
  const float X = fminf(fmaxf(0.0f, x0), x1);  // the edge (or centre column) nearest the mean
  const float Y = fminf(fmaxf(0.0f, y0), y1);
  const float yX = fminf(fmaxf(__fdividef(-b * X, c), y0), y1);  // line minimum on x = X
  const float xY = fminf(fmaxf(__fdividef(-b * Y, a), x0), x1);  // line minimum on y = Y
  const float qX = fmaf(a * X, X, fmaf(2.0f * b * X, yX, c * yX * yX));
  const float qY = fmaf(a * xY, xY, fmaf(2.0f * b * xY, Y, c * Y * Y));
  const float tau = 2.0f * __logf(255.0f * r1.w);
  return fminf(qX, qY) <= fmaf(tau, 1.01f, 1e-3f);
}

__device__ __forceinline__ float approx_sqrt(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Which rows of the warp's pixel block (pixel centres [wx0, wx0 + 7] x [wy0, wy0 + 4 kPix - 1])
// can splat record (r0 = (mean, extent), r1 = (conic, opacity)) reach? Bit q of the result
// stands for the 8 x 4 sub-block of rows [4q, 4q + 3], the pixels q of the warp's threads;
// 0 means the splat misses the block. A pixel passes the opacity test only where
// Q(d) = d^T conic d <= tau = 2 ln(255 o) (d: offset from the mean), an ellipse. Past the extent
// box test, the ellipse's y-range over the block's column band x in [x0, x1] is exact by
// convexity: the top of the band's slice is the ellipse's upper boundary at the band point
// nearest the ellipse's topmost point (clamped), the bottom likewise at the bottommost point.
// The test is conservative: tau is inflated as the extent is (1% + 1e-3), the range widened by
// 0.05 px, and a degenerate conic keeps the extent box.
template <int kPix>
__device__ __forceinline__ unsigned warp_block_reach(float4 r0, float4 r1, float wx0, float wy0) {
  constexpr float kSpanY = 4.0f * kPix - 1.0f;
  if (!(r0.x + r0.z >= wx0 && r0.x - r0.z <= wx0 + 7.0f && r0.y + r0.w >= wy0 &&
        r0.y - r0.w <= wy0 + kSpanY))
    return 0u;
  const float y0 = wy0 - r0.y;
  float lo = -r0.w - y0, hi = r0.w - y0;  // reached rows, relative to wy0 (extent box)
  const float a = r1.x, b = r1.y, c = r1.z;
  const float det = a * c - b * b;
  if (a > 0.0f && c > 0.0f && det > 0.0f) {
    const float x0 = wx0 - r0.x, x1 = x0 + 7.0f;
    const float tau = fmaf(2.0f * __logf(255.0f * r1.w), 1.01f, 1e-3f);
    const float ct = c * tau;
    const float yt = approx_sqrt(fmaxf(__fdividef(tau * a, det), 0.0f));  // topmost point
    const float xt = __fdividef(-b * yt, a);
    const float xa = fminf(fmaxf(xt, x0), x1), xb = fminf(fmaxf(-xt, x0), x1);
    const float inv_c = __fdividef(1.0f, c);
    const float ya = (-b * xa + approx_sqrt(fmaxf(fmaf(-det * xa, xa, ct), 0.0f))) * inv_c;
    const float yb = (-b * xb - approx_sqrt(fmaxf(fmaf(-det * xb, xb, ct), 0.0f))) * inv_c;
    lo = fmaxf(lo, yb - 0.05f - y0);
    hi = fminf(hi, ya + 0.05f - y0);
  }
  if (!(hi >= 0.0f && lo <= kSpanY && lo <= hi)) return 0u;
  // sub-block q is reached iff hi >= 4q and lo <= 4q + 3
  const int q_hi = min((int)(fminf(hi, kSpanY) * 0.25f), kPix - 1);
  const int q_lo = max((int)ceilf((fmaxf(lo, -4.0f) - 3.0f) * 0.25f), 0);
  if (q_lo > q_hi) return 0u;
  return ((2u << q_hi) - 1u) & ~((1u << q_lo) - 1u);
}

// Rows of the block a record reaches (bit q: pixels q of the warp's threads). With four
// pixels per thread the per-row mask pays for its cost (40% of the row groups of a hit block
// are missed at config 4); with one or two the plain block test is cheaper.
template <int kPix>
__device__ __forceinline__ unsigned warp_block_rows(float4 r0, float4 r1, float wx0, float wy0) {
  if constexpr (kPix >= 4) {
    return warp_block_reach<kPix>(r0, r1, wx0, wy0);
  } else {
    return warp_block_hit<kPix>(r0, r1, wx0, wy0) ? (1u << kPix) - 1u : 0u;
  }
}

struct BlendFwdParams {
  int W, H, tiles_x, num_tiles;
  const int2* ranges;
  const int* tile_order;  // CTA -> tile (tile_order_kernel); null: raster order
  const int* sorted_ids;
  const float4* records;
  const int* pair_count;
  long long pair_capacity;
  float* img;
  float* final_T;
  int* n_contrib;
};

// Forward blend (csrc/forward/rasterize.cu:188-280): for each pixel, in depth order,
// alpha = min(0.99, o * exp(power)), skipped when power > 0 or alpha < 1/255; colour
// accumulates c * alpha * T and T *= 1 - alpha; the pixel stops after the Gaussian that
// takes T below 1e-4. n_contrib is the 1-based list position of the last Gaussian applied.
// A warp skips splats whose opacity ellipse misses its pixel block, and the pixels q of its
// threads skip splats that miss their rows of the block (warp_block_rows): those
// fail the opacity test at every pixel of the block, so the outputs are unchanged.
template <int kPix>
static __global__ void __launch_bounds__(kTilePixels / kPix)
    blend_forward_kernel(BlendFwdParams p) {
  constexpr int kThreads = kTilePixels / kPix;
  __shared__ float4 s_rec[2][3][kBlendBatch];
  if ((long long)(*p.pair_count) > p.pair_capacity) return;
  const int tile = p.tile_order ? p.tile_order[blockIdx.x] : (int)blockIdx.x;
  if (tile < 0 || tile >= p.num_tiles) {  // never for a tile order the sort wrote
    if (threadIdx.x == 0) raise_device_error(kErrBadIndex);
    return;
  }
  const int tile_x = tile % p.tiles_x, tile_y = tile / p.tiles_x;
  const int tid = threadIdx.x, lane = tid & 31;
  const BlendGeometry<kPix> geo(tile_x, tile_y);
  const int2 range = p.ranges[tile];
  const int K = range.y - range.x;
  const int nbatches = (K + kBlendBatch - 1) / kBlendBatch;

  static_assert(kBlendBatch % kThreads == 0, "each thread issues whole records");
  auto issue = [&](int b) {
    float4(*dst)[kBlendBatch] = s_rec[b & 1];
#pragma unroll
    for (int r = 0; r < kBlendBatch / kThreads; ++r) {
      const int slot = tid + r * kThreads;
      const int j = b * kBlendBatch + slot;
      if (j < K) {
        const int g = p.sorted_ids[range.x + j];
        const float4* src = p.records + 3 * (size_t)g;
        cp_async16(&dst[0][slot], src);
        cp_async16(&dst[1][slot], src + 1);
        cp_async16(&dst[2][slot], src + 2);
      }
    }
    cp_async_commit();
  };

  float T[kPix], cr[kPix], cg[kPix], cb[kPix], fpy[kPix];
  int last[kPix];
  bool done[kPix];
  const float fpx = (float)geo.px;
#pragma unroll
  for (int q = 0; q < kPix; ++q) {
    T[q] = 1.0f;
    cr[q] = cg[q] = cb[q] = 0.0f;
    last[q] = 0;
    done[q] = !(geo.px < p.W && geo.py0 + 4 * q < p.H);
    fpy[q] = (float)(geo.py0 + 4 * q);
  }
  if (nbatches > 0) issue(0);
  for (int b = 0; b < nbatches; ++b) {
    if (b + 1 < nbatches) {
      issue(b + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int n = min(kBlendBatch, K - b * kBlendBatch);
    const float4(*rec)[kBlendBatch] = s_rec[b & 1];
    bool all_done = true;
#pragma unroll
    for (int q = 0; q < kPix; ++q) all_done = all_done && done[q];
    // 32 records at a time: each lane tests one against the warp's pixel block, the warp
    // walks the hits in list order (pixels that are done skip them)
    for (int k = 0; k < n && !__all_sync(0xffffffffu, all_done); k += 32) {
      const int i_lane = k + lane;
      const unsigned reach =
          i_lane < n ? warp_block_rows<kPix>(rec[0][i_lane], rec[1][i_lane], geo.wx0, geo.wy0)
                     : 0u;
      unsigned hits = __ballot_sync(0xffffffffu, reach != 0u);
      while (hits) {
        const int src = __ffs(hits) - 1;
        const int i = k + src;
        hits &= hits - 1;
        const unsigned rows =  // warp-uniform
            kPix >= 4 ? __shfl_sync(0xffffffffu, reach, src) : (1u << kPix) - 1u;
        const float4 r0 = rec[0][i];
        const float4 r1 = rec[1][i];
        const float dx = fpx - r0.x;
#pragma unroll
        for (int q = 0; q < kPix; ++q) {
          if (!((rows >> q) & 1u)) continue;  // the splat misses these rows of the block
          if (done[q]) continue;
          const float dy = fpy[q] - r0.y;
          const float power = splat_power(make_float3(r1.x, r1.y, r1.z), dx, dy);
          if (power > 0.0f) continue;
          const float alpha = fminf(0.99f, __fmul_rn(r1.w, __expf(power)));
          if (alpha < (1.0f / 255.0f)) continue;
          blend_step(alpha, rec[2][i], T[q], cr[q], cg[q], cb[q]);
          last[q] = b * kBlendBatch + i + 1;
          if (T[q] < 1e-4f) done[q] = true;
        }
      }
      all_done = true;
#pragma unroll
      for (int q = 0; q < kPix; ++q) all_done = all_done && done[q];
    }
    if (__syncthreads_count(all_done) == kThreads) break;
  }
  cp_async_wait<0>();
#pragma unroll
  for (int q = 0; q < kPix; ++q) {
    const int py = geo.py0 + 4 * q;
    if (geo.px < p.W && py < p.H) {
      const int pix = py * p.W + geo.px;
      p.img[3 * pix + 0] = cr[q];
      p.img[3 * pix + 1] = cg[q];
      p.img[3 * pix + 2] = cb[q];
      p.final_T[pix] = T[q];
      p.n_contrib[pix] = last[q];
    }
  }
}

struct BlendBwdParams {
  int N, W, H, tiles_x;
  int num_tiles;
  // the forward's pair count and capacity (fused path): a forward whose pairs overflowed its
  // buffers wrote no tile order, ranges or counts, so its backward does nothing; null: the
  // caller's tile ranges are valid (stand-alone API)
  const int* pair_count;
  long long pair_capacity;
  const float* grad_img;
  const int2* ranges;
  const int* tile_order;  // CTA -> tile (tile_order_kernel); null: raster order
  const int* sorted_ids;
  const float4* records;  // 3 per Gaussian, indexed by Gaussian id
  const float* final_T;
  const int* n_contrib;
  float* g_mean2d;
  float* g_cov2d;
  float* g_colors;
  float* g_alpha;
  float4* g_accum;  // fused mode: 3 float4 per Gaussian (see blend_backward_kernel)
};

// Butterfly reduce-scatter of 9 per-lane values over a warp in 12 shuffles. On return the
// even lane of each lane pair holding a real value index (0..8) has the warp total of
// that value in *out and the index in *slot; other lanes get slot = -1.
__device__ __forceinline__ void warp_reduce9(const float (&v)[9], float* out, int* slot) {
  const int lane = threadIdx.x & 31;
  const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1,
             b1 = (lane >> 1) & 1;
  float w[6];
  {
    const float p[10] = {v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], 0.0f};
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const float keep = b4 ? p[k + 5] : p[k];
      const float send = b4 ? p[k] : p[k + 5];
      w[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    w[5] = 0.0f;
  }
  float x[4];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float keep = b3 ? w[k + 3] : w[k];
    const float send = b3 ? w[k] : w[k + 3];
    x[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  x[3] = 0.0f;
  float y[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float keep = b2 ? x[k + 2] : x[k];
    const float send = b2 ? x[k] : x[k + 2];
    y[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  float z;
  {
    const float keep = b1 ? y[1] : y[0];
    const float send = b1 ? y[0] : y[1];
    z = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  z += __shfl_xor_sync(0xffffffffu, z, 1);
  const int xi = (b2 ? 2 : 0) + (b1 ? 1 : 0);
  const int wi = (b3 ? 3 : 0) + xi;
  const int vi = (b4 ? 5 : 0) + wi;
  *out = z;
  *slot = ((lane & 1) == 0 && xi < 3 && wi < 5 && vi < 9) ? vi : -1;
}

constexpr int kAccStride = 9;  // 9 gradient sums per batch slot (odd: conflict-free flush)

// Per-hit reduction through shared memory (four pixels per thread): each lane stores its 9
// sums of a hit as column `lane` of 9 rows of 32 floats; after kRedHits hits, lane r < 9 kRedHits
// sums row r (eight 16-byte loads starting at a lane-dependent quarter, so the 8 lanes of a
// load phase hit distinct banks) and adds it to the hit's batch slot. 9 stores per hit and one
// 8-load, 31-add pass per kRedHits hits replace the 12-shuffle reduce-scatter (config-4 step
// 650 -> 658 views/s). The rows cost 2.3 KB per warp: 16 CTAs of 64 threads still fit an SM,
// 10 CTAs of 128 threads (two pixels per thread) would not.
constexpr int kRedHits = 2;

__device__ __forceinline__ void flush_hit_rows(const float* rows, int n_hits, int k0, int k1,
                                               float* s_acc) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  if (lane < 9 * n_hits) {
    const float4* row = reinterpret_cast<const float4*>(rows + lane * 32);
    float4 acc = row[lane & 7];
#pragma unroll
    for (int t = 1; t < 8; ++t) {
      const float4 x = row[(lane + t) & 7];
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    const float sum = (acc.x + acc.y) + (acc.z + acc.w);
    const int h = lane >= 9 ? 1 : 0;
    const int slot = (h ? k1 : k0) * kAccStride + (lane - 9 * h);
    if (sum != 0.0f) atomicAdd(&s_acc[slot], sum);
  }
  __syncwarp();
}

// Backward blend (csrc/backward/rasterize_backward.cu:60-235). Each pixel replays its
// Gaussians back to front from its n_contrib, recovering T before each one as
// T / max(1 - alpha, 1e-4), and produces dL/d(mean, conic, colour, opacity). The tile
// walk starts at the batch holding the tile's largest n_contrib instead of the list end;
// each warp starts at its own largest n_contrib and skips splats whose opacity ellipse misses
// its pixel block and each pixel row group q the splats that miss its rows (warp_block_rows;
// exact: they fail the opacity test there). Per Gaussian, the contributions of a
// thread's pixels are summed, reduced per warp (warp_reduce9) and added into a per-batch shared
// slot; after each batch the slot sums are flushed to the global gradients.
//
// Two rewrites keep the per-pixel work small (both linear, so only the rounding differs from
// the reference's per-pixel expressions): the mean and conic gradients are accumulated as the
// moments St = sum(dL/dpower dx), Su = sum(dL/dpower dy), sum(dL/dpower dx dx), sum(dL/dpower dx dy),
// sum(dL/dpower dy dy) and multiplied by the splat's conic at the flush; and the three
// accumulated colours behind the splat enter dL/dalpha only through their dot product with
// dL/dpixel, so one scalar D replaces them (D' = alpha (c . g) + (1 - alpha) D). A thread's
// pixels share one column, so per pixel only sum(dL/dpower), sum(dL/dpower dy) and
// sum(dL/dpower dy^2) are kept and the dx factors are applied once per splat.
//
// Both flushes convert each tile's dL/dconic to dL/dSigma2 = -V G V with the tile's own sums, as
// the reference does per (tile, Gaussian) (csrc/backward/rasterize_backward.cu:211-221): the
// conversion is linear, but for near-singular 2D covariances (needle-like splats) its
// cancellation error depends on what is summed first, and converting per tile keeps the
// reference's rounding. kFusedAccum selects the destination: false adds into the four
// reference-layout gradient arrays (9 scalar atomics, as the reference does); true adds into
// g_accum with vector atomics, 3 float4 per Gaussian:
//   [0] = (dmean.x, dmean.y, dSigma2.a, dSigma2.b), [1] = (dSigma2.c, dopacity, dcol.r,
//   dcol.g), [2] = (dcol.b, -, -, -).
template <bool kFusedAccum, int kPix>
__global__ void __launch_bounds__(kTilePixels / kPix, BlendBwdShape<kPix>::kMinBlocks)
    blend_backward_kernel(BlendBwdParams p) {
  constexpr int kThreads = kTilePixels / kPix;
  constexpr int kBlendBwdBatch = BlendBwdShape<kPix>::kBatch;
  __shared__ float4 s_rec[2][3][kBlendBwdBatch];
  __shared__ float s_acc[kBlendBwdBatch * kAccStride];
  __shared__ int s_max_last;
  constexpr bool kRowReduce = kPix >= 4;  // shared memory allows it at 16 CTAs per SM
  __shared__ __align__(16) float s_red[kRowReduce ? kThreads / 32 : 1][kRowReduce ? kRedHits * 9 * 32 : 4];
  float* const my_rows = s_red[kRowReduce ? (threadIdx.x >> 5) : 0];
  int pending = 0, pend_k0 = 0;
  if (p.pair_count && (long long)(*p.pair_count) > p.pair_capacity) return;
  const int tile = p.tile_order ? p.tile_order[blockIdx.x] : (int)blockIdx.x;
  if (tile < 0 || tile >= p.num_tiles) {  // never for a tile order the forward wrote
    if (threadIdx.x == 0) raise_device_error(kErrBadIndex);
    return;
  }
  const int tile_x = tile % p.tiles_x, tile_y = tile / p.tiles_x;
  const int tid = threadIdx.x, lane = tid & 31;
  const BlendGeometry<kPix> geo(tile_x, tile_y);
  const int2 range = p.ranges[tile];
  const int K = range.y - range.x;

  // D = sum over channels of (colour accumulated behind the current splat) x dL/dpixel
  float gr[kPix], gg[kPix], gb[kPix], T[kPix], D[kPix], fpy[kPix];
  int last[kPix];
  int my_last = 0;
#pragma unroll
  for (int q = 0; q < kPix; ++q) {
    const int py = geo.py0 + 4 * q;
    gr[q] = gg[q] = gb[q] = T[q] = 0.0f;
    D[q] = 0.0f;
    last[q] = 0;
    fpy[q] = (float)py;
    if (geo.px < p.W && py < p.H) {
      const int pix = py * p.W + geo.px;
      gr[q] = p.grad_img[3 * pix];
      gg[q] = p.grad_img[3 * pix + 1];
      gb[q] = p.grad_img[3 * pix + 2];
      T[q] = p.final_T[pix];
      last[q] = min(p.n_contrib[pix], K);
    }
    my_last = max(my_last, last[q]);
  }
  if (tid == 0) s_max_last = 0;
  for (int k = tid; k < kBlendBwdBatch * kAccStride; k += kThreads) s_acc[k] = 0.0f;
  __syncthreads();
  const int warp_last = __reduce_max_sync(0xffffffffu, my_last);  // this warp's replay length
  if ((tid & 31) == 0 && warp_last > 0) atomicMax(&s_max_last, warp_last);
  __syncthreads();
  const int K_eff = s_max_last;  // list prefix that any pixel of this tile replays
  const int nbatches = (K_eff + kBlendBwdBatch - 1) / kBlendBwdBatch;

  // batch b covers list indices [lo(b), hi(b)) walking from the back
  auto batch_hi = [&](int b) { return K_eff - b * kBlendBwdBatch; };
  auto batch_lo = [&](int b) { return max(0, K_eff - (b + 1) * kBlendBwdBatch); };
  static_assert(kBlendBwdBatch % kThreads == 0, "each thread issues whole records");
  auto issue = [&](int b) {
    const int lo = batch_lo(b), hi = batch_hi(b);
    float4(*dst)[kBlendBwdBatch] = s_rec[b & 1];
#pragma unroll
    for (int r = 0; r < kBlendBwdBatch / kThreads; ++r) {
      const int slot = tid + r * kThreads;
      const int j = lo + slot;
      if (j < hi) {
        const int g = p.sorted_ids[range.x + j];
        if (g >= 0 && g < p.N) {
          const float4* src = p.records + 3 * (size_t)g;
          cp_async16(&dst[0][slot], src);
          cp_async16(&dst[1][slot], src + 1);
          cp_async16(&dst[2][slot], src + 2);
        } else {
          // out-of-range id: a record no warp touches and the flush skips
          dst[0][slot] = make_float4(0.0f, 0.0f, -INFINITY, -INFINITY);
          dst[1][slot] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          dst[2][slot] = make_float4(0.0f, 0.0f, 0.0f, __int_as_float(-1));
        }
      }
    }
    cp_async_commit();
  };

  const float fpx = (float)geo.px;
  if (nbatches > 0) issue(0);
  for (int b = 0; b < nbatches; ++b) {
    if (b + 1 < nbatches) {
      issue(b + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int lo = batch_lo(b), hi = batch_hi(b);
    const float4(*rec)[kBlendBwdBatch] = s_rec[b & 1];
    // 32 list positions at a time from the back: lane l tests position top - 1 - l against
    // the warp's pixel block, the warp walks the hits back to front
    for (int top = min(hi, warp_last); top > lo; top -= 32) {
      const int j_lane = top - 1 - lane;
      const unsigned reach =
          j_lane >= lo
              ? warp_block_rows<kPix>(rec[0][j_lane - lo], rec[1][j_lane - lo], geo.wx0, geo.wy0)
              : 0u;
      unsigned hits = __ballot_sync(0xffffffffu, reach != 0u);
      while (hits) {
        const int src = __ffs(hits) - 1;
        const int j = top - 1 - src;
        hits &= hits - 1;
        const unsigned rows =  // warp-uniform
            kPix >= 4 ? __shfl_sync(0xffffffffu, reach, src) : (1u << kPix) - 1u;
        const int k = j - lo;  // slot in this batch
        const float4 r0 = rec[0][k];
        float v[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // the thread's pixels share one column (one dx): per pixel only sums over dL/dpower,
        // dL/dpower dy and dL/dpower dy^2; dx enters once per splat below
        float sp = 0.f, spy = 0.f, spyy = 0.f;
        bool active = false;
        const float4 r1 = rec[1][k];
        const float dx = fpx - r0.x;
#pragma unroll
        for (int q = 0; q < kPix; ++q) {
          if (!((rows >> q) & 1u)) continue;  // the splat misses these rows of the block
          if (j >= last[q]) continue;  // contributor j + 1 > n_contrib of this pixel
          const float dy = fpy[q] - r0.y;
          const float power = splat_power(make_float3(r1.x, r1.y, r1.z), dx, dy);
          if (power > 0.0f) continue;
          const float G = __expf(power);
          const float alpha_raw = r1.w * G;
          const float alpha = fminf(0.99f, alpha_raw);
          if (alpha < (1.0f / 255.0f)) continue;
          active = true;
          const float4 r2 = rec[2][k];
          // the reference divides by max(1 - alpha, 1e-4); alpha <= 0.99 keeps 1 - alpha >= 0.01,
          // so the clamp never acts and is left out. Approximate division (2 ulp): the
          // recovered T drifts by a few 1e-6 over a pixel's replay, far inside the gradient
          // tolerance
          const float one_minus = 1.0f - alpha;
          const float T_before = __fdividef(T[q], one_minus);
          const float wgt = alpha * T_before;
          v[5] += wgt * gr[q];
          v[6] += wgt * gg[q];
          v[7] += wgt * gb[q];
          const float cdotg = r2.x * gr[q] + r2.y * gg[q] + r2.z * gb[q];
          const float diff = cdotg - D[q];
          const float dL_dalpha = diff * T_before;
          float dL_dpower = 0.0f;
          if (alpha_raw < 0.99f) {
            v[8] += G * dL_dalpha;
            dL_dpower = alpha * dL_dalpha;
          }
          const float ty = dL_dpower * dy;
          sp += dL_dpower;
          spy += ty;
          spyy += ty * dy;
          D[q] += alpha * diff;  // alpha cdotg + (1 - alpha) D
          T[q] = T_before;
        }
        if (__any_sync(0xffffffffu, active)) {
          v[0] = sp * dx;   // sum dL/dpower dx
          v[1] = spy;       // sum dL/dpower dy
          v[2] = v[0] * dx; // sum dL/dpower dx^2
          v[3] = spy * dx;  // sum dL/dpower dx dy
          v[4] = spyy;      // sum dL/dpower dy^2
          if constexpr (kRowReduce) {
            float* rows = my_rows + pending * 9 * 32;
#pragma unroll
            for (int c = 0; c < 9; ++c) rows[c * 32 + lane] = v[c];
            if (pending + 1 == kRedHits) {
              flush_hit_rows(my_rows, kRedHits, pend_k0, k, s_acc);
              pending = 0;
            } else {
              pend_k0 = k;
              ++pending;
            }
          } else {
            float sum;
            int slot;
            warp_reduce9(v, &sum, &slot);
            if (slot >= 0 && sum != 0.0f) atomicAdd(&s_acc[k * kAccStride + slot], sum);
          }
        }
      }
    }
    if constexpr (kRowReduce) {
      if (pending > 0) flush_hit_rows(my_rows, pending, pend_k0, pend_k0, s_acc);
      pending = 0;
    }
    __syncthreads();
    // flush this batch's slot sums to the global gradients; the moments become
    // dL/dmean = (cx St + cy Su, cy St + cz Su) and dL/dconic = (-St.dx / 2, -St.dy, -Su.dy / 2)
    for (int t = tid; t < hi - lo; t += kThreads) {
      float* acc = &s_acc[t * kAccStride];
      const int g = __float_as_int(rec[2][t].w);
      bool any = false;
#pragma unroll
      for (int q = 0; q < 9; ++q) any |= acc[q] != 0.0f;
      const float4 r1 = rec[1][t];
      const float vx = r1.x, vy = r1.y, vz = r1.z;
      const float gmx = vx * acc[0] + vy * acc[1], gmy = vy * acc[0] + vz * acc[1];
      const float gx = -0.5f * acc[2], gy = 0.5f * -acc[3], gz = -0.5f * acc[4];
      const float ga = -(vx * vx * gx + 2.0f * vx * vy * gy + vy * vy * gz);
      const float gb = -2.0f * (vx * vy * gx + (vx * vz + vy * vy) * gy + vy * vz * gz);
      const float gc = -(vy * vy * gx + 2.0f * vy * vz * gy + vz * vz * gz);
      if (kFusedAccum && any && g >= 0 && g < p.N) {
        float4* dst = p.g_accum + 3 * (size_t)g;
        atomicAdd(dst, make_float4(gmx, gmy, ga, gb));
        atomicAdd(dst + 1, make_float4(gc, acc[8], acc[5], acc[6]));
        atomicAdd(&dst[2].x, acc[7]);
      } else if (any && g >= 0 && g < p.N) {
        atomicAdd(p.g_mean2d + 2 * g, gmx);
        atomicAdd(p.g_mean2d + 2 * g + 1, gmy);
        atomicAdd(p.g_cov2d + 3 * g, ga);
        atomicAdd(p.g_cov2d + 3 * g + 1, gb);
        atomicAdd(p.g_cov2d + 3 * g + 2, gc);
        atomicAdd(p.g_colors + 3 * g, acc[5]);
        atomicAdd(p.g_colors + 3 * g + 1, acc[6]);
        atomicAdd(p.g_colors + 3 * g + 2, acc[7]);
        atomicAdd(p.g_alpha + g, acc[8]);
      }
#pragma unroll
      for (int q = 0; q < kAccStride; ++q) acc[q] = 0.0f;
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

}  // namespace gs
