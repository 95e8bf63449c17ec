// Shared device helpers for the sm_100a Gaussian-splatting kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gs {

constexpr int kTileSide = 16;                     // 16 x 16 pixel tiles
constexpr int kTilePixels = kTileSide * kTileSide;

// Device error bits (OR-ed into g_device_errors by the kernels).
constexpr unsigned kErrLookbackTimeout = 1u;  // a decoupled look-back wait hit its limit
constexpr unsigned kErrCapacity = 2u;         // pair count exceeded the pair capacity
constexpr unsigned kErrBadIndex = 4u;         // an index was out of range
constexpr unsigned kErrPeerTimeout = 8u;      // a cross-GPU barrier wait hit its limit
constexpr unsigned kErrCopyTimeout = 16u;     // a wait for a tensor-memory-accelerator copy hit its limit

// Iteration limit of every spin-wait. Each iteration is one L2 round trip plus a short
// sleep, so the limit bounds a wait to well under a second.
constexpr unsigned kSpinLimit = 1u << 20;

// Real spherical-harmonic normalisation constants for degrees 0..3 (the Inria 3DGS basis;
// the reference lists them at csrc/forward/SH.cu:12-28).
constexpr float kShC0 = 0.28209479177387814f;
constexpr float kShC1 = 0.4886025119029199f;
constexpr float kShC2_0 = 1.0925484305920792f;
constexpr float kShC2_1 = -1.0925484305920792f;
constexpr float kShC2_2 = 0.31539156525252005f;
constexpr float kShC2_3 = -1.0925484305920792f;
constexpr float kShC2_4 = 0.5462742152960396f;
constexpr float kShC3_0 = -0.5900435899266435f;
constexpr float kShC3_1 = 2.890611442640554f;
constexpr float kShC3_2 = -0.4570457994644658f;
constexpr float kShC3_3 = 0.3731763325901154f;
constexpr float kShC3_4 = -0.4570457994644658f;
constexpr float kShC3_5 = 1.445305721320277f;
constexpr float kShC3_6 = -0.5900435899266435f;

extern __device__ unsigned g_device_errors;

__device__ __forceinline__ void raise_device_error(unsigned bits) {
  atomicOr(&g_device_errors, bits);
}

// ---------------------------------------------------------------------------------------
// Tile footprint of one splat. The arithmetic follows the reference's count_overlaps /
// key_generation (csrc/forward/rasterize.cu:27-57): a 3-sigma radius from the larger
// eigenvalue of the 2x2 covariance, a pixel bounding box clamped to the image, and the
// 16x16 tile rectangle [x0,x1) x [y0,y1). The expressions are written as the reference
// writes them so that nvcc contracts them into the same fused multiply-adds.
// ---------------------------------------------------------------------------------------
struct TileRect {
  int x0, y0, x1, y1;
};

// Written with explicit round-to-nearest intrinsics in the form nvcc gives the reference's
// source under its default --fmad=true (a * c - b * b -> fma(a, c, -(b * b)), and so on), so the
// rounding cannot change with the surrounding code.
__device__ __forceinline__ float cov_det(float a, float b, float c) {
  return __fmaf_rn(a, c, -__fmul_rn(b, b));
}

__device__ __forceinline__ bool splat_tile_rect(float2 mean, float a, float b, float c,
                                                int width, int height, int tiles_x,
                                                int tiles_y, TileRect& r) {
  const float det = cov_det(a, b, c);
  if (det <= 0.0f) return false;
  const float mid = __fmul_rn(0.5f, __fadd_rn(a, c));
  const float lambda_max = __fadd_rn(mid, __fsqrt_rn(fmaxf(0.1f, __fmaf_rn(mid, mid, -det))));
  const float radius = ceilf(__fmul_rn(3.0f, __fsqrt_rn(lambda_max)));
  int min_x = max(0, (int)floorf(__fsub_rn(mean.x, radius)));
  int max_x = min(width, (int)ceilf(__fadd_rn(mean.x, radius)));
  int min_y = max(0, (int)floorf(__fsub_rn(mean.y, radius)));
  int max_y = min(height, (int)ceilf(__fadd_rn(mean.y, radius)));
  int tx0 = min_x / kTileSide, tx1 = (max_x + kTileSide - 1) / kTileSide;
  int ty0 = min_y / kTileSide, ty1 = (max_y + kTileSide - 1) / kTileSide;
  r.x0 = max(0, min(tiles_x, tx0));
  r.x1 = max(0, min(tiles_x, tx1));
  r.y0 = max(0, min(tiles_y, ty0));
  r.y1 = max(0, min(tiles_y, ty1));
  return true;
}

__device__ __forceinline__ int rect_count(const TileRect& r) {
  return max(0, r.x1 - r.x0) * max(0, r.y1 - r.y0);
}

// Conic (inverse 2D covariance) with the reference's guard det <= 0 -> 0
// (csrc/forward/rasterize.cu:224-232).
__device__ __forceinline__ float3 conic_from_cov(float a, float b, float c) {
  const float det = cov_det(a, b, c);
  const float det_inv = (det > 0.0f) ? __fdiv_rn(1.0f, det) : 0.0f;
  return make_float3(__fmul_rn(c, det_inv), __fmul_rn(-b, det_inv), __fmul_rn(a, det_inv));
}

// Conservative half-extents (hx, hy) of the screen region where a splat can pass the blend's
// opacity test, o * exp(-0.5 d^T Q d) >= 1/255, i.e. d^T Q d <= 2 ln(255 o): the axis-aligned
// bounding box of that ellipse (half-widths sqrt(r^2 (Q^-1)_xx), sqrt(r^2 (Q^-1)_yy), with Q^-1
// formed in double from the float conic) inflated by 1% in r^2 and 0.5 px. Pixels outside the
// box fail the test for certain, so a warp whose pixels all lie outside may skip the splat
// without changing any result. A splat that can never pass gets -inf; a conic whose inverse
// cannot be formed gets +inf (never skipped).
__device__ __forceinline__ float2 splat_extent(float3 conic, float opacity) {
  const double r2_base = 2.0 * log(255.0 * (double)opacity);
  if (!(opacity > 0.0f) || r2_base < -1e-3) return make_float2(-INFINITY, -INFINITY);
  const double qx = conic.x, qy = conic.y, qz = conic.z;
  const double det = qx * qz - qy * qy;
  if (!(det > 0.0) || !(qx > 0.0) || !(qz > 0.0)) return make_float2(INFINITY, INFINITY);
  const double r2 = fmax(r2_base, 0.0) * 1.01 + 1e-3;
  const double hx = sqrt(r2 * qz / det) + 0.5, hy = sqrt(r2 * qx / det) + 0.5;
  return make_float2((float)hx, (float)hy);
}

// Gaussian falloff exponent of a pixel offset (dx, dy) under a conic:
// -0.5 (q.x dx dx + 2 q.y dx dy + q.z dy dy) (csrc/forward/rasterize.cu:249-251), evaluated as
// nvcc contracts that source: -0.5 * fma(q.z dy, dy, fma(q.x dx, dx, ((2 q.y) dx) dy)).
__device__ __forceinline__ float splat_power(float3 conic, float dx, float dy) {
  const float cross = __fmul_rn(__fmul_rn(__fmul_rn(2.0f, conic.y), dx), dy);
  const float s1 = __fmaf_rn(__fmul_rn(conic.x, dx), dx, cross);
  const float s = __fmaf_rn(__fmul_rn(conic.z, dy), dy, s1);
  return __fmul_rn(-0.5f, s);
}

// One front-to-back blend step of a pixel (csrc/forward/rasterize.cu:260-264): the colour gains
// c * (alpha T) and T becomes T (1 - alpha), with nvcc's contraction of the reference source.
__device__ __forceinline__ void blend_step(float alpha, float4 col, float& T, float& r,
                                           float& g, float& b) {
  const float weight = __fmul_rn(alpha, T);
  r = __fmaf_rn(col.x, weight, r);
  g = __fmaf_rn(col.y, weight, g);
  b = __fmaf_rn(col.z, weight, b);
  T = __fmul_rn(T, __fsub_rn(1.0f, alpha));
}

// ---------------------------------------------------------------------------------------
// Decoupled look-back status words: bits [31:30] = flag, bits [29:0] = value.
// ---------------------------------------------------------------------------------------
// Initial value of both words of a tile range before the final tile-sort pass fills it in:
// the byte pattern 0x7f, above any pair index.
constexpr int kRangeUnset = 0x7f7f7f7f;

constexpr unsigned kFlagAggregate = 1u << 30;
constexpr unsigned kFlagPrefix = 2u << 30;
constexpr unsigned kFlagMask = 3u << 30;
constexpr unsigned kValueMask = (1u << 30) - 1u;

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits (bounded) until the status word is published; returns the word, or kFlagPrefix|0
// after raising kErrLookbackTimeout.
__device__ __forceinline__ unsigned wait_status(const unsigned* p) {
  unsigned v = ld_relaxed(p);
  unsigned spins = 0;
  while ((v & kFlagMask) == 0u) {
    if (++spins > kSpinLimit) {
      raise_device_error(kErrLookbackTimeout);
      return kFlagPrefix;
    }
    __nanosleep(64);
    v = ld_relaxed(p);
  }
  return v;
}

// Single-thread look-back: exclusive prefix of `tile` from the status words of its
// predecessors (status[0..tile-1]); each status word is strided by `stride` words. The
// predecessors are read kLookbackBatch at a time (independent loads in flight together), then
// consumed nearest first until one carries an inclusive prefix: when every tile of a pass runs
// at once, a tile's walk back to the nearest prefix is long, and one dependent L2 round trip per
// predecessor made the walk, not the data, set the pass's time.
constexpr int kLookbackBatch = 8;

__device__ __forceinline__ unsigned lookback_serial(const unsigned* status, int tile,
                                                    int stride) {
  unsigned excl = 0;
  for (int base = tile - 1; base >= 0; base -= kLookbackBatch) {
    unsigned v[kLookbackBatch];
#pragma unroll
    for (int k = 0; k < kLookbackBatch; ++k)
      v[k] = base - k >= 0 ? ld_relaxed(status + (size_t)(base - k) * stride) : kFlagPrefix;
    bool done = false;
#pragma unroll
    for (int k = 0; k < kLookbackBatch; ++k) {
      if (done) continue;
      unsigned w = v[k];
      if ((w & kFlagMask) == 0u) w = wait_status(status + (size_t)(base - k) * stride);
      excl += w & kValueMask;
      done = (w & kFlagPrefix) != 0u;
    }
    if (done) break;
  }
  return excl;
}

// Warp-cooperative look-back for a single counter per tile (status stride 1). All 32 lanes
// call it; every lane returns the exclusive prefix.
__device__ __forceinline__ unsigned lookback_warp(const unsigned* status, int tile) {
  const int lane = threadIdx.x & 31;
  unsigned excl = 0;
  int base = tile - 1;
  while (base >= 0) {
    int p = base - lane;
    unsigned v = kFlagPrefix;  // lanes past tile 0 act as a zero prefix
    if (p >= 0) v = wait_status(status + p);
    unsigned prefix_mask = __ballot_sync(0xffffffffu, (v & kFlagPrefix) != 0u);
    // lanes up to and including the first (nearest) prefix contribute
    int stop = prefix_mask ? (__ffs(prefix_mask) - 1) : 31;
    unsigned contrib = (lane <= stop && p >= 0) ? (v & kValueMask) : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
    excl += contrib;
    if (prefix_mask) break;
    base -= 32;
  }
  return excl;
}

// Block-wide exclusive scan of one unsigned per thread (blockDim.x a multiple of 32,
// <= 1024). `smem` holds at least 33 words. Returns the exclusive prefix; *total gets the
// block sum.
__device__ __forceinline__ unsigned block_exclusive_scan(unsigned v, unsigned* smem,
                                                         unsigned* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) smem[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    unsigned w = lane < nwarps ? smem[lane] : 0u;
    unsigned wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      unsigned n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < nwarps) smem[lane] = wi - w;  // exclusive per warp
    if (lane == nwarps - 1) smem[32] = wi;   // block total
  }
  __syncthreads();
  unsigned excl = smem[warp] + incl - v;
  *total = smem[32];
  __syncthreads();
  return excl;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace gs
