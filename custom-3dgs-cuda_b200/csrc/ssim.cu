// Fused photometric loss of the training step: L = (1 - l) * mean|x - y| + l * (1 - SSIM(x, y))
// on [H, W, 3] images, with the semantics of the reference's loss
// (gaussian_splatting/utils/loss.py:8-33: torchmetrics'
// structural_similarity_index_measure(preds = x, target = y, data_range = 1.0) on the images
// clamped to [0, 1]): an 11x11 Gaussian window (sigma 1.5), C1 = 0.01^2, C2 = 0.03^2, variances
// clamped at zero, and the SSIM map averaged over the channels and the (H - 10) x (W - 10)
// interior positions. torchmetrics reflect-pads by 5 and then crops those 5 rows and columns
// from the map, so every remaining window lies inside the image and the padding never reaches
// the result: the interior map is what is computed here. The L1 term uses the unclamped
// images and is averaged over all 3 H W values.
//
// Forward (one kernel + a one-block reduction): each CTA takes a 32x32 output tile and, one
// channel at a time, stages that channel's x and y with a 5-pixel halo in shared memory, blurs
// the five moments
// (x, y, x^2, y^2, xy) of the three channels separably (11 horizontal taps into shared memory,
// then 11 vertical taps; each thread produces a run of 8 outputs from an 18-value window held
// in registers, so a tap costs an FMA and no shared-memory load), forms the SSIM map and, per
// pixel and channel, the three derivative maps (stored planar, one plane per map and channel)
//   B  = dS/dE[x^2] = -S / (var_x + var_y + C2)
//   Cm = dS/dE[xy]  = 2 (2 mu_x mu_y + C1) / den
//   A  = dS/dmu_x - 2 mu_x B - mu_y Cm
// so that d(sum_p S_p)/dx_q = (G*A)(q) + 2 x_q (G*B)(q) + y_q (G*Cm)(q). Per-block partial sums
// of S and |x - y| (in double) are reduced in a fixed order, so the loss is deterministic.
// Backward: the same tiling, a channel at a time, blurs A, B, Cm and combines them with x,
// y and sign(x - y). One channel's planes (41 KB / 37 KB of shared memory) leave room for 5-6
// CTAs per SM.
#include <cstdlib>
#include <cstring>

#include "capi_internal.h"
#include "gs_common.cuh"
#include "tma.cuh"

namespace gs {

constexpr int kSsimTW = 32, kSsimTH = 32, kSsimR = 5, kSsimTaps = 11;
constexpr int kSsimInW = kSsimTW + 2 * kSsimR;  // 42
constexpr int kSsimInH = kSsimTH + 2 * kSsimR;  // 42
constexpr int kSsimRun = 8;                     // outputs per thread and blur pass
constexpr int kSsimWin = kSsimRun + kSsimTaps - 1;  // 18 inputs per run
constexpr int kSsimThreads = 128;
constexpr int kSsimWarps = kSsimThreads / 32;
constexpr float kSsimC1 = 0.01f * 0.01f, kSsimC2 = 0.03f * 0.03f;
static_assert(kSsimTW % kSsimRun == 0 && kSsimTH % kSsimRun == 0, "runs tile the output");
static_assert(kSsimTW * (kSsimTH / kSsimRun) == kSsimThreads,
              "one vertical run per thread and channel");
// The backward's halo box: columns bx - 8 .. bx + 39 (its start a multiple of 4 floats, as a
// tile copy's innermost coordinate must be), the 5-pixel halo starting at offset 3.
constexpr int kSsimBoxW = 48, kSsimBoxOff = 3;
static_assert(kSsimBoxOff + kSsimInW <= kSsimBoxW && (kSsimBoxOff + kSsimR) % 4 == 0,
              "the box covers the halo from a 16-byte aligned column");
constexpr unsigned kSsimBoxBytes = 3u * kSsimInH * kSsimBoxW * sizeof(float);
constexpr unsigned long long kCopyWaitNs = 1000000000ull;  // 1 s for a tile copy to land

// The 11-tap Gaussian window (sigma 1.5, normalised in double, each weight rounded to float) as
// literals, so that the blurs' FMAs take them as immediates (with the window in constant memory
// the compiler kept the weights in registers: the SSIM backward went from 96 to 77 registers
// with literals). check_gauss compares them with the formula on the host.
__host__ __device__ constexpr float gauss_w(int t) {
  const int d = t < 5 ? t : 10 - t;
  return d == 0 ? 0x1.0d956cp-10f : d == 1 ? 0x1.f1fe02p-8f : d == 2 ? 0x1.26eb18p-5f
       : d == 3 ? 0x1.bff0fep-4f : d == 4 ? 0x1.b43c4p-3f : 0x1.106562p-2f;
}

// One channel at a time: its input planes and the horizontal blurs of its 5 moments.
struct SsimForwardSmem {
  float x[kSsimInH][kSsimInW];
  float y[kSsimInH][kSsimInW];
  float h[5][kSsimInH][kSsimTW];
  double part[2][kSsimWarps];
};

// One channel at a time: its A, B, Cm planes (halo box, 128-byte aligned: a tile copy's
// destination) and their horizontal blurs.
struct __align__(128) SsimBackwardSmem {
  float m[3][kSsimInH][kSsimBoxW];
  float h[3][kSsimInH][kSsimTW];
  uint64_t bar;  // completion of the tile copies (mbarrier)
};

// out[o] = sum_t g[t] in[o + t] for a run of kSsimRun outputs (registers only).
__device__ __forceinline__ void blur_run(const float (&in)[kSsimWin], float (&out)[kSsimRun]) {
#pragma unroll
  for (int o = 0; o < kSsimRun; ++o) {
    float v = 0.f;
#pragma unroll
    for (int t = 0; t < kSsimTaps; ++t) v += gauss_w(t) * in[o + t];
    out[o] = v;
  }
}

__device__ __forceinline__ void load_row_window(const float* row, float (&w)[kSsimWin]) {
  const float2* r2 = reinterpret_cast<const float2*>(row);  // 8-byte aligned: even offsets
#pragma unroll
  for (int k = 0; k < kSsimWin / 2; ++k) {
    const float2 v = r2[k];
    w[2 * k] = v.x;
    w[2 * k + 1] = v.y;
  }
}

// The window of a run of the backward's halo box: `row` points at the run's first output
// column (16-byte aligned), the window starts kSsimBoxOff further.
__device__ __forceinline__ void load_box_window(const float* row, float (&w)[kSsimWin]) {
  const float4* r4 = reinterpret_cast<const float4*>(row);
  float v[24];
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const float4 q = r4[k];
    v[4 * k] = q.x;
    v[4 * k + 1] = q.y;
    v[4 * k + 2] = q.z;
    v[4 * k + 3] = q.w;
  }
#pragma unroll
  for (int k = 0; k < kSsimWin; ++k) w[k] = v[k + kSsimBoxOff];
}

__device__ __forceinline__ void store_run(float* dst, const float (&v)[kSsimRun]) {
  float4* d4 = reinterpret_cast<float4*>(dst);  // 16-byte aligned: offsets of 8 floats
#pragma unroll
  for (int k = 0; k < kSsimRun / 4; ++k)
    d4[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

// Derivative maps are planar, channel-major: maps[(3 * channel + kind) * H * pitch + y * pitch
// + x], kind A, B, Cm, with the row pitch W rounded up to a multiple of 4 floats (so a tile copy
// can address them, and a channel's three planes are one box); they are zero outside the
// interior (positions whose window leaves the image), so the backward's blurs of them only
// gather from interior positions.
__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }

__global__ void __launch_bounds__(kSsimThreads, 5) ssim_forward_kernel(
    int H, int W, int pitch, const float* __restrict__ img, const float* __restrict__ ref,
    float* __restrict__ maps, double* __restrict__ partials) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  SsimForwardSmem& s = *reinterpret_cast<SsimForwardSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bx = blockIdx.x * kSsimTW, by = blockIdx.y * kSsimTH;
  const int x0 = bx - kSsimR, y0 = by - kSsimR;
  const size_t plane = (size_t)H * pitch;
  // this thread's vertical run: column col, output rows [rb * 8, rb * 8 + 8)
  const int rb = tid / kSsimTW, col = tid % kSsimTW;
  const int gx = bx + col;
  double ssim_sum = 0.0, l1_sum = 0.0;
#pragma unroll 1
  for (int c = 0; c < 3; ++c) {
    // channel c of the halo rows: one warp per row, lanes along it, 6 rows in flight per warp
    {
      constexpr int kRowsPerWarp = (kSsimInH + kSsimWarps - 1) / kSsimWarps;
      constexpr int kBatch = 6;
#pragma unroll 1
      for (int r0 = 0; r0 < kRowsPerWarp; r0 += kBatch) {
        float a[kBatch][2], b[kBatch][2];
#pragma unroll
        for (int rr = 0; rr < kBatch; ++rr) {
          const int py = warp + (r0 + rr) * kSsimWarps, gy = y0 + py;
          const bool row_ok = r0 + rr < kRowsPerWarp && py < kSsimInH && gy >= 0 && gy < H;
          // channel c of the row; the lanes index it with 32-bit offsets
          const size_t row_off = row_ok ? (size_t)gy * W * 3 + c : 0;
          const float* irow = img + row_off;
          const float* rrow = ref + row_off;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int px = lane + 32 * u, gxx = x0 + px;
            const bool ok = row_ok && px < kSsimInW && (unsigned)gxx < (unsigned)W;
            a[rr][u] = ok ? clamp01(__ldg(irow + 3 * gxx)) : 0.f;
            b[rr][u] = ok ? clamp01(__ldg(rrow + 3 * gxx)) : 0.f;
          }
        }
#pragma unroll
        for (int rr = 0; rr < kBatch; ++rr) {
          const int py = warp + (r0 + rr) * kSsimWarps;
          if (r0 + rr >= kRowsPerWarp || py >= kSsimInH) break;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int px = lane + 32 * u;
            if (px < kSsimInW) {
              s.x[py][px] = a[rr][u];
              s.y[py][px] = b[rr][u];
            }
          }
        }
      }
    }
    __syncthreads();
    // horizontal: runs of 8 outputs of the 5 moments
    for (int it = tid; it < kSsimInH * (kSsimTW / kSsimRun); it += kSsimThreads) {
      const int r = it / (kSsimTW / kSsimRun), cb = it - r * (kSsimTW / kSsimRun);
      float xa[kSsimWin], ya[kSsimWin], w[kSsimWin], out[kSsimRun];
      load_row_window(&s.x[r][cb * kSsimRun], xa);
      load_row_window(&s.y[r][cb * kSsimRun], ya);
      blur_run(xa, out);
      store_run(&s.h[0][r][cb * kSsimRun], out);
      blur_run(ya, out);
      store_run(&s.h[1][r][cb * kSsimRun], out);
#pragma unroll
      for (int k = 0; k < kSsimWin; ++k) w[k] = xa[k] * xa[k];
      blur_run(w, out);
      store_run(&s.h[2][r][cb * kSsimRun], out);
#pragma unroll
      for (int k = 0; k < kSsimWin; ++k) w[k] = ya[k] * ya[k];
      blur_run(w, out);
      store_run(&s.h[3][r][cb * kSsimRun], out);
#pragma unroll
      for (int k = 0; k < kSsimWin; ++k) w[k] = xa[k] * ya[k];
      blur_run(w, out);
      store_run(&s.h[4][r][cb * kSsimRun], out);
    }
    __syncthreads();
    // vertical run, SSIM and its derivative maps
    {
      float m[5][kSsimRun];
#pragma unroll
      for (int q = 0; q < 5; ++q) {
        float v[kSsimWin];
#pragma unroll
        for (int k = 0; k < kSsimWin; ++k) v[k] = s.h[q][rb * kSsimRun + k][col];
        blur_run(v, m[q]);
      }
      float run_ssim = 0.f, run_l1 = 0.f;  // at most 8 terms each; summed in double below
#pragma unroll
      for (int o = 0; o < kSsimRun; ++o) {
        const int r = rb * kSsimRun + o, gy = by + r;
        if (gx >= W || gy >= H) continue;
        const size_t pix = (size_t)gy * W + gx;
        const bool interior = gx >= kSsimR && gx < W - kSsimR && gy >= kSsimR && gy < H - kSsimR;
        float A = 0.f, B = 0.f, Cm = 0.f;
        if (interior) {
          const float mx = m[0][o], my = m[1][o];
          const float vx_raw = m[2][o] - mx * mx, vy_raw = m[3][o] - my * my;
          const float vx = fmaxf(vx_raw, 0.f), vy = fmaxf(vy_raw, 0.f), cxy = m[4][o] - mx * my;
          const float n1 = 2.f * mx * my + kSsimC1, n2 = 2.f * cxy + kSsimC2;
          const float d1 = mx * mx + my * my + kSsimC1, d2 = vx + vy + kSsimC2;
          // one reciprocal: 1/den, 1/d1 = d2/den, 1/d2 = d1/den
          const float rden = 1.0f / (d1 * d2);
          const float S = n1 * n2 * rden;
          // the clamp of var_x at zero passes no gradient where it is active
          B = vx_raw >= 0.f ? -S * (d1 * rden) : 0.f;
          Cm = 2.f * n1 * rden;
          const float dmx = 2.f * my * n2 * rden - 2.f * mx * S * (d2 * rden);
          A = dmx - 2.f * mx * B - my * Cm;
          run_ssim += S;
        }
        const size_t mp = (size_t)(3 * c) * plane + (size_t)gy * pitch + gx;
        maps[mp] = A;
        maps[mp + plane] = B;
        maps[mp + 2 * plane] = Cm;
        const size_t p3 = pix * 3 + c;
        run_l1 += fabsf(__ldg(img + p3) - __ldg(ref + p3));
      }
      ssim_sum += (double)run_ssim;
      l1_sum += (double)run_l1;
    }
    __syncthreads();  // the next channel overwrites the planes
  }
  // block reduction in a fixed order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ssim_sum += __shfl_xor_sync(0xffffffffu, ssim_sum, o);
    l1_sum += __shfl_xor_sync(0xffffffffu, l1_sum, o);
  }
  if (lane == 0) {
    s.part[0][warp] = ssim_sum;
    s.part[1][warp] = l1_sum;
  }
  __syncthreads();
  if (tid == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kSsimWarps; ++w) {
      a += s.part[0][w];
      b += s.part[1][w];
    }
    const size_t blk = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    partials[2 * blk] = a;
    partials[2 * blk + 1] = b;
  }
}

__global__ void __launch_bounds__(256) ssim_finalize_kernel(const double* __restrict__ partials,
                                                            int nblocks, double n_ssim,
                                                            double n_l1, float lambda,
                                                            float* __restrict__ loss,
                                                            float* __restrict__ ssim_out) {
  __shared__ double s_a[256], s_b[256];
  double a = 0.0, b = 0.0;
  for (int i = threadIdx.x; i < nblocks; i += 256) {
    a += partials[2 * i];
    b += partials[2 * i + 1];
  }
  s_a[threadIdx.x] = a;
  s_b[threadIdx.x] = b;
  __syncthreads();
  for (int st = 128; st > 0; st >>= 1) {
    if (threadIdx.x < st) {
      s_a[threadIdx.x] += s_a[threadIdx.x + st];
      s_b[threadIdx.x] += s_b[threadIdx.x + st];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double ssim = s_a[0] / n_ssim, l1 = s_b[0] / n_l1;
    *loss = (float)((1.0 - lambda) * l1 + lambda * (1.0 - ssim));
    if (ssim_out) *ssim_out = (float)ssim;
  }
}

// Backward, one channel at a time: the channel's A, B, Cm planes over the tile and its 5-pixel
// halo arrive in s.m (columns bx - 8 .. bx + 39: the copy's start column must be a multiple of
// 4 floats, so the halo's first column sits at offset kSsimBoxOff), are blurred horizontally
// into s.h, then vertically per thread run, and combined with x, y and sign(x - y). kTma: one
// tensor-memory-accelerator copy of the three planes per channel (they are adjacent in the map
// layout), issued by thread 0 as soon as the previous channel's horizontal pass has read s.m,
// so it overlaps that channel's vertical pass; otherwise the warps load the planes themselves.
template <bool kTma>
__global__ void __launch_bounds__(kSsimThreads, 5) ssim_backward_kernel(
    int H, int W, int pitch, const float* __restrict__ img, const float* __restrict__ ref,
    const float* __restrict__ maps, const __grid_constant__ CUtensorMap map_desc,
    const float* __restrict__ grad_loss, float lambda, float inv_n_l1, float inv_n_ssim,
    float* __restrict__ grad_img) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  SsimBackwardSmem& s = *reinterpret_cast<SsimBackwardSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bx = blockIdx.x * kSsimTW, by = blockIdx.y * kSsimTH;
  const int x0 = bx - kSsimBoxOff - kSsimR, y0 = by - kSsimR;  // box origin
  const size_t plane = (size_t)H * pitch;
  const float g = __ldg(grad_loss);
  const float w_l1 = g * (1.0f - lambda) * inv_n_l1, w_ssim = -g * lambda * inv_n_ssim;
  const int rb = tid / kSsimTW, col = tid % kSsimTW;
  const int gx = bx + col;
  bool copies_ok = true;
  if (kTma) {
    if (tid == 0) {
      mbar_init(&s.bar, 1);
      mbar_arrive_expect_tx(&s.bar, kSsimBoxBytes);
      tma_load_3d(&s.m[0][0][0], &map_desc, x0, y0, 0, &s.bar);
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
  }
#pragma unroll 1
  for (int c = 0; c < 3; ++c) {
    if (kTma) {
      if (!mbar_wait(&s.bar, (unsigned)(c & 1), kCopyWaitNs)) copies_ok = false;
    } else {
      // planes A_c, B_c, Cm_c: one warp per halo row, lanes along it (48 columns)
      const float* chan = maps + (size_t)(3 * c) * plane;
#pragma unroll 1
      for (int row = warp; row < 3 * kSsimInH; row += kSsimWarps) {
        const int kind = row / kSsimInH, py = row - kind * kSsimInH, gy = y0 + py;
        const float* src = chan + (size_t)kind * plane + (size_t)gy * pitch;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int px = lane + 32 * u, gxx = x0 + px;
          if (px < kSsimBoxW)
            s.m[kind][py][px] = (gy >= 0 && gy < H && gxx >= 0 && gxx < W) ? __ldg(src + gxx)
                                                                           : 0.f;
        }
      }
      __syncthreads();
    }
    for (int it = tid; it < 3 * kSsimInH * (kSsimTW / kSsimRun); it += kSsimThreads) {
      const int kind = it / (kSsimInH * (kSsimTW / kSsimRun));
      const int rem = it - kind * (kSsimInH * (kSsimTW / kSsimRun));
      const int r = rem / (kSsimTW / kSsimRun), cb = rem - r * (kSsimTW / kSsimRun);
      float w[kSsimWin], out[kSsimRun];
      load_box_window(&s.m[kind][r][cb * kSsimRun], w);
      blur_run(w, out);
      store_run(&s.h[kind][r][cb * kSsimRun], out);
    }
    __syncthreads();
    if (kTma && tid == 0 && c < 2) {  // s.m is free: the next channel's planes
      mbar_arrive_expect_tx(&s.bar, kSsimBoxBytes);
      tma_load_3d(&s.m[0][0][0], &map_desc, x0, y0, 3 * (c + 1), &s.bar);
    }
    float bl[3][kSsimRun];
#pragma unroll
    for (int kind = 0; kind < 3; ++kind) {
      float v[kSsimWin];
#pragma unroll
      for (int k = 0; k < kSsimWin; ++k) v[k] = s.h[kind][rb * kSsimRun + k][col];
      blur_run(v, bl[kind]);
    }
#pragma unroll
    for (int o = 0; o < kSsimRun; ++o) {
      const int gy = by + rb * kSsimRun + o;
      if (gx >= W || gy >= H) continue;
      const size_t p = ((size_t)gy * W + gx) * 3 + c;
      const float xr = __ldg(img + p), yr = __ldg(ref + p);
      const float d = xr - yr;
      const float sgn = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
      // SSIM sees the clamped images; the clamp passes the gradient where 0 <= x <= 1
      const float xv = clamp01(xr), yv = clamp01(yr);
      const float gs = (xr >= 0.f && xr <= 1.f)
                           ? w_ssim * (bl[0][o] + 2.f * xv * bl[1][o] + yv * bl[2][o])
                           : 0.f;
      grad_img[p] = w_l1 * sgn + gs;
    }
    __syncthreads();  // the next channel overwrites s.h (and, without kTma, s.m)
  }
  if (kTma && !copies_ok) {
    raise_device_error(kErrCopyTimeout);
    // no copy may still be landing in this CTA's shared memory when it exits
    if (tid == 0) mbar_wait(&s.bar, 0u, kCopyWaitNs);
  }
}

// The window's literals (gauss_w) against its formula: exp(-x^2 / (2 sigma^2)) in double for
// x = -5..5, each rounded to float, normalised by their double sum and rounded again.
static int check_gauss() {
  static const bool ok = [] {
    float w[kSsimTaps];
    double sum = 0.0;
    for (int k = 0; k < kSsimTaps; ++k) {
      const double x = k - (kSsimTaps - 1) / 2.0;
      sum += w[k] = (float)exp(-(x * x) / (2.0 * 1.5 * 1.5));
    }
    bool same = true;
    for (int k = 0; k < kSsimTaps; ++k) same = same && (float)(w[k] / sum) == gauss_w(k);
    return same;
  }();
  GS_REQUIRE(ok, "SSIM window literals differ from the Gaussian formula");
  return GS_OK;
}

static size_t ssim_blocks(int H, int W) {
  return (size_t)((W + kSsimTW - 1) / kSsimTW) * ((H + kSsimTH - 1) / kSsimTH);
}

// Workspace: the derivative maps (row pitch W rounded up to 4 floats) from the first 256-byte
// boundary, then the per-block partial sums.
static int map_pitch(int W) { return (W + 3) & ~3; }
static size_t maps_bytes(int H, int W) { return (size_t)H * map_pitch(W) * 9 * sizeof(float); }
static float* maps_of(const void* workspace) {
  return reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255u) &
                                  ~uintptr_t(255u));
}
static double* partials_of(const void* workspace, int H, int W) {
  return reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(maps_of(workspace)) + maps_bytes(H, W) + 255u) &
      ~uintptr_t(255u));
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_l1_ssim_workspace_size(int H, int W) {
  if (H <= 0 || W <= 0) return 0;
  return 256 + maps_bytes(H, W) + 256 + ssim_blocks(H, W) * 2 * sizeof(double);
}

static double ssim_count(int H, int W) { return 3.0 * (H - 2 * kSsimR) * (W - 2 * kSsimR); }

extern "C" int gs_l1_ssim_forward(int H, int W, const float* img, const float* target,
                                  float lambda_dssim, void* workspace, size_t workspace_bytes,
                                  float* loss, float* ssim_value, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(H > 2 * kSsimR && W > 2 * kSsimR,
             "SSIM needs images of at least 11 x 11 pixels (an 11 x 11 window inside the image)");
  GS_REQUIRE(img && target && workspace && loss, "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_l1_ssim_workspace_size(H, W), "workspace too small");
  const int rc = check_gauss();
  if (rc != GS_OK) return rc;
  float* maps = maps_of(workspace);
  double* partials = partials_of(workspace, H, W);
  const dim3 grid((W + kSsimTW - 1) / kSsimTW, (H + kSsimTH - 1) / kSsimTH);
  const size_t smem = sizeof(SsimForwardSmem);
  GS_CUDA(cudaFuncSetAttribute(ssim_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  cudaStream_t st = (cudaStream_t)stream;
  ssim_forward_kernel<<<grid, kSsimThreads, smem, st>>>(H, W, map_pitch(W), img, target, maps,
                                                        partials);
  GS_CHECK_LAUNCH();
  ssim_finalize_kernel<<<1, 256, 0, st>>>(partials, (int)(grid.x * grid.y), ssim_count(H, W),
                                          (double)H * W * 3, lambda_dssim, loss, ssim_value);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_l1_ssim_backward(int H, int W, const float* img, const float* target,
                                   float lambda_dssim, const void* workspace,
                                   size_t workspace_bytes, const float* grad_loss,
                                   float* grad_img, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(H > 2 * kSsimR && W > 2 * kSsimR,
             "SSIM needs images of at least 11 x 11 pixels (an 11 x 11 window inside the image)");
  GS_REQUIRE(img && target && workspace && grad_loss && grad_img, "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_l1_ssim_workspace_size(H, W), "workspace too small");
  const int rc = check_gauss();
  if (rc != GS_OK) return rc;
  const dim3 grid((W + kSsimTW - 1) / kSsimTW, (H + kSsimTH - 1) / kSsimTH);
  const size_t smem = sizeof(SsimBackwardSmem);
  const float* maps = maps_of(workspace);
  const int pitch = map_pitch(W);
  // the channel's three planes as one tile copy where the driver can describe them;
  // GS3D_SSIM_NO_TMA=1 selects the warps' own loads (same results), which tests compare
  CUtensorMap desc;
  std::memset(&desc, 0, sizeof(desc));
  const char* no_tma = std::getenv("GS3D_SSIM_NO_TMA");
  const bool tma = !(no_tma && no_tma[0] == '1') &&
                   encode_f32_3d(&desc, maps, (uint64_t)W, (uint64_t)H, 9, (uint64_t)pitch,
                                 (uint64_t)H * pitch, kSsimBoxW, kSsimInH, 3);
  const float inv_n_l1 = (float)(1.0 / ((double)H * W * 3));
  const float inv_n_ssim = (float)(1.0 / ssim_count(H, W));
  cudaStream_t st = (cudaStream_t)stream;
  if (tma) {
    GS_CUDA(cudaFuncSetAttribute(ssim_backward_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ssim_backward_kernel<true><<<grid, kSsimThreads, smem, st>>>(
        H, W, pitch, img, target, maps, desc, grad_loss, lambda_dssim, inv_n_l1, inv_n_ssim,
        grad_img);
  } else {
    GS_CUDA(cudaFuncSetAttribute(ssim_backward_kernel<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ssim_backward_kernel<false><<<grid, kSsimThreads, smem, st>>>(
        H, W, pitch, img, target, maps, desc, grad_loss, lambda_dssim, inv_n_l1, inv_n_ssim,
        grad_img);
  }
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
