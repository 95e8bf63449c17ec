// Fused photometric loss of the training step: L = (1 - l) * mean|x - y| + l * (1 - SSIM(x, y))
// on [H, W, 3] images, SSIM with an 11x11 Gaussian window (sigma 1.5, zero padding,
// C1 = 0.01^2, C2 = 0.03^2), averaged over pixels and channels.
//
// Forward (one kernel + a one-block reduction): each CTA stages a 32x16 output tile plus a
// 5-pixel halo of x and y in shared memory, blurs the five moments (x, y, x^2, y^2, xy) of the
// three channels separably (11 horizontal taps into shared memory, then 11 vertical taps),
// forms the SSIM map and, per pixel and channel, the three derivative maps
//   B  = dS/dE[x^2] = -S / (var_x + var_y + C2)
//   Cm = dS/dE[xy]  = 2 (2 mu_x mu_y + C1) / den
//   A  = dS/dmu_x - 2 mu_x B - mu_y Cm
// so that d(sum_p S_p)/dx_q = (G*A)(q) + 2 x_q (G*B)(q) + y_q (G*Cm)(q). Per-block partial sums
// of S and |x - y| (in double) are reduced in a fixed order, so the loss is deterministic.
// Backward: the same tiling blurs A, B, Cm and combines them with x, y and sign(x - y).
#include "capi_internal.h"
#include "gs_common.cuh"

namespace gs {

constexpr int kSsimTW = 32, kSsimTH = 16, kSsimR = 5, kSsimTaps = 11;
constexpr int kSsimInW = kSsimTW + 2 * kSsimR;  // 42
constexpr int kSsimInH = kSsimTH + 2 * kSsimR;  // 26
constexpr int kSsimThreads = 256;
constexpr float kSsimC1 = 0.01f * 0.01f, kSsimC2 = 0.03f * 0.03f;

__constant__ float c_gauss[kSsimTaps];

struct SsimForwardSmem {
  float x[kSsimInH][kSsimInW][3];
  float y[kSsimInH][kSsimInW][3];
  float h[15][kSsimInH][kSsimTW];  // horizontal blurs: 5 moments x 3 channels
  double part[2][kSsimThreads / 32];
};

struct SsimBackwardSmem {
  float m[kSsimInH][kSsimInW][9];  // A, B, Cm x 3 channels
  float h[9][kSsimInH][kSsimTW];
};

__device__ __forceinline__ float load_px(const float* img, int W, int H, int x, int y, int c) {
  return (x >= 0 && x < W && y >= 0 && y < H) ? __ldg(img + ((size_t)y * W + x) * 3 + c) : 0.0f;
}

__global__ void __launch_bounds__(kSsimThreads) ssim_forward_kernel(
    int H, int W, const float* __restrict__ img, const float* __restrict__ ref,
    float* __restrict__ maps, double* __restrict__ partials) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SsimForwardSmem& s = *reinterpret_cast<SsimForwardSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kSsimTW - kSsimR, y0 = blockIdx.y * kSsimTH - kSsimR;
  for (int i = tid; i < kSsimInH * kSsimInW * 3; i += kSsimThreads) {
    const int c = i % 3, px = (i / 3) % kSsimInW, py = i / (3 * kSsimInW);
    s.x[py][px][c] = load_px(img, W, H, x0 + px, y0 + py, c);
    s.y[py][px][c] = load_px(ref, W, H, x0 + px, y0 + py, c);
  }
  __syncthreads();
  for (int i = tid; i < kSsimInH * kSsimTW; i += kSsimThreads) {
    const int r = i / kSsimTW, col = i % kSsimTW;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float mx = 0.f, my = 0.f, xx = 0.f, yy = 0.f, xy = 0.f;
#pragma unroll
      for (int k = 0; k < kSsimTaps; ++k) {
        const float g = c_gauss[k], a = s.x[r][col + k][c], b = s.y[r][col + k][c];
        mx += g * a;
        my += g * b;
        xx += g * (a * a);
        yy += g * (b * b);
        xy += g * (a * b);
      }
      s.h[c * 5 + 0][r][col] = mx;
      s.h[c * 5 + 1][r][col] = my;
      s.h[c * 5 + 2][r][col] = xx;
      s.h[c * 5 + 3][r][col] = yy;
      s.h[c * 5 + 4][r][col] = xy;
    }
  }
  __syncthreads();
  double ssim_sum = 0.0, l1_sum = 0.0;
  for (int i = tid; i < kSsimTH * kSsimTW; i += kSsimThreads) {
    const int oy = i / kSsimTW, ox = i % kSsimTW;
    const int gx = blockIdx.x * kSsimTW + ox, gy = blockIdx.y * kSsimTH + oy;
    if (gx >= W || gy >= H) continue;
    float out[9];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float m[5];
#pragma unroll
      for (int q = 0; q < 5; ++q) {
        float v = 0.f;
#pragma unroll
        for (int k = 0; k < kSsimTaps; ++k) v += c_gauss[k] * s.h[c * 5 + q][oy + k][ox];
        m[q] = v;
      }
      const float mx = m[0], my = m[1];
      const float vx = m[2] - mx * mx, vy = m[3] - my * my, cxy = m[4] - mx * my;
      const float n1 = 2.f * mx * my + kSsimC1, n2 = 2.f * cxy + kSsimC2;
      const float d1 = mx * mx + my * my + kSsimC1, d2 = vx + vy + kSsimC2;
      const float den = d1 * d2;
      const float S = (n1 * n2) / den;
      const float B = -S / d2;
      const float Cm = 2.f * n1 / den;
      const float dmx = (2.f * my * n2) / den - S * (2.f * mx) / d1;
      const float A = dmx - 2.f * mx * B - my * Cm;
      out[c] = A;
      out[3 + c] = B;
      out[6 + c] = Cm;
      ssim_sum += (double)S;
      const float xv = s.x[oy + kSsimR][ox + kSsimR][c], yv = s.y[oy + kSsimR][ox + kSsimR][c];
      l1_sum += (double)fabsf(xv - yv);
    }
    float* dst = maps + ((size_t)gy * W + gx) * 9;
#pragma unroll
    for (int q = 0; q < 9; ++q) dst[q] = out[q];
  }
  // block reduction in a fixed order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ssim_sum += __shfl_xor_sync(0xffffffffu, ssim_sum, o);
    l1_sum += __shfl_xor_sync(0xffffffffu, l1_sum, o);
  }
  if ((tid & 31) == 0) {
    s.part[0][tid >> 5] = ssim_sum;
    s.part[1][tid >> 5] = l1_sum;
  }
  __syncthreads();
  if (tid == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kSsimThreads / 32; ++w) {
      a += s.part[0][w];
      b += s.part[1][w];
    }
    const size_t blk = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    partials[2 * blk] = a;
    partials[2 * blk + 1] = b;
  }
}

__global__ void __launch_bounds__(256) ssim_finalize_kernel(const double* __restrict__ partials,
                                                            int nblocks, double n, float lambda,
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
    const double ssim = s_a[0] / n, l1 = s_b[0] / n;
    *loss = (float)((1.0 - lambda) * l1 + lambda * (1.0 - ssim));
    if (ssim_out) *ssim_out = (float)ssim;
  }
}

__global__ void __launch_bounds__(kSsimThreads) ssim_backward_kernel(
    int H, int W, const float* __restrict__ img, const float* __restrict__ ref,
    const float* __restrict__ maps, const float* __restrict__ grad_loss, float lambda,
    float inv_n, float* __restrict__ grad_img) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SsimBackwardSmem& s = *reinterpret_cast<SsimBackwardSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kSsimTW - kSsimR, y0 = blockIdx.y * kSsimTH - kSsimR;
  for (int i = tid; i < kSsimInH * kSsimInW * 9; i += kSsimThreads) {
    const int q = i % 9, px = (i / 9) % kSsimInW, py = i / (9 * kSsimInW);
    const int gx = x0 + px, gy = y0 + py;
    s.m[py][px][q] =
        (gx >= 0 && gx < W && gy >= 0 && gy < H) ? __ldg(maps + ((size_t)gy * W + gx) * 9 + q) : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < kSsimInH * kSsimTW; i += kSsimThreads) {
    const int r = i / kSsimTW, col = i % kSsimTW;
#pragma unroll
    for (int q = 0; q < 9; ++q) {
      float v = 0.f;
#pragma unroll
      for (int k = 0; k < kSsimTaps; ++k) v += c_gauss[k] * s.m[r][col + k][q];
      s.h[q][r][col] = v;
    }
  }
  __syncthreads();
  const float g = __ldg(grad_loss);
  const float w_l1 = g * (1.0f - lambda) * inv_n, w_ssim = -g * lambda * inv_n;
  for (int i = tid; i < kSsimTH * kSsimTW; i += kSsimThreads) {
    const int oy = i / kSsimTW, ox = i % kSsimTW;
    const int gx = blockIdx.x * kSsimTW + ox, gy = blockIdx.y * kSsimTH + oy;
    if (gx >= W || gy >= H) continue;
    const size_t p = ((size_t)gy * W + gx) * 3;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float bA = 0.f, bB = 0.f, bC = 0.f;
#pragma unroll
      for (int k = 0; k < kSsimTaps; ++k) {
        const float gk = c_gauss[k];
        bA += gk * s.h[c][oy + k][ox];
        bB += gk * s.h[3 + c][oy + k][ox];
        bC += gk * s.h[6 + c][oy + k][ox];
      }
      const float xv = __ldg(img + p + c), yv = __ldg(ref + p + c);
      const float d = xv - yv;
      const float sgn = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
      grad_img[p + c] = w_l1 * sgn + w_ssim * (bA + 2.f * xv * bB + yv * bC);
    }
  }
}

// The window lives in per-device constant memory; it is uploaded once per device.
static int g_gauss_ready[64] = {};

static int ensure_gauss() {
  int dev = 0;
  GS_CUDA(cudaGetDevice(&dev));
  GS_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range");
  if (g_gauss_ready[dev]) return GS_OK;
  float w[kSsimTaps];
  double sum = 0.0;
  for (int k = 0; k < kSsimTaps; ++k) {
    const double x = k - (kSsimTaps - 1) / 2.0;
    sum += w[k] = (float)exp(-(x * x) / (2.0 * 1.5 * 1.5));
  }
  for (int k = 0; k < kSsimTaps; ++k) w[k] = (float)(w[k] / sum);
  GS_CUDA(cudaMemcpyToSymbol(c_gauss, w, sizeof(w)));
  g_gauss_ready[dev] = 1;
  return GS_OK;
}

static size_t ssim_blocks(int H, int W) {
  return (size_t)((W + kSsimTW - 1) / kSsimTW) * ((H + kSsimTH - 1) / kSsimTH);
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_l1_ssim_workspace_size(int H, int W) {
  if (H <= 0 || W <= 0) return 0;
  return (size_t)H * W * 9 * sizeof(float) + ssim_blocks(H, W) * 2 * sizeof(double) + 256;
}

extern "C" int gs_l1_ssim_forward(int H, int W, const float* img, const float* target,
                                  float lambda_dssim, void* workspace, size_t workspace_bytes,
                                  float* loss, float* ssim_value, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  GS_REQUIRE(img && target && workspace && loss, "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_l1_ssim_workspace_size(H, W), "workspace too small");
  const int rc = ensure_gauss();
  if (rc != GS_OK) return rc;
  float* maps = static_cast<float*>(workspace);
  double* partials = reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(maps + (size_t)H * W * 9) + 255u) & ~uintptr_t(255u));
  const dim3 grid((W + kSsimTW - 1) / kSsimTW, (H + kSsimTH - 1) / kSsimTH);
  const size_t smem = sizeof(SsimForwardSmem);
  GS_CUDA(cudaFuncSetAttribute(ssim_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  cudaStream_t st = (cudaStream_t)stream;
  ssim_forward_kernel<<<grid, kSsimThreads, smem, st>>>(H, W, img, target, maps, partials);
  GS_CHECK_LAUNCH();
  ssim_finalize_kernel<<<1, 256, 0, st>>>(partials, (int)(grid.x * grid.y),
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
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  GS_REQUIRE(img && target && workspace && grad_loss && grad_img, "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_l1_ssim_workspace_size(H, W), "workspace too small");
  const int rc = ensure_gauss();
  if (rc != GS_OK) return rc;
  const dim3 grid((W + kSsimTW - 1) / kSsimTW, (H + kSsimTH - 1) / kSsimTH);
  const size_t smem = sizeof(SsimBackwardSmem);
  GS_CUDA(cudaFuncSetAttribute(ssim_backward_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ssim_backward_kernel<<<grid, kSsimThreads, smem, (cudaStream_t)stream>>>(
      H, W, img, target, static_cast<const float*>(workspace), grad_loss, lambda_dssim,
      1.0f / (float)((double)H * W * 3), grad_img);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
