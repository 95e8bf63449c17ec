// Per-Gaussian kernels behind gs_project, gs_sh_forward, gs_sh_backward and
// gs_project_backward: one thread per Gaussian; the 45-float SH rows are moved between
// HBM and shared memory a warp at a time with 16-byte coalesced accesses.
#include "capi_internal.h"
#include "gaussian_ops.cuh"
#include "projection.cuh"
#include "sh.cuh"

namespace gs {

__global__ void __launch_bounds__(256) project_kernel(int N, const float* __restrict__ mu,
                                                      const float* __restrict__ q,
                                                      const float* __restrict__ s,
                                                      const float* __restrict__ R,
                                                      const float* __restrict__ t, float fx,
                                                      float fy, float cx, float cy,
                                                      float* __restrict__ mean2d,
                                                      float* __restrict__ cov2d,
                                                      float* __restrict__ depths) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  Camera cam;
  load_camera(R, t, fx, fy, cx, cy, cam);
  const float4 qi = make_float4(__ldg(q + 4 * i), __ldg(q + 4 * i + 1), __ldg(q + 4 * i + 2),
                                __ldg(q + 4 * i + 3));
  const float3 si = make_float3(__ldg(s + 3 * i), __ldg(s + 3 * i + 1), __ldg(s + 3 * i + 2));
  Projected p;
  project_gaussian(cam, __ldg(mu + 3 * i), __ldg(mu + 3 * i + 1), __ldg(mu + 3 * i + 2), qi,
                   si, p);
  mean2d[2 * i] = p.mean.x;
  mean2d[2 * i + 1] = p.mean.y;
  cov2d[3 * i] = p.cov.x;
  cov2d[3 * i + 1] = p.cov.y;
  cov2d[3 * i + 2] = p.cov.z;
  depths[i] = p.depth;
}

__global__ void __launch_bounds__(256) project_backward_kernel(
    int N, const float* __restrict__ g_mean2d, const float* __restrict__ g_cov2d,
    const float* __restrict__ mu, const float* __restrict__ q, const float* __restrict__ s,
    const float* __restrict__ R, const float* __restrict__ t, float fx, float fy, float cx,
    float cy, float* __restrict__ g_mu, float* __restrict__ g_q, float* __restrict__ g_s) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  Camera cam;
  load_camera(R, t, fx, fy, cx, cy, cam);
  const float4 qi = make_float4(__ldg(q + 4 * i), __ldg(q + 4 * i + 1), __ldg(q + 4 * i + 2),
                                __ldg(q + 4 * i + 3));
  const float3 si = make_float3(__ldg(s + 3 * i), __ldg(s + 3 * i + 1), __ldg(s + 3 * i + 2));
  const float2 gm = make_float2(__ldg(g_mean2d + 2 * i), __ldg(g_mean2d + 2 * i + 1));
  const float3 gc =
      make_float3(__ldg(g_cov2d + 3 * i), __ldg(g_cov2d + 3 * i + 1), __ldg(g_cov2d + 3 * i + 2));
  ProjectionGrad g;
  project_gaussian_backward(cam, __ldg(mu + 3 * i), __ldg(mu + 3 * i + 1),
                            __ldg(mu + 3 * i + 2), qi, si, gm, gc, g);
  g_mu[3 * i] = g.mu.x;
  g_mu[3 * i + 1] = g.mu.y;
  g_mu[3 * i + 2] = g.mu.z;
  g_q[4 * i] = g.q.x;
  g_q[4 * i + 1] = g.q.y;
  g_q[4 * i + 2] = g.q.z;
  g_q[4 * i + 3] = g.q.w;
  g_s[3 * i] = g.s.x;
  g_s[3 * i + 1] = g.s.y;
  g_s[3 * i + 2] = g.s.z;
}

__global__ void __launch_bounds__(256) sh_forward_kernel(int N, const float* __restrict__ cam_pos,
                                                         const float* __restrict__ mu,
                                                         const float* __restrict__ albedo,
                                                         const float* __restrict__ k_j,
                                                         float* __restrict__ colors) {
  __shared__ __align__(16) float s_kj[8][32 * kShRestFloats];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= N) return;
  float* stage = s_kj[warp];
  warp_load_rows<kShRestFloats>(k_j, row0, N, stage);
  const int i = row0 + lane;
  if (i >= N) return;
  const float3 cam = make_float3(__ldg(cam_pos), __ldg(cam_pos + 1), __ldg(cam_pos + 2));
  const float3 m = make_float3(__ldg(mu + 3 * i), __ldg(mu + 3 * i + 1), __ldg(mu + 3 * i + 2));
  const float3 A =
      make_float3(__ldg(albedo + 3 * i), __ldg(albedo + 3 * i + 1), __ldg(albedo + 3 * i + 2));
  float kj[kShRestFloats];
#pragma unroll
  for (int k = 0; k < kShRestFloats; ++k) kj[k] = stage[lane * kShRestFloats + k];
  const float3 d = sh_forward_direction(m, cam);
  float Y[kShRest];
  sh_basis(d.x, d.y, d.z, Y);
  const float3 rgb = sh_unclamped(Y, A, kj);
  colors[3 * i] = clamp01(rgb.x);
  colors[3 * i + 1] = clamp01(rgb.y);
  colors[3 * i + 2] = clamp01(rgb.z);
}

__global__ void __launch_bounds__(256) sh_backward_kernel(
    int N, const float* __restrict__ g_colors, const float* __restrict__ mu,
    const float* __restrict__ albedo, const float* __restrict__ k_j,
    const float* __restrict__ cam_pos, float* __restrict__ g_albedo, float* __restrict__ g_kj,
    float* __restrict__ g_mu) {
  __shared__ __align__(16) float s_kj[8][32 * kShRestFloats];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= N) return;
  float* stage = s_kj[warp];
  warp_load_rows<kShRestFloats>(k_j, row0, N, stage);
  const int i = row0 + lane;
  if (i < N) {
    const float3 cam = make_float3(__ldg(cam_pos), __ldg(cam_pos + 1), __ldg(cam_pos + 2));
    const float3 m =
        make_float3(__ldg(mu + 3 * i), __ldg(mu + 3 * i + 1), __ldg(mu + 3 * i + 2));
    const float3 A = make_float3(__ldg(albedo + 3 * i), __ldg(albedo + 3 * i + 1),
                                 __ldg(albedo + 3 * i + 2));
    const float3 gc = make_float3(__ldg(g_colors + 3 * i), __ldg(g_colors + 3 * i + 1),
                                  __ldg(g_colors + 3 * i + 2));
    float kj[kShRestFloats], gkj[kShRestFloats];
#pragma unroll
    for (int k = 0; k < kShRestFloats; ++k) kj[k] = stage[lane * kShRestFloats + k];
    float3 gA;
    const float3 gm = sh_backward(gc, m, cam, A, kj, gA, gkj);
#pragma unroll
    for (int k = 0; k < kShRestFloats; ++k) stage[lane * kShRestFloats + k] = gkj[k];
    g_albedo[3 * i] = gA.x;
    g_albedo[3 * i + 1] = gA.y;
    g_albedo[3 * i + 2] = gA.z;
    g_mu[3 * i] = gm.x;
    g_mu[3 * i + 1] = gm.y;
    g_mu[3 * i + 2] = gm.z;
  }
  __syncwarp();
  warp_store_rows<kShRestFloats>(g_kj, row0, N, stage);
}

}  // namespace gs

using namespace gs;

extern "C" int gs_project(int N, const float* mu, const float* q, const float* s,
                          const float* R, const float* t, float fx, float fy, float cx,
                          float cy, float* mean2d, float* cov2d, float* depths, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  if (N == 0) return GS_OK;
  GS_REQUIRE(mu && q && s && R && t && mean2d && cov2d && depths, "null pointer");
  project_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(N, mu, q, s, R, t, fx, fy,
                                                                   cx, cy, mean2d, cov2d, depths);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_project_backward(int N, const float* g_mean2d, const float* g_cov2d,
                                   const float* mu, const float* q, const float* s,
                                   const float* R, const float* t, float fx, float fy,
                                   float cx, float cy, float* g_mu, float* g_q, float* g_s,
                                   void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  if (N == 0) return GS_OK;
  GS_REQUIRE(g_mean2d && g_cov2d && mu && q && s && R && t && g_mu && g_q && g_s,
             "null pointer");
  project_backward_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      N, g_mean2d, g_cov2d, mu, q, s, R, t, fx, fy, cx, cy, g_mu, g_q, g_s);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_sh_forward(int N, const float* cam_pos, const float* mu, const float* albedo,
                             const float* k_j, float* colors, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  if (N == 0) return GS_OK;
  GS_REQUIRE(cam_pos && mu && albedo && k_j && colors, "null pointer");
  sh_forward_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(N, cam_pos, mu, albedo,
                                                                      k_j, colors);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_sh_backward(int N, const float* grad_colors, const float* mu,
                              const float* albedo, const float* k_j, const float* cam_pos,
                              float* g_albedo, float* g_k_j, float* g_mu, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  if (N == 0) return GS_OK;
  GS_REQUIRE(grad_colors && mu && albedo && k_j && cam_pos && g_albedo && g_k_j && g_mu,
             "null pointer");
  sh_backward_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      N, grad_colors, mu, albedo, k_j, cam_pos, g_albedo, g_k_j, g_mu);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
