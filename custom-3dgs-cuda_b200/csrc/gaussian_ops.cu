// Per-Gaussian kernels behind gs_project, gs_sh_forward, gs_sh_backward and
// gs_project_backward: one thread per Gaussian; every [N, F] row array (the 45-float SH rows,
// means, quaternions, log-scales, the projected outputs and the gradients) moves between HBM
// and shared memory a warp at a time with 16-byte coalesced accesses.
#include "capi_internal.h"
#include "gaussian_ops.cuh"
#include "projection.cuh"
#include "sh.cuh"

namespace gs {

// Rows [row0, row0 + 32) of a [N, F] array into `stage`: asynchronous 16-byte copies for a
// full, aligned group (the caller waits with cp.async.wait_group 0), scalar loads otherwise.
template <int F>
__device__ __forceinline__ void stage_rows(const float* __restrict__ src, int row0, int n,
                                           float* stage) {
  if (!warp_prefetch_rows<F>(src, row0, n, stage)) warp_load_rows<F>(src, row0, n, stage);
}

__device__ __forceinline__ void wait_staged() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncwarp();
}

// One warp per 32 Gaussians: their mu, q, s rows arrive as 16-byte copies into shared memory
// (all three in flight at once), each lane projects one Gaussian, and the mean2d, cov2d and
// depth rows leave as 16-byte stores from the same staging area.
__global__ void __launch_bounds__(256) project_kernel(int N, const float* __restrict__ mu,
                                                      const float* __restrict__ q,
                                                      const float* __restrict__ s,
                                                      const float* __restrict__ R,
                                                      const float* __restrict__ t, float fx,
                                                      float fy, float cx, float cy,
                                                      float* __restrict__ mean2d,
                                                      float* __restrict__ cov2d,
                                                      float* __restrict__ depths) {
  constexpr int kIn = 32 * (3 + 4 + 3);
  __shared__ __align__(16) float s_stage[8][kIn];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= N) return;
  float* st = s_stage[warp];
  stage_rows<3>(mu, row0, N, st);
  stage_rows<4>(q, row0, N, st + 96);
  stage_rows<3>(s, row0, N, st + 224);
  Camera cam;
  load_camera(R, t, fx, fy, cx, cy, cam);
  wait_staged();
  Projected p;
  const float* m = st + 3 * lane;
  const float* qq = st + 96 + 4 * lane;
  const float* ss = st + 224 + 3 * lane;
  project_gaussian(cam, m[0], m[1], m[2], make_float4(qq[0], qq[1], qq[2], qq[3]),
                   make_float3(ss[0], ss[1], ss[2]), p);
  __syncwarp();
  // outputs: mean2d rows [0, 64), cov2d rows [64, 160), depths [160, 192)
  st[2 * lane] = p.mean.x;
  st[2 * lane + 1] = p.mean.y;
  st[64 + 3 * lane] = p.cov.x;
  st[64 + 3 * lane + 1] = p.cov.y;
  st[64 + 3 * lane + 2] = p.cov.z;
  st[160 + lane] = p.depth;
  __syncwarp();
  warp_store_rows<2>(mean2d, row0, N, st);
  warp_store_rows<3>(cov2d, row0, N, st + 64);
  warp_store_rows<1>(depths, row0, N, st + 160);
}

// The same staging for the projection backward: g_mean2d, g_cov2d, mu, q, s in; g_mu, g_q,
// g_s out.
__global__ void __launch_bounds__(256) project_backward_kernel(
    int N, const float* __restrict__ g_mean2d, const float* __restrict__ g_cov2d,
    const float* __restrict__ mu, const float* __restrict__ q, const float* __restrict__ s,
    const float* __restrict__ R, const float* __restrict__ t, float fx, float fy, float cx,
    float cy, float* __restrict__ g_mu, float* __restrict__ g_q, float* __restrict__ g_s) {
  constexpr int kIn = 32 * (2 + 3 + 3 + 4 + 3);
  __shared__ __align__(16) float s_stage[8][kIn];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= N) return;
  float* st = s_stage[warp];
  stage_rows<2>(g_mean2d, row0, N, st);
  stage_rows<3>(g_cov2d, row0, N, st + 64);
  stage_rows<3>(mu, row0, N, st + 160);
  stage_rows<4>(q, row0, N, st + 256);
  stage_rows<3>(s, row0, N, st + 384);
  Camera cam;
  load_camera(R, t, fx, fy, cx, cy, cam);
  wait_staged();
  const float* gm = st + 2 * lane;
  const float* gc = st + 64 + 3 * lane;
  const float* m = st + 160 + 3 * lane;
  const float* qq = st + 256 + 4 * lane;
  const float* ss = st + 384 + 3 * lane;
  ProjectionGrad g;
  project_gaussian_backward(cam, m[0], m[1], m[2], make_float4(qq[0], qq[1], qq[2], qq[3]),
                            make_float3(ss[0], ss[1], ss[2]), make_float2(gm[0], gm[1]),
                            make_float3(gc[0], gc[1], gc[2]), g);
  __syncwarp();
  // outputs: g_mu rows [0, 96), g_q rows [96, 224), g_s rows [224, 320)
  st[3 * lane] = g.mu.x;
  st[3 * lane + 1] = g.mu.y;
  st[3 * lane + 2] = g.mu.z;
  st[96 + 4 * lane] = g.q.x;
  st[96 + 4 * lane + 1] = g.q.y;
  st[96 + 4 * lane + 2] = g.q.z;
  st[96 + 4 * lane + 3] = g.q.w;
  st[224 + 3 * lane] = g.s.x;
  st[224 + 3 * lane + 1] = g.s.y;
  st[224 + 3 * lane + 2] = g.s.z;
  __syncwarp();
  warp_store_rows<3>(g_mu, row0, N, st);
  warp_store_rows<4>(g_q, row0, N, st + 96);
  warp_store_rows<3>(g_s, row0, N, st + 224);
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
