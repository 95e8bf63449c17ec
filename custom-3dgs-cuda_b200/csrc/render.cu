// Fused render path used by RasterizeFunction: the whole forward of one view from the
// Gaussian parameters (gs_render_forward) and the whole backward to the parameter gradients
// (gs_render_backward). Same device functions, hence the same results, as the per-op entry
// points; the intermediates mean2d / cov2d / depths / colours never go through HBM.
//
// Forward: render_preprocess_kernel (projection + SH colour + screen radius + binning prep,
// one thread per Gaussian, SH rows staged warp-wide) followed by the shared depth sort, pair
// duplication, tile sort, tile ranges and blend of launch_sort_and_blend.
// Backward: blend_backward_kernel<true> accumulates per-Gaussian sums (dL/dmean2d, dL/dSigma2
// converted per tile, opacity and colour gradients) with vector atomics;
// render_gaussian_backward_kernel then, per Gaussian, runs the SH and projection backward and
// writes (or accumulates into) the six parameter gradients and dL/dmean2d.
#include "binning.cuh"
#include "blend.cuh"
#include "capi_internal.h"
#include "gaussian_ops.cuh"
#include "onesweep.cuh"
#include "projection.cuh"
#include "raster_internal.h"
#include "sh.cuh"

namespace gs {

// torch's radius formula of the reference wrapper (rasterize.py:49-53), op by op with
// round-to-nearest intrinsics (no contraction) so that it matches torch bit for bit:
// mid = 0.5 (a + c); r = mid + sqrt(clamp(((a - c) / 2)^2 + b^2, min 0.1));
// radius = 3 sqrt(clamp(r, min 0)). clamp keeps NaN as torch does.
__device__ __forceinline__ float torch_clamp_min(float x, float m) {
  return (x != x) ? x : fmaxf(x, m);
}
__device__ __forceinline__ float screen_radius(float a, float b, float c) {
  const float mid = __fmul_rn(0.5f, __fadd_rn(a, c));
  const float h = __fmul_rn(0.5f, __fsub_rn(a, c));
  const float r2 = __fadd_rn(__fmul_rn(h, h), __fmul_rn(b, b));
  const float r = __fadd_rn(mid, __fsqrt_rn(torch_clamp_min(r2, 0.1f)));
  return __fmul_rn(3.0f, __fsqrt_rn(torch_clamp_min(r, 0.0f)));
}

struct PreprocessParams {
  BinParams bin;
  const float *mu, *q, *s, *opacity, *albedo, *k_j, *R, *t, *cam_pos;
  float fx, fy, cx, cy;
  float* radii;
};

constexpr size_t kPreprocessSmem = 8 * 32 * kShRestFloats * sizeof(float);

__global__ void __launch_bounds__(kBinThreads) render_preprocess_kernel(PreprocessParams pp) {
  __shared__ unsigned s_scan[33];
  __shared__ unsigned s_hist[4][256];
  __shared__ bool s_last;
  extern __shared__ __align__(16) float s_stage[];  // [8 warps][32 * 45]
  const BinParams& p = pp.bin;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int k = tid; k < 4 * 256; k += kBinThreads) (&s_hist[0][0])[k] = 0u;
  __syncthreads();
  const int tile = (int)blockIdx.x;
  const int i = tile * kBinThreads + tid;

  // the warp's SH rows are copied into its stage while the projection runs
  float* stage = s_stage + warp * 32 * kShRestFloats;
  const bool rows_async =
      warp_prefetch_rows<kShRestFloats>(pp.k_j, tile * kBinThreads + warp * 32, p.N, stage);
  Camera cam;
  load_camera(pp.R, pp.t, pp.fx, pp.fy, pp.cx, pp.cy, cam);
  Projected pr;
  unsigned count = 0, depth_bits = 0;
  float3 m = make_float3(0.f, 0.f, 0.f);
  if (i < p.N) {
    m = make_float3(__ldg(pp.mu + 3 * i), __ldg(pp.mu + 3 * i + 1), __ldg(pp.mu + 3 * i + 2));
    const float4 qi = make_float4(__ldg(pp.q + 4 * i), __ldg(pp.q + 4 * i + 1),
                                  __ldg(pp.q + 4 * i + 2), __ldg(pp.q + 4 * i + 3));
    const float3 si =
        make_float3(__ldg(pp.s + 3 * i), __ldg(pp.s + 3 * i + 1), __ldg(pp.s + 3 * i + 2));
    const bool front = project_gaussian(cam, m.x, m.y, m.z, qi, si, pr);
    pp.radii[i] = screen_radius(pr.cov.x, pr.cov.y, pr.cov.z);
    TileRect r;
    if (front && splat_tile_rect(pr.mean, pr.cov.x, pr.cov.y, pr.cov.z, p.W, p.H, p.tiles_x,
                                 p.tiles_y, r))
      count = (unsigned)rect_count(r);
  }
  // SH colour only for splats that cover a tile; the warp stages its SH rows if any lane does
  if (rows_async) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  if (__ballot_sync(0xffffffffu, count > 0)) {
    if (!rows_async)
      warp_load_rows<kShRestFloats>(pp.k_j, tile * kBinThreads + warp * 32, p.N, stage);
    if (count > 0) {
      const float* kj = stage + lane * kShRestFloats;
      const float3 cp = make_float3(__ldg(pp.cam_pos), __ldg(pp.cam_pos + 1), __ldg(pp.cam_pos + 2));
      const float3 A = make_float3(__ldg(pp.albedo + 3 * i), __ldg(pp.albedo + 3 * i + 1),
                                   __ldg(pp.albedo + 3 * i + 2));
      const float3 d = sh_forward_direction(m, cp);
      float Y[kShRest];
      sh_basis(d.x, d.y, d.z, Y);
      const float3 rgb = sh_unclamped(Y, A, kj);
      const float3 col = make_float3(clamp01(rgb.x), clamp01(rgb.y), clamp01(rgb.z));
      count = bin_gaussian(p, i, pr.mean, pr.cov.x, pr.cov.y, pr.cov.z, pr.depth, col,
                           __ldg(pp.opacity + i), depth_bits);
    }
  }
  bin_block(p, tile, i, count, depth_bits, s_scan, s_hist, s_last);
}

struct GaussianBwdParams {
  int N;
  const float4* accum;  // 3 per Gaussian from blend_backward_kernel<true>
  const float *mu, *q, *s, *albedo, *k_j, *R, *t, *cam_pos;
  float fx, fy, cx, cy;
  float *g_mu, *g_q, *g_s, *g_opacity, *g_albedo, *g_k_j, *g_mean2d;
  int accumulate;
  // densification statistics (optional): per Gaussian, n = |dL/dmean2d * (sx, sy)|; where
  // n > 0: norm_sum += n, count += 1; norm_max = max(norm_max, n)
  float *stat_norm_sum, *stat_count, *stat_max;
  float stat_sx, stat_sy;
};

template <int F>
__device__ __forceinline__ void warp_add_rows(float* __restrict__ dst, int row0, int n_rows,
                                              const float* stage) {
  const int lane = threadIdx.x & 31;
  const int n = min(32, n_rows - row0) * F;
  float* base = dst + (size_t)row0 * F;
  for (int i = lane; i < n; i += 32) base[i] += stage[i];
}

__device__ __forceinline__ void put(float* p, float v, bool acc) {
  if (acc) *p += v; else *p = v;
}

__global__ void __launch_bounds__(256, 3) render_gaussian_backward_kernel(GaussianBwdParams p) {
  extern __shared__ __align__(16) float s_stage[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= p.N) return;
  const int i = row0 + lane;
  const bool valid = i < p.N;
  // the warp's SH rows are copied into its stage while the blend sums are read
  float* stage = s_stage + warp * 32 * kShRestFloats;
  const bool rows_async = warp_prefetch_rows<kShRestFloats>(p.k_j, row0, p.N, stage);
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, a2 = a0;
  if (valid) {
    a0 = p.accum[3 * i];
    a1 = p.accum[3 * i + 1];
    a2 = p.accum[3 * i + 2];
  }
  const bool touched = a0.x != 0.f || a0.y != 0.f || a0.z != 0.f || a0.w != 0.f ||
                       a1.x != 0.f || a1.y != 0.f || a1.z != 0.f || a1.w != 0.f || a2.x != 0.f;
  const bool acc = p.accumulate != 0;
  const bool warp_touched = __ballot_sync(0xffffffffu, touched) != 0u;
  if (rows_async) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
  } else if (warp_touched) {
    warp_load_rows<kShRestFloats>(p.k_j, row0, p.N, stage);
  }
  float* row = stage + lane * kShRestFloats;
  if (valid && touched) {
    const float3 gcov = make_float3(a0.z, a0.w, a1.x);  // dL/dSigma2, converted per tile
    const float2 gmean = make_float2(a0.x, a0.y);
    const float3 gcol = make_float3(a1.z, a1.w, a2.x);
    Camera cam;
    load_camera(p.R, p.t, p.fx, p.fy, p.cx, p.cy, cam);
    const float3 m = make_float3(__ldg(p.mu + 3 * i), __ldg(p.mu + 3 * i + 1), __ldg(p.mu + 3 * i + 2));
    const float4 qi = make_float4(__ldg(p.q + 4 * i), __ldg(p.q + 4 * i + 1),
                                  __ldg(p.q + 4 * i + 2), __ldg(p.q + 4 * i + 3));
    const float3 si = make_float3(__ldg(p.s + 3 * i), __ldg(p.s + 3 * i + 1), __ldg(p.s + 3 * i + 2));
    ProjectionGrad pg;
    project_gaussian_backward(cam, m.x, m.y, m.z, qi, si, gmean, gcov, pg);
    const float3 cp = make_float3(__ldg(p.cam_pos), __ldg(p.cam_pos + 1), __ldg(p.cam_pos + 2));
    const float3 A = make_float3(__ldg(p.albedo + 3 * i), __ldg(p.albedo + 3 * i + 1),
                                 __ldg(p.albedo + 3 * i + 2));
    float3 gA;
    const float3 gmu_sh = sh_backward_inplace(gcol, m, cp, A, row, gA);
    put(p.g_mu + 3 * i, pg.mu.x + gmu_sh.x, acc);
    put(p.g_mu + 3 * i + 1, pg.mu.y + gmu_sh.y, acc);
    put(p.g_mu + 3 * i + 2, pg.mu.z + gmu_sh.z, acc);
    put(p.g_q + 4 * i, pg.q.x, acc);
    put(p.g_q + 4 * i + 1, pg.q.y, acc);
    put(p.g_q + 4 * i + 2, pg.q.z, acc);
    put(p.g_q + 4 * i + 3, pg.q.w, acc);
    put(p.g_s + 3 * i, pg.s.x, acc);
    put(p.g_s + 3 * i + 1, pg.s.y, acc);
    put(p.g_s + 3 * i + 2, pg.s.z, acc);
    put(p.g_opacity + i, a1.y, acc);
    put(p.g_albedo + 3 * i, gA.x, acc);
    put(p.g_albedo + 3 * i + 1, gA.y, acc);
    put(p.g_albedo + 3 * i + 2, gA.z, acc);
    if (p.g_mean2d) {
      put(p.g_mean2d + 2 * i, gmean.x, acc);
      put(p.g_mean2d + 2 * i + 1, gmean.y, acc);
    }
    if (p.stat_norm_sum) {
      const float nx = gmean.x * p.stat_sx, ny = gmean.y * p.stat_sy;
      const float n = sqrtf(nx * nx + ny * ny);
      if (n > 0.0f) {
        p.stat_norm_sum[i] += n;
        p.stat_count[i] += 1.0f;
        p.stat_max[i] = fmaxf(p.stat_max[i], n);
      }
    }
  } else if (valid && !acc) {
    for (int k = 0; k < 3; ++k) p.g_mu[3 * i + k] = 0.f;
    for (int k = 0; k < 4; ++k) p.g_q[4 * i + k] = 0.f;
    for (int k = 0; k < 3; ++k) p.g_s[3 * i + k] = 0.f;
    p.g_opacity[i] = 0.f;
    for (int k = 0; k < 3; ++k) p.g_albedo[3 * i + k] = 0.f;
    if (p.g_mean2d) p.g_mean2d[2 * i] = p.g_mean2d[2 * i + 1] = 0.f;
  }
  // SH-rest gradient rows (computed in place in the stage; zero for untouched lanes), written
  // or added coalesced
  if (warp_touched || !acc) {
    if (!(valid && touched))
      for (int k = 0; k < kShRestFloats; ++k) row[k] = 0.f;
    __syncwarp();
    if (acc) warp_add_rows<kShRestFloats>(p.g_k_j, row0, p.N, stage);
    else warp_store_rows<kShRestFloats>(p.g_k_j, row0, p.N, stage);
  }
}

constexpr int kMaxViewsPerCall = GS_MAX_VIEWS_PER_CALL;

struct ViewsBwdParams {
  int N, n_views;
  const float *mu, *q, *s, *albedo, *k_j;
  float *g_mu, *g_q, *g_s, *g_opacity, *g_albedo, *g_k_j;
  int accumulate;
  float *stat_norm_sum, *stat_count, *stat_max;  // all three or none
  const float4* accum[kMaxViewsPerCall];        // 3 per Gaussian, per view
  gs_view_sums views[kMaxViewsPerCall];
};

__device__ __forceinline__ float3 ld3(const float* p, int i) {
  return make_float3(__ldg(p + 3 * i), __ldg(p + 3 * i + 1), __ldg(p + 3 * i + 2));
}

// render_gaussian_backward_kernel over several views: per Gaussian, the parameters are read
// once, each view that reached it (non-zero blend sums) runs the projection and SH backward
// with its own camera, and the contributions are summed in registers in view order, starting
// from the buffers' values (accumulate) or zero. Each view's contribution is formed and
// rounded as the single-view kernel forms it, so one call over all views and one call per view
// give the same bits. Per warp, two shared-memory stages of 32 rows: the SH coefficient rows
// (read warp-wide, coalesced) and their gradient sums (read and written warp-wide).
constexpr size_t kViewsBwdSmem = 2 * kPreprocessSmem;

__global__ void __launch_bounds__(256, 2) render_gaussian_backward_views_kernel(
    const __grid_constant__ ViewsBwdParams p) {
  extern __shared__ __align__(16) float s_stage[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.x * blockDim.x + warp * 32;
  if (row0 >= p.N) return;
  const int i = row0 + lane;
  const bool valid = i < p.N;
  float* stage = s_stage + warp * 32 * kShRestFloats;
  float* gstage = s_stage + (8 + warp) * 32 * kShRestFloats;  // 8 warps per CTA
  const bool rows_async = warp_prefetch_rows<kShRestFloats>(p.k_j, row0, p.N, stage);
  const bool acc = p.accumulate != 0;
  const bool stats = p.stat_norm_sum != nullptr;
  float3 gmu = make_float3(0.f, 0.f, 0.f), gs = gmu, gA = gmu;
  float4 gq = make_float4(0.f, 0.f, 0.f, 0.f);
  float gop = 0.f, st_sum = 0.f, st_cnt = 0.f, st_max = 0.f;
  float* gkj = gstage + lane * kShRestFloats;
  if (acc) {
    warp_load_rows<kShRestFloats>(p.g_k_j, row0, p.N, gstage);
  } else {
#pragma unroll
    for (int k = 0; k < kShRestFloats; ++k) gkj[k] = 0.f;
  }
  if (valid && acc) {
    gmu = make_float3(p.g_mu[3 * i], p.g_mu[3 * i + 1], p.g_mu[3 * i + 2]);
    gq = make_float4(p.g_q[4 * i], p.g_q[4 * i + 1], p.g_q[4 * i + 2], p.g_q[4 * i + 3]);
    gs = make_float3(p.g_s[3 * i], p.g_s[3 * i + 1], p.g_s[3 * i + 2]);
    gop = p.g_opacity[i];
    gA = make_float3(p.g_albedo[3 * i], p.g_albedo[3 * i + 1], p.g_albedo[3 * i + 2]);
  }
  if (valid && stats) {
    st_sum = p.stat_norm_sum[i];
    st_cnt = p.stat_count[i];
    st_max = p.stat_max[i];
  }
  float3 m = make_float3(0.f, 0.f, 0.f), si = m, A = m;
  float4 qi = make_float4(0.f, 0.f, 0.f, 0.f);
  if (valid) {
    m = ld3(p.mu, i);
    qi = make_float4(__ldg(p.q + 4 * i), __ldg(p.q + 4 * i + 1), __ldg(p.q + 4 * i + 2),
                     __ldg(p.q + 4 * i + 3));
    si = ld3(p.s, i);
    A = ld3(p.albedo, i);
  }
  if (rows_async) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
  } else {
    warp_load_rows<kShRestFloats>(p.k_j, row0, p.N, stage);
  }
  const float* row = stage + lane * kShRestFloats;
  bool touched = false;
  if (valid) {
#pragma unroll 1
    for (int v = 0; v < p.n_views; ++v) {
      const float4* a = p.accum[v] + 3 * (size_t)i;
      const float4 a0 = __ldg(a), a1 = __ldg(a + 1);
      const float a2x = __ldg(&a[2].x);
      if (!(a0.x != 0.f || a0.y != 0.f || a0.z != 0.f || a0.w != 0.f || a1.x != 0.f ||
            a1.y != 0.f || a1.z != 0.f || a1.w != 0.f || a2x != 0.f))
        continue;  // this view never reached the Gaussian: it adds nothing
      touched = true;
      const gs_view_sums& vw = p.views[v];
      const float3 gcov = make_float3(a0.z, a0.w, a1.x);  // dL/dSigma2, converted per tile
      const float2 gmean = make_float2(a0.x, a0.y);
      const float3 gcol = make_float3(a1.z, a1.w, a2x);
      Camera cam;
      load_camera(vw.R, vw.t, vw.fx, vw.fy, vw.cx, vw.cy, cam);
      ProjectionGrad pg;
      project_gaussian_backward(cam, m.x, m.y, m.z, qi, si, gmean, gcov, pg);
      const float3 cp = make_float3(__ldg(vw.cam_pos), __ldg(vw.cam_pos + 1),
                                    __ldg(vw.cam_pos + 2));
      float3 gA_v;
      const float3 gmu_sh = sh_backward_accumulate(gcol, m, cp, A, row, gkj, gA_v);
      gmu.x = __fadd_rn(gmu.x, pg.mu.x + gmu_sh.x);
      gmu.y = __fadd_rn(gmu.y, pg.mu.y + gmu_sh.y);
      gmu.z = __fadd_rn(gmu.z, pg.mu.z + gmu_sh.z);
      gq.x = __fadd_rn(gq.x, pg.q.x);
      gq.y = __fadd_rn(gq.y, pg.q.y);
      gq.z = __fadd_rn(gq.z, pg.q.z);
      gq.w = __fadd_rn(gq.w, pg.q.w);
      gs.x = __fadd_rn(gs.x, pg.s.x);
      gs.y = __fadd_rn(gs.y, pg.s.y);
      gs.z = __fadd_rn(gs.z, pg.s.z);
      gop = __fadd_rn(gop, a1.y);
      gA.x = __fadd_rn(gA.x, gA_v.x);
      gA.y = __fadd_rn(gA.y, gA_v.y);
      gA.z = __fadd_rn(gA.z, gA_v.z);
      if (stats) {
        const float nx = gmean.x * vw.stat_scale_x, ny = gmean.y * vw.stat_scale_y;
        const float n = sqrtf(nx * nx + ny * ny);
        if (n > 0.0f) {
          st_sum = __fadd_rn(st_sum, n);
          st_cnt = __fadd_rn(st_cnt, 1.0f);
          st_max = fmaxf(st_max, n);
        }
      }
    }
  }
  // with accumulate, a Gaussian no view reached keeps its buffers as they are
  if (valid && (touched || !acc)) {
    p.g_mu[3 * i] = gmu.x;
    p.g_mu[3 * i + 1] = gmu.y;
    p.g_mu[3 * i + 2] = gmu.z;
    p.g_q[4 * i] = gq.x;
    p.g_q[4 * i + 1] = gq.y;
    p.g_q[4 * i + 2] = gq.z;
    p.g_q[4 * i + 3] = gq.w;
    p.g_s[3 * i] = gs.x;
    p.g_s[3 * i + 1] = gs.y;
    p.g_s[3 * i + 2] = gs.z;
    p.g_opacity[i] = gop;
    p.g_albedo[3 * i] = gA.x;
    p.g_albedo[3 * i + 1] = gA.y;
    p.g_albedo[3 * i + 2] = gA.z;
  }
  if (valid && touched && stats) {
    p.stat_norm_sum[i] = st_sum;
    p.stat_count[i] = st_cnt;
    p.stat_max[i] = st_max;
  }
  // SH-rest gradient rows, coalesced
  __syncwarp();
  warp_store_rows<kShRestFloats>(p.g_k_j, row0, p.N, gstage);
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_render_workspace_size(int N, int H, int W, long long pair_capacity) {
  if (N < 0 || H <= 0 || W <= 0 || pair_capacity < 0) return 0;
  return make_raster_layout(N, W, H, pair_capacity).total;
}

extern "C" int gs_render_forward(int N, int H, int W, const float* mu, const float* q,
                                 const float* s, const float* opacity, const float* albedo,
                                 const float* k_j, const float* R, const float* t,
                                 const float* cam_pos, float fx, float fy, float cx, float cy,
                                 void* workspace, size_t workspace_bytes,
                                 long long pair_capacity, float* img, int* sorted_ids,
                                 int* tile_ranges, float* final_T, int* n_contrib, float* radii,
                                 int* pair_count_host, void* m_ready_event, unsigned flags,
                                 void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE((flags & ~(GS_RENDER_TIGHT_BINS | GS_RENDER_CONCURRENT)) == 0u,
             "unknown render flag");
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  GS_REQUIRE((W + 15) / 16 < 65536 && (H + 15) / 16 < 65536, "image too large");
  GS_REQUIRE(pair_capacity >= 0 && pair_capacity < (1ll << 30),
             "pair capacity must be in [0, 2^30)");
  GS_REQUIRE(img && tile_ranges && final_T && n_contrib && workspace, "null pointer");
  GS_REQUIRE(N == 0 || (mu && q && s && opacity && albedo && k_j && R && t && cam_pos && radii),
             "null input pointer");
  GS_REQUIRE(pair_capacity == 0 || sorted_ids, "null sorted_ids with a non-zero capacity");
  const RasterLayout L = make_raster_layout(N, W, H, pair_capacity);
  GS_REQUIRE(workspace_bytes >= L.total, "workspace too small");
  GS_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0u,
             "workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  RasterHeader* hdr = reinterpret_cast<RasterHeader*>(ws + L.header);
  GS_CUDA(cudaMemsetAsync(ws, 0, L.zero_bytes, st));
  GS_CUDA(cudaMemsetAsync(tile_ranges, 0x7f, (size_t)L.T * 2 * sizeof(int), st));  // kRangeUnset
  mark_stage(0, st);
  if (N > 0) {
    PreprocessParams pp;
    fill_bin_params(pp.bin, L, ws, N, H, W, nullptr, nullptr, nullptr, nullptr, nullptr,
                    pair_capacity);
    pp.bin.tight = (flags & GS_RENDER_TIGHT_BINS) ? 1 : 0;
    pp.mu = mu;
    pp.q = q;
    pp.s = s;
    pp.opacity = opacity;
    pp.albedo = albedo;
    pp.k_j = k_j;
    pp.R = R;
    pp.t = t;
    pp.cam_pos = cam_pos;
    pp.fx = fx;
    pp.fy = fy;
    pp.cx = cx;
    pp.cy = cy;
    pp.radii = radii;
    GS_CUDA(cudaFuncSetAttribute(render_preprocess_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPreprocessSmem));
    GS_CUDA(cudaFuncSetAttribute(render_preprocess_kernel,
                                 cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    render_preprocess_kernel<<<(unsigned)L.nb, kBinThreads, kPreprocessSmem, st>>>(pp);
    GS_CHECK_LAUNCH();
  }
  mark_stage(1, st);
  if (pair_count_host)
    GS_CUDA(cudaMemcpyAsync(pair_count_host, &hdr->pair_count, sizeof(int),
                            cudaMemcpyDeviceToHost, st));
  if (m_ready_event) GS_CUDA(cudaEventRecord((cudaEvent_t)m_ready_event, st));
  return launch_sort_and_blend(L, N, H, W, ws, pair_capacity, img, sorted_ids, tile_ranges,
                               final_T, n_contrib,
                               (flags & GS_RENDER_CONCURRENT) != 0u, st);
  GS_API_END();
}

namespace gs {

// The per-Gaussian blend sums of a backward workspace: 3 float4 per Gaussian from its first
// 256-byte boundary.
static float4* blend_sums(void* workspace) {
  return reinterpret_cast<float4*>(
      (reinterpret_cast<uintptr_t>(workspace) + 255u) & ~uintptr_t(255u));
}

// Clears `accum` and runs the fused-accumulator blend backward of one view into it.
static int launch_blend_backward(int N, int H, int W, const float* grad_img,
                                 const void* fwd_workspace, long long pair_capacity,
                                 const int* sorted_ids, const int* tile_ranges,
                                 const float* final_T, const int* n_contrib, float4* accum,
                                 unsigned flags, cudaStream_t st) {
  const RasterLayout L = make_raster_layout(N, W, H, pair_capacity);
  const char* fws = static_cast<const char*>(fwd_workspace);
  GS_CUDA(cudaMemsetAsync(accum, 0, (size_t)N * 3 * sizeof(float4), st));
  mark_stage(7, st);
  BlendBwdParams bp;
  bp.N = N;
  bp.W = W;
  bp.H = H;
  bp.tiles_x = L.tiles_x;
  bp.num_tiles = (int)L.T;
  bp.pair_count = &reinterpret_cast<const RasterHeader*>(fws + L.header)->pair_count;
  bp.pair_capacity = pair_capacity;
  bp.grad_img = grad_img;
  bp.ranges = reinterpret_cast<const int2*>(tile_ranges);
  bp.tile_order = reinterpret_cast<const int*>(fws + L.tile_order);
  bp.sorted_ids = sorted_ids;
  bp.records = reinterpret_cast<const float4*>(fws + L.records);
  bp.final_T = final_T;
  bp.n_contrib = n_contrib;
  bp.g_mean2d = bp.g_cov2d = bp.g_colors = bp.g_alpha = nullptr;
  bp.g_accum = accum;
  if (flags & GS_RENDER_CONCURRENT) {
    blend_backward_kernel<true, kBlendBwdPixThroughput>
        <<<(unsigned)L.T, kTilePixels / kBlendBwdPixThroughput, 0, st>>>(bp);
  } else {
    blend_backward_kernel<true, kBlendBwdPix>
        <<<(unsigned)L.T, kTilePixels / kBlendBwdPix, 0, st>>>(bp);
  }
  GS_CHECK_LAUNCH();
  mark_stage(8, st);
  return GS_OK;
}

}  // namespace gs

extern "C" size_t gs_render_backward_workspace_size(int N) {
  if (N < 0) return 0;
  return (size_t)N * 3 * sizeof(float4) + 256;
}

extern "C" int gs_render_backward(int N, int H, int W, const float* grad_img, const float* mu,
                                  const float* q, const float* s, const float* albedo,
                                  const float* k_j, const float* R, const float* t,
                                  const float* cam_pos, float fx, float fy, float cx, float cy,
                                  const void* fwd_workspace, long long pair_capacity,
                                  const int* sorted_ids, const int* tile_ranges,
                                  const float* final_T, const int* n_contrib, void* workspace,
                                  size_t workspace_bytes, float* g_mu, float* g_q, float* g_s,
                                  float* g_opacity, float* g_albedo, float* g_k_j,
                                  float* g_mean2d, int accumulate, float* stat_norm_sum,
                                  float* stat_count, float* stat_max, float stat_scale_x,
                                  float stat_scale_y, void* accum_wait_event,
                                  void* accum_done_event, unsigned flags, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE((flags & ~GS_RENDER_CONCURRENT) == 0u, "unknown render backward flag");
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  if (N == 0) return GS_OK;
  GS_REQUIRE(grad_img && mu && q && s && albedo && k_j && R && t && cam_pos && fwd_workspace &&
                 tile_ranges && final_T && n_contrib && workspace && g_mu && g_q && g_s &&
                 g_opacity && g_albedo && g_k_j,
             "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_render_backward_workspace_size(N), "workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  float4* accum = blend_sums(workspace);
  const int rc = launch_blend_backward(N, H, W, grad_img, fwd_workspace, pair_capacity,
                                       sorted_ids, tile_ranges, final_T, n_contrib, accum, flags,
                                       st);
  if (rc != GS_OK) return rc;
  GaussianBwdParams gp;
  gp.N = N;
  gp.accum = accum;
  gp.mu = mu;
  gp.q = q;
  gp.s = s;
  gp.albedo = albedo;
  gp.k_j = k_j;
  gp.R = R;
  gp.t = t;
  gp.cam_pos = cam_pos;
  gp.fx = fx;
  gp.fy = fy;
  gp.cx = cx;
  gp.cy = cy;
  gp.g_mu = g_mu;
  gp.g_q = g_q;
  gp.g_s = g_s;
  gp.g_opacity = g_opacity;
  gp.g_albedo = g_albedo;
  gp.g_k_j = g_k_j;
  gp.g_mean2d = g_mean2d;
  gp.accumulate = accumulate;
  GS_REQUIRE((stat_norm_sum == nullptr) == (stat_count == nullptr) &&
                 (stat_count == nullptr) == (stat_max == nullptr),
             "the three statistics buffers go together");
  gp.stat_norm_sum = stat_norm_sum;
  gp.stat_count = stat_count;
  gp.stat_max = stat_max;
  gp.stat_sx = stat_scale_x;
  gp.stat_sy = stat_scale_y;
  GS_CUDA(cudaFuncSetAttribute(render_gaussian_backward_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kPreprocessSmem));
  GS_CUDA(cudaFuncSetAttribute(render_gaussian_backward_kernel,
                               cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  // the only kernel of the backward that writes the caller's gradient / statistic buffers:
  // ordered after accum_wait_event so that views rendered on other streams can share them
  if (accum_wait_event) GS_CUDA(cudaStreamWaitEvent(st, (cudaEvent_t)accum_wait_event, 0));
  mark_stage(10, st);
  render_gaussian_backward_kernel<<<(N + 255) / 256, 256, kPreprocessSmem, st>>>(gp);
  GS_CHECK_LAUNCH();
  if (accum_done_event) GS_CUDA(cudaEventRecord((cudaEvent_t)accum_done_event, st));
  mark_stage(9, st);
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_render_backward_blend(int N, int H, int W, const float* grad_img,
                                        const void* fwd_workspace, long long pair_capacity,
                                        const int* sorted_ids, const int* tile_ranges,
                                        const float* final_T, const int* n_contrib,
                                        void* workspace, size_t workspace_bytes, unsigned flags,
                                        void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE((flags & ~GS_RENDER_CONCURRENT) == 0u, "unknown render backward flag");
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(H > 0 && W > 0, "image height and width must be positive");
  if (N == 0) return GS_OK;
  GS_REQUIRE(grad_img && fwd_workspace && tile_ranges && final_T && n_contrib && workspace,
             "null pointer");
  GS_REQUIRE(workspace_bytes >= gs_render_backward_workspace_size(N), "workspace too small");
  return launch_blend_backward(N, H, W, grad_img, fwd_workspace, pair_capacity, sorted_ids,
                               tile_ranges, final_T, n_contrib, blend_sums(workspace), flags,
                               (cudaStream_t)stream);
  GS_API_END();
}

extern "C" int gs_render_backward_gaussians(int N, int n_views, const gs_view_sums* views,
                                            const float* mu, const float* q, const float* s,
                                            const float* albedo, const float* k_j, float* g_mu,
                                            float* g_q, float* g_s, float* g_opacity,
                                            float* g_albedo, float* g_k_j, int accumulate,
                                            float* stat_norm_sum, float* stat_count,
                                            float* stat_max, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(n_views >= 1 && n_views <= kMaxViewsPerCall,
             "n_views must be in [1, GS_MAX_VIEWS_PER_CALL]");
  GS_REQUIRE(views != nullptr, "null views");
  if (N == 0) return GS_OK;
  GS_REQUIRE(mu && q && s && albedo && k_j && g_mu && g_q && g_s && g_opacity && g_albedo &&
                 g_k_j,
             "null pointer");
  GS_REQUIRE((stat_norm_sum == nullptr) == (stat_count == nullptr) &&
                 (stat_count == nullptr) == (stat_max == nullptr),
             "the three statistics buffers go together");
  ViewsBwdParams p;
  p.N = N;
  p.n_views = n_views;
  p.mu = mu;
  p.q = q;
  p.s = s;
  p.albedo = albedo;
  p.k_j = k_j;
  p.g_mu = g_mu;
  p.g_q = g_q;
  p.g_s = g_s;
  p.g_opacity = g_opacity;
  p.g_albedo = g_albedo;
  p.g_k_j = g_k_j;
  p.accumulate = accumulate;
  p.stat_norm_sum = stat_norm_sum;
  p.stat_count = stat_count;
  p.stat_max = stat_max;
  for (int v = 0; v < kMaxViewsPerCall; ++v) {
    p.accum[v] = nullptr;
    p.views[v] = gs_view_sums{};
  }
  for (int v = 0; v < n_views; ++v) {
    const gs_view_sums& w = views[v];
    GS_REQUIRE(w.workspace && w.R && w.t && w.cam_pos, "null pointer in a view");
    GS_REQUIRE(w.workspace_bytes >= gs_render_backward_workspace_size(N),
               "a view's workspace is smaller than gs_render_backward_workspace_size(N)");
    p.views[v] = w;
    p.accum[v] = blend_sums(const_cast<void*>(w.workspace));
  }
  cudaStream_t st = (cudaStream_t)stream;
  GS_CUDA(cudaFuncSetAttribute(render_gaussian_backward_views_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kViewsBwdSmem));
  GS_CUDA(cudaFuncSetAttribute(render_gaussian_backward_views_kernel,
                               cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  mark_stage(10, st);
  render_gaussian_backward_views_kernel<<<(N + 255) / 256, 256, kViewsBwdSmem, st>>>(p);
  GS_CHECK_LAUNCH();
  mark_stage(9, st);
  return GS_OK;
  GS_API_END();
}
