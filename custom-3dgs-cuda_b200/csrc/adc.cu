// Adaptive density control on the device: the clone / split / prune / opacity-reset step of
// the reference trainer (gaussian_splatting/utils/adc.py:330-392), which the reference runs
// as Python over torch ops with host syncs. Two calls:
//
// gs_adc_plan classifies every Gaussian (one thread each) with the reference's rules:
//   g = nan_to_num(grad_accum / max(denom, 1)), m = max_k exp(s_k), o = sigmoid(alpha);
//   clone if densify and g >= threshold and m <= percent_dense * extent,
//   split if densify and g >= threshold and m >  percent_dense * extent;
//   a Gaussian, its clone and its two split children are pruned when o < min_opacity or
//   their largest scale exceeds 0.1 * extent or (max_screen_size given) their screen radius
//   does (the radius of a new Gaussian is 0; a child's scales are exp(log(exp(s) / 1.6))).
// It writes a decision byte per Gaussian and, per block of 256, the number of kept
// originals, kept clones, split Gaussians, kept children and clones; one CTA then scans the block
// counts into block offsets and totals, which reach the host through a pinned copy.
//
// gs_adc_apply writes the result in the reference's order, [kept originals][kept clones]
// [kept first children][kept second children], each in index order (each warp copies its 32
// Gaussians' rows group by group with coalesced loads): parameters copied (a
// child's mean is R(q) (z * exp(s)) + mu with the caller's unit normals z, its log-scales
// log(exp(s) / 1.6)), Adam moments copied for originals and zero for new Gaussians, and
// with the opacity reset alpha = min(alpha, logit(0.01)) and zero opacity moments.
#include <algorithm>
#include <cmath>

#include "capi_internal.h"
#include "gs_common.cuh"

namespace gs {

constexpr int kAdcThreads = 256;
constexpr int kAdcScanThreads = 1024;
constexpr int kAdcGroups = 6;
constexpr int kAdcCats = 5;  // kept originals, kept clones, split, kept children, clones

enum : unsigned char {
  kAdcClone = 1, kAdcSplit = 2, kAdcKeepOrig = 4, kAdcKeepClone = 8, kAdcKeepChild = 16,
};

struct AdcRules {
  float grad_threshold, pd_line, big_line, min_opacity, max_screen;  // max_screen < 0: none
  int densify, prune;
};

struct AdcLayout {  // workspace: decisions, per-block counts and offsets, totals
  size_t flags, counts, offsets, totals, total;
  int blocks;
};

static AdcLayout adc_layout(int N) {
  AdcLayout L;
  L.blocks = (N + kAdcThreads - 1) / kAdcThreads;
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t at = off;
    off += (b + 255) / 256 * 256;
    return at;
  };
  L.flags = take((size_t)std::max(N, 1));
  L.counts = take((size_t)std::max(L.blocks, 1) * kAdcCats * sizeof(unsigned));
  L.offsets = take((size_t)std::max(L.blocks, 1) * kAdcCats * sizeof(unsigned));
  L.totals = take(kAdcCats * sizeof(long long));
  L.total = off;
  return L;
}

__device__ __forceinline__ float adc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __launch_bounds__(kAdcThreads) adc_classify_kernel(
    int N, const float* __restrict__ s, const float* __restrict__ alpha,
    const float* __restrict__ grad_accum, const float* __restrict__ denom,
    const float* __restrict__ max_radii, AdcRules r, unsigned char* __restrict__ flags,
    unsigned* __restrict__ block_counts) {
  __shared__ unsigned s_cnt[kAdcCats];
  const int i = blockIdx.x * kAdcThreads + threadIdx.x;
  if (threadIdx.x < kAdcCats) s_cnt[threadIdx.x] = 0u;
  __syncthreads();
  unsigned char f = 0;
  if (i < N) {
    float g = grad_accum[i] / fmaxf(denom[i], 1.0f);
    if (g != g) g = 0.0f;  // nan_to_num(nan=0); +-inf map to the finite extremes
    if (isinf(g)) g = g > 0.0f ? 3.402823466e38f : -3.402823466e38f;
    const float e0 = expf(s[3 * i]), e1 = expf(s[3 * i + 1]), e2 = expf(s[3 * i + 2]);
    const float m = fmaxf(fmaxf(e0, e1), e2);
    const bool grad_ok = r.densify && g >= r.grad_threshold;
    const bool clone = grad_ok && m <= r.pd_line;
    const bool split = grad_ok && m > r.pd_line;
    const float o = adc_sigmoid(alpha[i]);
    const float c0 = expf(logf(e0 / 1.6f)), c1 = expf(logf(e1 / 1.6f)), c2 = expf(logf(e2 / 1.6f));
    const float mc = fmaxf(fmaxf(c0, c1), c2);
    const bool low = o < r.min_opacity;
    const bool prune_orig =
        r.prune && (low || m > r.big_line || (r.max_screen >= 0.0f && max_radii[i] > r.max_screen));
    // a new Gaussian's screen radius is 0, so only its opacity and scales can prune it
    const bool prune_new = r.prune && (low || m > r.big_line);
    const bool prune_child = r.prune && (low || mc > r.big_line);
    f = (clone ? kAdcClone : 0) | (split ? kAdcSplit : 0) |
        (!split && !prune_orig ? kAdcKeepOrig : 0) | (clone && !prune_new ? kAdcKeepClone : 0) |
        (split && !prune_child ? kAdcKeepChild : 0);
    flags[i] = f;
  }
  const unsigned full = 0xffffffffu;
  const unsigned a = __popc(__ballot_sync(full, f & kAdcKeepOrig));
  const unsigned b = __popc(__ballot_sync(full, f & kAdcKeepClone));
  const unsigned c = __popc(__ballot_sync(full, f & kAdcSplit));
  const unsigned d = __popc(__ballot_sync(full, f & kAdcKeepChild));
  const unsigned e = __popc(__ballot_sync(full, f & kAdcClone));
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&s_cnt[0], a);
    atomicAdd(&s_cnt[1], b);
    atomicAdd(&s_cnt[2], c);
    atomicAdd(&s_cnt[3], d);
    atomicAdd(&s_cnt[4], e);
  }
  __syncthreads();
  if (threadIdx.x < kAdcCats)
    block_counts[kAdcCats * blockIdx.x + threadIdx.x] = s_cnt[threadIdx.x];
}

// One CTA: exclusive scan of the per-block counts of each category; totals last.
__global__ void __launch_bounds__(kAdcScanThreads) adc_scan_kernel(
    int blocks, const unsigned* __restrict__ counts, unsigned* __restrict__ offsets,
    long long* __restrict__ totals) {
  __shared__ unsigned s_scan[33];
  for (int cat = 0; cat < kAdcCats; ++cat) {
    unsigned carry = 0;
    for (int b0 = 0; b0 < blocks; b0 += kAdcScanThreads) {
      const int b = b0 + threadIdx.x;
      const unsigned v = b < blocks ? counts[kAdcCats * b + cat] : 0u;
      unsigned chunk;
      const unsigned ex = block_exclusive_scan(v, s_scan, &chunk);
      if (b < blocks) offsets[kAdcCats * b + cat] = carry + ex;
      carry += chunk;
    }
    if (threadIdx.x == 0) totals[cat] = (long long)carry;
  }
}

struct AdcApply {
  int N;
  const unsigned char* flags;
  const unsigned* offsets;
  long long n_orig, n_clone, n_child;  // kept originals, kept clones, kept children per copy
  long long n_split;                   // split Gaussians (rows of z per copy)
  const float* in[kAdcGroups];
  const float* m_in[kAdcGroups];
  const float* v_in[kAdcGroups];
  float* out[kAdcGroups];
  float* m_out[kAdcGroups];
  float* v_out[kAdcGroups];
  const float* z;
  int reset_opacity;
  float opacity_cap;  // logit(0.01)
};

__device__ __forceinline__ unsigned block_rank(bool pred, unsigned* s_warp, unsigned* total) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned ballot = __ballot_sync(full, pred);
  if (lane == 0) s_warp[warp] = __popc(ballot);
  __syncthreads();
  unsigned before = 0, all = 0;
  for (int w = 0; w < kAdcThreads / 32; ++w) {
    const unsigned c = s_warp[w];
    if (w < warp) before += c;
    all += c;
  }
  __syncthreads();
  *total = all;
  return before + __popc(ballot & ((1u << lane) - 1u));
}

// Warp-cooperative row copy of one parameter group (D floats per row): the warp's 32
// Gaussians' rows are contiguous in the source, so the lanes walk those 32 D floats in order
// (coalesced loads); each float goes to row dst_row of its owner lane (taken by shuffle), or
// nowhere when that is negative. `zero` writes zeros instead (new Gaussians' Adam moments),
// `cap` applies the opacity reset min(v, cap_v).
template <int D>
__device__ __forceinline__ void warp_copy_rows(const float* __restrict__ src,
                                               float* __restrict__ dst, long long row0,
                                               long long dst_row, bool zero, bool cap,
                                               float cap_v) {
  const int lane = threadIdx.x & 31;
  const float* s = src + row0 * D;
#pragma unroll 4
  for (int e = lane; e < 32 * D; e += 32) {
    const int r = e / D, c = e - r * D;
    const long long dr = __shfl_sync(0xffffffffu, dst_row, r);
    if (dr >= 0) {
      float v = zero ? 0.0f : s[e];
      if (cap) v = fminf(v, cap_v);
      dst[dr * D + c] = v;
    }
  }
}

// Group k of the warp's rows to up to four destinations (kept original, kept clone, the two
// kept children), with the moments; the children's means and log-scales are written per lane
// afterwards (do_params false for those groups).
template <int D>
__device__ __forceinline__ void warp_copy_group(const AdcApply& a, int k, long long row0,
                                                const long long (&dst)[4], bool do_params,
                                                bool reset) {
  const bool cap = k == 3 && reset;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    if (!__any_sync(0xffffffffu, dst[t] >= 0)) continue;
    if (do_params || t < 2) warp_copy_rows<D>(a.in[k], a.out[k], row0, dst[t], false, cap,
                                              a.opacity_cap);
    // moments: copied for originals (zero under the opacity reset), zero for new Gaussians
    const bool zero = t > 0 || cap;
    if (a.m_out[k]) warp_copy_rows<D>(a.m_in[k], a.m_out[k], row0, dst[t], zero, false, 0.f);
    if (a.v_out[k]) warp_copy_rows<D>(a.v_in[k], a.v_out[k], row0, dst[t], zero, false, 0.f);
  }
}

__global__ void __launch_bounds__(kAdcThreads) adc_apply_kernel(AdcApply a) {
  __shared__ unsigned s_warp[kAdcThreads / 32];
  const int i = blockIdx.x * kAdcThreads + threadIdx.x;
  const unsigned char f = i < a.N ? a.flags[i] : 0;
  const unsigned* off = a.offsets + kAdcCats * blockIdx.x;
  unsigned tot;
  const unsigned r_orig = block_rank(f & kAdcKeepOrig, s_warp, &tot);
  const unsigned r_clone = block_rank(f & kAdcKeepClone, s_warp, &tot);
  const unsigned r_split = block_rank(f & kAdcSplit, s_warp, &tot);
  const unsigned r_child = block_rank(f & kAdcKeepChild, s_warp, &tot);
  const bool reset = a.reset_opacity != 0;
  // destination rows of this lane's Gaussian: kept original, kept clone, first and second child
  long long dst[4] = {-1, -1, -1, -1};
  if (f & kAdcKeepOrig) dst[0] = (long long)off[0] + r_orig;
  if (f & kAdcKeepClone) dst[1] = a.n_orig + (long long)off[1] + r_clone;
  if (f & kAdcKeepChild) {
    dst[2] = a.n_orig + a.n_clone + (long long)off[3] + r_child;
    dst[3] = dst[2] + a.n_child;
  }
  const long long row0 = (long long)blockIdx.x * kAdcThreads + (threadIdx.x & ~31);
  warp_copy_group<3>(a, 0, row0, dst, false, reset);  // mu: children computed below
  warp_copy_group<4>(a, 1, row0, dst, true, reset);
  warp_copy_group<3>(a, 2, row0, dst, false, reset);  // s: children computed below
  warp_copy_group<1>(a, 3, row0, dst, true, reset);
  warp_copy_group<3>(a, 4, row0, dst, true, reset);
  warp_copy_group<45>(a, 5, row0, dst, true, reset);
  if (i >= a.N || !(f & kAdcKeepChild)) return;
  // the two children's means R(q)(z * exp(s)) + mu and log-scales log(exp(s) / 1.6)
  const long long row = (long long)off[2] + r_split;  // this Gaussian's rank among splits
  const float* mu = a.in[0] + 3 * (size_t)i;
  const float* q = a.in[1] + 4 * (size_t)i;
  const float* s = a.in[2] + 3 * (size_t)i;
  const float nq = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
  const float inv = 1.0f / fmaxf(nq, 1e-12f);
  const float w = q[0] * inv, x = q[1] * inv, y = q[2] * inv, z = q[3] * inv;
  const float R[3][3] = {
      {1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - w * z), 2.0f * (x * z + w * y)},
      {2.0f * (x * y + w * z), 1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - w * x)},
      {2.0f * (x * z - w * y), 2.0f * (y * z + w * x), 1.0f - 2.0f * (x * x + y * y)}};
  const float e[3] = {expf(s[0]), expf(s[1]), expf(s[2])};
  for (int copy = 0; copy < 2; ++copy) {
    const long long d = dst[2 + copy];
    const float* zr = a.z + 3 * (size_t)(copy * a.n_split + row);
    const float smp[3] = {0.0f + zr[0] * e[0], 0.0f + zr[1] * e[1], 0.0f + zr[2] * e[2]};
    float* mo = a.out[0] + 3 * (size_t)d;
    float* so = a.out[2] + 3 * (size_t)d;
    for (int c = 0; c < 3; ++c) {
      mo[c] = (R[c][0] * smp[0] + R[c][1] * smp[1] + R[c][2] * smp[2]) + mu[c];
      so[c] = logf(e[c] / 1.6f);
    }
  }
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_adc_workspace_size(int N) {
  if (N < 0) return 0;
  return adc_layout(N).total;
}

extern "C" int gs_adc_plan(int N, const float* s, const float* alpha, const float* grad_accum,
                           const float* denom, const float* max_radii, float grad_threshold,
                           float percent_dense_extent, float big_extent, float min_opacity,
                           float max_screen_size, int densify, int prune, void* workspace,
                           size_t workspace_bytes, long long* totals_host, void* done_event,
                           void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  const AdcLayout L = adc_layout(N);
  GS_REQUIRE(workspace && workspace_bytes >= L.total, "workspace too small");
  GS_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0u,
             "workspace must be 256-byte aligned");
  GS_REQUIRE(N == 0 || (s && alpha && grad_accum && denom && max_radii), "null input pointer");
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  long long* totals = reinterpret_cast<long long*>(ws + L.totals);
  if (N == 0) {
    GS_CUDA(cudaMemsetAsync(totals, 0, kAdcCats * sizeof(long long), st));
  } else {
    AdcRules r{grad_threshold, percent_dense_extent, big_extent, min_opacity, max_screen_size,
               densify ? 1 : 0, prune ? 1 : 0};
    adc_classify_kernel<<<L.blocks, kAdcThreads, 0, st>>>(
        N, s, alpha, grad_accum, denom, max_radii, r,
        reinterpret_cast<unsigned char*>(ws + L.flags), reinterpret_cast<unsigned*>(ws + L.counts));
    GS_CHECK_LAUNCH();
    adc_scan_kernel<<<1, kAdcScanThreads, 0, st>>>(
        L.blocks, reinterpret_cast<const unsigned*>(ws + L.counts),
        reinterpret_cast<unsigned*>(ws + L.offsets), totals);
    GS_CHECK_LAUNCH();
  }
  if (totals_host)
    GS_CUDA(cudaMemcpyAsync(totals_host, totals, kAdcCats * sizeof(long long),
                            cudaMemcpyDeviceToHost, st));
  if (done_event) GS_CUDA(cudaEventRecord((cudaEvent_t)done_event, st));
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_adc_apply(int N, const void* workspace, size_t workspace_bytes,
                            const long long* totals, const float* const* params,
                            const float* const* exp_avg, const float* const* exp_avg_sq,
                            const float* z, int reset_opacity, float* const* out_params,
                            float* const* out_exp_avg, float* const* out_exp_avg_sq,
                            void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  const AdcLayout L = adc_layout(N);
  GS_REQUIRE(workspace && workspace_bytes >= L.total, "workspace too small");
  GS_REQUIRE(totals && params && out_params, "null pointer");
  GS_REQUIRE(totals[0] >= 0 && totals[1] >= 0 && totals[2] >= 0 && totals[3] >= 0 &&
                 totals[0] <= N && totals[1] <= N && totals[3] <= totals[2] && totals[2] <= N,
             "totals do not come from gs_adc_plan for this N");
  GS_REQUIRE(totals[2] == 0 || z, "null split samples");
  if (N == 0) return GS_OK;
  AdcApply a{};
  a.N = N;
  const char* ws = static_cast<const char*>(workspace);
  a.flags = reinterpret_cast<const unsigned char*>(ws + L.flags);
  a.offsets = reinterpret_cast<const unsigned*>(ws + L.offsets);
  a.n_orig = totals[0];
  a.n_clone = totals[1];
  a.n_split = totals[2];
  a.n_child = totals[3];
  for (int k = 0; k < kAdcGroups; ++k) {
    GS_REQUIRE(params[k] && out_params[k], "null parameter pointer");
    a.in[k] = params[k];
    a.out[k] = out_params[k];
    const bool has_m = exp_avg && exp_avg[k] && out_exp_avg && out_exp_avg[k];
    const bool has_v = exp_avg_sq && exp_avg_sq[k] && out_exp_avg_sq && out_exp_avg_sq[k];
    a.m_in[k] = has_m ? exp_avg[k] : nullptr;
    a.m_out[k] = has_m ? out_exp_avg[k] : nullptr;
    a.v_in[k] = has_v ? exp_avg_sq[k] : nullptr;
    a.v_out[k] = has_v ? out_exp_avg_sq[k] : nullptr;
  }
  a.z = z;
  a.reset_opacity = reset_opacity ? 1 : 0;
  a.opacity_cap = (float)std::log(0.01 / (1.0 - 0.01));
  adc_apply_kernel<<<L.blocks, kAdcThreads, 0, (cudaStream_t)stream>>>(a);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}

// ---- densification statistics of one view (the reference trainer's
// accumulate_densification_stats, gaussian_splatting/utils/adc.py:58-80) ----
namespace gs {

// One thread per Gaussian: n = |(gx * sx, gy * sy)| of its screen-space mean gradient; where
// n > 0, norm_sum += n and count += 1; norm_max = max(norm_max, n) when given.
__global__ void __launch_bounds__(256) densify_stats_kernel(int N, const float* __restrict__ g2,
                                                            int g_stride, float sx, float sy,
                                                            float* __restrict__ norm_sum,
                                                            float* __restrict__ count,
                                                            float* __restrict__ norm_max) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const float gx = __ldg(g2 + (size_t)i * g_stride) * sx;
  const float gy = __ldg(g2 + (size_t)i * g_stride + 1) * sy;
  const float n = sqrtf(gx * gx + gy * gy);
  if (n > 0.f) {
    norm_sum[i] += n;
    count[i] += 1.f;
  }
  if (norm_max) norm_max[i] = fmaxf(norm_max[i], n);
}

}  // namespace gs

extern "C" int gs_densify_stats(int N, const float* mean2d_grad, int grad_stride, float scale_x,
                                float scale_y, float* norm_sum, float* count, float* norm_max,
                                void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(N >= 0, "N must be non-negative");
  GS_REQUIRE(grad_stride >= 2, "the gradient rows need at least two floats");
  if (N == 0) return GS_OK;
  GS_REQUIRE(mean2d_grad && norm_sum && count, "null pointer");
  densify_stats_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      N, mean2d_grad, grad_stride, scale_x, scale_y, norm_sum, count, norm_max);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
