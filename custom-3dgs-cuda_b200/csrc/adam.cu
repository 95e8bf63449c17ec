// One Adam step over up to kAdamMaxGroups parameter tensors in a single launch.
//
// The update is torch.optim.Adam's (amsgrad off, no weight decay), which the reference's
// trainer uses with eps = 1e-15 (gaussian_splatting/utils/optim.py:31):
//   m = b1 m + (1 - b1) g (as m + (1 - b1)(g - m)),  v = b2 v + (1 - b2) g^2,
//   p -= (lr / (1 - b1^t)) m / (sqrt(v) / sqrt(1 - b2^t) + eps).
// Gradients come from one flat buffer and the moments live in flat buffers of the same
// layout, so a group's slice is contiguous everywhere; each CTA updates float4 chunks of one
// group (parameters, gradients and both moments read once and written once: 28 bytes per
// element of HBM traffic). A group may carry clamp bounds applied to the updated parameter in
// the same pass, as the reference trainer clamps the opacity logits and log-scales right after
// optimizer.step() (scripts/train.py:171-178): p = min(max(p, lo), hi).
#include <cmath>

#include "capi_internal.h"
#include "gs_common.cuh"

namespace gs {

constexpr int kAdamMaxGroups = 8;
constexpr int kAdamThreads = 256;
constexpr int kAdamVec = 4;                               // floats per thread and pass
constexpr int kAdamBlockItems = kAdamThreads * kAdamVec * 4;  // 4 float4 per thread

struct AdamParams {
  int n_groups;
  float* param[kAdamMaxGroups];
  long long offset[kAdamMaxGroups];     // start of the group in the flat buffers
  long long size[kAdamMaxGroups];
  unsigned block_start[kAdamMaxGroups + 1];
  float step_size[kAdamMaxGroups];      // lr / (1 - b1^t)
  float clamp_lo[kAdamMaxGroups], clamp_hi[kAdamMaxGroups];
  unsigned clamp_mask;                  // bit k: group k is clamped
  float bc2_sqrt;                       // sqrt(1 - b2^t)
  float beta1, beta2, one_minus_beta1, one_minus_beta2, eps;  // 1 - beta formed in double
  const float* grad;
  float* exp_avg;
  float* exp_avg_sq;
};

__device__ __forceinline__ float adam_one(float& p, float g, float& m, float& v, float step_size,
                                          const AdamParams& a, bool clamp, float lo, float hi) {
  m = m + a.one_minus_beta1 * (g - m);  // the lerp form torch uses
  v = a.beta2 * v + a.one_minus_beta2 * g * g;
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p -= step_size * (m / denom);
  if (clamp) p = fminf(fmaxf(p, lo), hi);
  return p;
}

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(AdamParams a) {
  int grp = 0;
#pragma unroll
  for (int k = 1; k < kAdamMaxGroups; ++k)
    if (k < a.n_groups && blockIdx.x >= a.block_start[k]) grp = k;
  const long long size = a.size[grp];
  const long long base = (long long)(blockIdx.x - a.block_start[grp]) * kAdamBlockItems;
  float* __restrict__ p = a.param[grp];
  const float* __restrict__ g = a.grad + a.offset[grp];
  float* __restrict__ m = a.exp_avg + a.offset[grp];
  float* __restrict__ v = a.exp_avg_sq + a.offset[grp];
  const float step_size = a.step_size[grp];
  const bool clamp = (a.clamp_mask >> grp) & 1u;
  const float lo = a.clamp_lo[grp], hi = a.clamp_hi[grp];
  // float4 path when every slice of the group is 16-byte aligned
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                     reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
#pragma unroll
  for (int r = 0; r < kAdamBlockItems / (kAdamThreads * kAdamVec); ++r) {
    const long long i = base + ((long long)r * kAdamThreads + threadIdx.x) * kAdamVec;
    if (i >= size) break;
    if (vec && i + kAdamVec <= size) {
      float4 pp = *reinterpret_cast<float4*>(p + i);
      const float4 gg = __ldg(reinterpret_cast<const float4*>(g + i));
      float4 mm = *reinterpret_cast<float4*>(m + i);
      float4 vv = *reinterpret_cast<float4*>(v + i);
      adam_one(pp.x, gg.x, mm.x, vv.x, step_size, a, clamp, lo, hi);
      adam_one(pp.y, gg.y, mm.y, vv.y, step_size, a, clamp, lo, hi);
      adam_one(pp.z, gg.z, mm.z, vv.z, step_size, a, clamp, lo, hi);
      adam_one(pp.w, gg.w, mm.w, vv.w, step_size, a, clamp, lo, hi);
      *reinterpret_cast<float4*>(p + i) = pp;
      *reinterpret_cast<float4*>(m + i) = mm;
      *reinterpret_cast<float4*>(v + i) = vv;
    } else {
      for (long long j = i; j < i + kAdamVec && j < size; ++j) {
        float pj = p[j], mj = m[j], vj = v[j];
        adam_one(pj, g[j], mj, vj, step_size, a, clamp, lo, hi);
        p[j] = pj;
        m[j] = mj;
        v[j] = vj;
      }
    }
  }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_adam_step(int n_groups, float* const* params, const long long* sizes,
                            const float* lrs, const float* grad, float* exp_avg,
                            float* exp_avg_sq, double beta1, double beta2, double eps, long long step,
                            const float* clamp_min, const float* clamp_max, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(n_groups >= 0 && n_groups <= kAdamMaxGroups, "n_groups must be in [0, 8]");
  GS_REQUIRE(step >= 1, "step must be >= 1");
  GS_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0,
             "betas must be in [0, 1)");
  if (n_groups == 0) return GS_OK;
  GS_REQUIRE(params && sizes && lrs && grad && exp_avg && exp_avg_sq, "null pointer");
  AdamParams a{};
  a.n_groups = n_groups;
  long long off = 0;
  unsigned blocks = 0;
  for (int k = 0; k < n_groups; ++k) {
    GS_REQUIRE(sizes[k] >= 0, "negative group size");
    GS_REQUIRE(sizes[k] == 0 || params[k], "null parameter pointer");
    a.param[k] = params[k];
    a.offset[k] = off;
    a.size[k] = sizes[k];
    a.block_start[k] = blocks;
    const long long nb = (sizes[k] + kAdamBlockItems - 1) / kAdamBlockItems;
    GS_REQUIRE((long long)blocks + nb < (1ll << 31), "too many elements");
    blocks += (unsigned)nb;
    off += sizes[k];
    const double bc1 = 1.0 - std::pow(beta1, (double)step);
    a.step_size[k] = (float)((double)lrs[k] / bc1);
    a.clamp_lo[k] = clamp_min ? clamp_min[k] : -INFINITY;
    a.clamp_hi[k] = clamp_max ? clamp_max[k] : INFINITY;
    GS_REQUIRE(!(a.clamp_lo[k] > a.clamp_hi[k]), "clamp_min above clamp_max");
    if (a.clamp_lo[k] > -INFINITY || a.clamp_hi[k] < INFINITY) a.clamp_mask |= 1u << k;
  }
  for (int k = n_groups; k < kAdamMaxGroups; ++k) a.block_start[k] = blocks;
  a.block_start[kAdamMaxGroups] = blocks;
  a.bc2_sqrt = (float)std::sqrt(1.0 - std::pow(beta2, (double)step));
  a.beta1 = (float)beta1;
  a.beta2 = (float)beta2;
  a.one_minus_beta1 = (float)(1.0 - beta1);
  a.one_minus_beta2 = (float)(1.0 - beta2);
  a.eps = (float)eps;
  a.grad = grad;
  a.exp_avg = exp_avg;
  a.exp_avg_sq = exp_avg_sq;
  if (blocks == 0) return GS_OK;
  adam_kernel<<<blocks, kAdamThreads, 0, (cudaStream_t)stream>>>(a);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
