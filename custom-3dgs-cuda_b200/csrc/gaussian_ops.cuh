// Warp-cooperative row staging between HBM and shared memory for [N, F] fp32 arrays.
#pragma once

#include "gs_common.cuh"

namespace gs {

// Copies rows [row0, row0 + 32) (clipped to n_rows) of a row-major [n_rows, F] array into
// `stage` (32 * F floats, 16-byte aligned). Full, 16-byte aligned chunks move as float4
// streaming loads; partial or unaligned chunks fall back to scalar loads.
template <int F>
__device__ __forceinline__ void warp_load_rows(const float* __restrict__ src, int row0,
                                               int n_rows, float* stage) {
  const int lane = threadIdx.x & 31;
  const int rows = min(32, n_rows - row0);
  const float* base = src + (size_t)row0 * F;
  if (rows == 32 && (32 * F) % 4 == 0 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0u) {
    const float4* b4 = reinterpret_cast<const float4*>(base);
    float4* s4 = reinterpret_cast<float4*>(stage);
#pragma unroll 4
    for (int i = lane; i < 32 * F / 4; i += 32) s4[i] = __ldcs(b4 + i);
  } else {
    const int n = rows * F;
    for (int i = lane; i < n; i += 32) stage[i] = __ldcs(base + i);
  }
  __syncwarp();
}

// Asynchronous form of warp_load_rows for a full, 16-byte aligned group of 32 rows: issues
// cp.async copies into `stage` and returns true (the caller waits with cp.async.wait_group and
// __syncwarp before reading); returns false, issuing nothing, for any other group.
template <int F>
__device__ __forceinline__ bool warp_prefetch_rows(const float* __restrict__ src, int row0,
                                                   int n_rows, float* stage) {
  const int lane = threadIdx.x & 31;
  const float* base = src + (size_t)row0 * F;
  if (n_rows - row0 < 32 || (32 * F) % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(base) & 15u) != 0u)
    return false;
  const unsigned s0 = (unsigned)__cvta_generic_to_shared(stage);
  for (int i = lane; i < 32 * F / 4; i += 32)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s0 + 16u * i),
                 "l"(base + 4 * i)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
  return true;
}

// Inverse of warp_load_rows: writes rows [row0, row0 + 32) (clipped) from `stage`.
template <int F>
__device__ __forceinline__ void warp_store_rows(float* __restrict__ dst, int row0, int n_rows,
                                                const float* stage) {
  const int lane = threadIdx.x & 31;
  const int rows = min(32, n_rows - row0);
  float* base = dst + (size_t)row0 * F;
  if (rows == 32 && (32 * F) % 4 == 0 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0u) {
    float4* b4 = reinterpret_cast<float4*>(base);
    const float4* s4 = reinterpret_cast<const float4*>(stage);
#pragma unroll 4
    for (int i = lane; i < 32 * F / 4; i += 32) __stcs(b4 + i, s4[i]);
  } else {
    const int n = rows * F;
    for (int i = lane; i < n; i += 32) __stcs(base + i, stage[i]);
  }
}

}  // namespace gs
