// Degree 0..3 spherical-harmonic colour and its backward (device functions shared by the
// stand-alone SH kernels and the fused render kernels).
#pragma once

#include "gs_common.cuh"

namespace gs {

constexpr int kShRest = 15;              // coefficients of degrees 1..3
constexpr int kShRestFloats = kShRest * 3;

// The 15 real SH basis functions of degrees 1..3 at a unit direction (x, y, z), in the
// Inria 3DGS order (the reference evaluates the same polynomials at
// csrc/forward/SH.cu:31-55).
__device__ __forceinline__ void sh_basis(float x, float y, float z, float* Y) {
  Y[0] = -kShC1 * y;
  Y[1] = kShC1 * z;
  Y[2] = -kShC1 * x;
  const float xx = x * x, yy = y * y, zz = z * z;
  const float xy = x * y, yz = y * z, xz = x * z;
  Y[3] = kShC2_0 * xy;
  Y[4] = kShC2_1 * yz;
  Y[5] = kShC2_2 * (2.0f * zz - xx - yy);
  Y[6] = kShC2_3 * xz;
  Y[7] = kShC2_4 * (xx - yy);
  Y[8] = kShC3_0 * y * (3.0f * xx - yy);
  Y[9] = kShC3_1 * xy * z;
  Y[10] = kShC3_2 * y * (4.0f * zz - xx - yy);
  Y[11] = kShC3_3 * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  Y[12] = kShC3_4 * x * (4.0f * zz - xx - yy);
  Y[13] = kShC3_5 * z * (xx - yy);
  Y[14] = kShC3_6 * x * (xx - 3.0f * yy);
}

// Unclamped colour 0.5 + C0 * A + sum_k Y_k k_j[k] (csrc/forward/SH.cu:80-85).
__device__ __forceinline__ float3 sh_unclamped(const float* Y, float3 A, const float* kj) {
  float3 rgb = make_float3(0.5f + kShC0 * A.x, 0.5f + kShC0 * A.y, 0.5f + kShC0 * A.z);
#pragma unroll
  for (int k = 0; k < kShRest; ++k) {
    rgb.x += Y[k] * kj[k * 3 + 0];
    rgb.y += Y[k] * kj[k * 3 + 1];
    rgb.z += Y[k] * kj[k * 3 + 2];
  }
  return rgb;
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.0f), 1.0f); }

// View direction for the forward colour: (mu - cam) / |mu - cam|, the length taken as
// 1 / sqrt((dx^2 + dy^2) + dz^2) without an epsilon (csrc/forward/SH.cu:73-74).
__device__ __forceinline__ float3 sh_forward_direction(float3 mu, float3 cam) {
  const float vx = mu.x - cam.x, vy = mu.y - cam.y, vz = mu.z - cam.z;
  const float inv = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz);
  return make_float3(vx * inv, vy * inv, vz * inv);
}

// dL/d(direction) from dL/dY (csrc/backward/delight_backward.cu:50-105).
__device__ __forceinline__ float3 sh_basis_backward(float x, float y, float z,
                                                    const float* dY) {
  const float xx = x * x, yy = y * y, zz = z * z;
  float gx = 0.0f, gy = 0.0f, gz = 0.0f;
  gy += dY[0] * (-kShC1);
  gz += dY[1] * kShC1;
  gx += dY[2] * (-kShC1);
  gx += dY[3] * (kShC2_0 * y);
  gy += dY[3] * (kShC2_0 * x);
  gy += dY[4] * (kShC2_1 * z);
  gz += dY[4] * (kShC2_1 * y);
  gx += dY[5] * (-2.0f * kShC2_2 * x);
  gy += dY[5] * (-2.0f * kShC2_2 * y);
  gz += dY[5] * (4.0f * kShC2_2 * z);
  gx += dY[6] * (kShC2_3 * z);
  gz += dY[6] * (kShC2_3 * x);
  gx += dY[7] * (2.0f * kShC2_4 * x);
  gy += dY[7] * (-2.0f * kShC2_4 * y);
  gx += dY[8] * (kShC3_0 * y * 6.0f * x);
  gy += dY[8] * (kShC3_0 * (3.0f * xx - 3.0f * yy));
  gx += dY[9] * (kShC3_1 * y * z);
  gy += dY[9] * (kShC3_1 * x * z);
  gz += dY[9] * (kShC3_1 * x * y);
  gx += dY[10] * (kShC3_2 * y * (-2.0f * x));
  gy += dY[10] * (kShC3_2 * (4.0f * zz - xx - 3.0f * yy));
  gz += dY[10] * (kShC3_2 * y * 8.0f * z);
  gx += dY[11] * (kShC3_3 * z * (-6.0f * x));
  gy += dY[11] * (kShC3_3 * z * (-6.0f * y));
  gz += dY[11] * (kShC3_3 * (6.0f * zz - 3.0f * xx - 3.0f * yy));
  gx += dY[12] * (kShC3_4 * (4.0f * zz - 3.0f * xx - yy));
  gy += dY[12] * (kShC3_4 * x * (-2.0f * y));
  gz += dY[12] * (kShC3_4 * x * 8.0f * z);
  gx += dY[13] * (kShC3_5 * z * 2.0f * x);
  gy += dY[13] * (kShC3_5 * z * (-2.0f * y));
  gz += dY[13] * (kShC3_5 * (xx - yy));
  gx += dY[14] * (kShC3_6 * (3.0f * xx - 3.0f * yy));
  gy += dY[14] * (kShC3_6 * x * (-6.0f * y));
  return make_float3(gx, gy, gz);
}

// Backward of the SH colour for one Gaussian (csrc/backward/delight_backward.cu:121-173).
// The direction is re-derived with rsqrt(|v|^2 + 1e-8); the colour gradient is zeroed per
// channel where the unclamped colour lies outside [0, 1]. Writes dL/dA (3), dL/dk_j (45)
// and returns dL/dmu.
__device__ __forceinline__ float3 sh_backward(float3 gcol, float3 mu, float3 cam, float3 A,
                                              const float* kj, float3& gA, float* gkj) {
  const float vx = mu.x - cam.x, vy = mu.y - cam.y, vz = mu.z - cam.z;
  const float inv_len = rsqrtf(vx * vx + vy * vy + vz * vz + 1e-8f);
  const float dx = vx * inv_len, dy = vy * inv_len, dz = vz * inv_len;
  float Y[kShRest];
  sh_basis(dx, dy, dz, Y);
  const float3 rgb = sh_unclamped(Y, A, kj);
  const float g0 = (rgb.x < 0.0f || rgb.x > 1.0f) ? 0.0f : gcol.x;
  const float g1 = (rgb.y < 0.0f || rgb.y > 1.0f) ? 0.0f : gcol.y;
  const float g2 = (rgb.z < 0.0f || rgb.z > 1.0f) ? 0.0f : gcol.z;
  gA = make_float3(g0 * kShC0, g1 * kShC0, g2 * kShC0);
  float dY[kShRest];
#pragma unroll
  for (int k = 0; k < kShRest; ++k) {
    gkj[k * 3 + 0] = g0 * Y[k];
    gkj[k * 3 + 1] = g1 * Y[k];
    gkj[k * 3 + 2] = g2 * Y[k];
    dY[k] = g0 * kj[k * 3 + 0] + g1 * kj[k * 3 + 1] + g2 * kj[k * 3 + 2];
  }
  const float3 gd = sh_basis_backward(dx, dy, dz, dY);
  const float ddot = dx * gd.x + dy * gd.y + dz * gd.z;
  return make_float3(inv_len * (gd.x - dx * ddot), inv_len * (gd.y - dy * ddot),
                     inv_len * (gd.z - dz * ddot));
}

// sh_backward on a staged coefficient row: reads the 45 coefficients from `kj` (shared memory)
// and overwrites them with dL/dk_j; the arithmetic and its order are those of sh_backward, so
// the results are identical, without holding the row in registers.
__device__ __forceinline__ float3 sh_backward_inplace(float3 gcol, float3 mu, float3 cam,
                                                      float3 A, float* kj, float3& gA) {
  const float vx = mu.x - cam.x, vy = mu.y - cam.y, vz = mu.z - cam.z;
  const float inv_len = rsqrtf(vx * vx + vy * vy + vz * vz + 1e-8f);
  const float dx = vx * inv_len, dy = vy * inv_len, dz = vz * inv_len;
  float Y[kShRest];
  sh_basis(dx, dy, dz, Y);
  const float3 rgb = sh_unclamped(Y, A, kj);
  const float g0 = (rgb.x < 0.0f || rgb.x > 1.0f) ? 0.0f : gcol.x;
  const float g1 = (rgb.y < 0.0f || rgb.y > 1.0f) ? 0.0f : gcol.y;
  const float g2 = (rgb.z < 0.0f || rgb.z > 1.0f) ? 0.0f : gcol.z;
  gA = make_float3(g0 * kShC0, g1 * kShC0, g2 * kShC0);
  float dY[kShRest];
#pragma unroll
  for (int k = 0; k < kShRest; ++k) {
    const float k0 = kj[k * 3 + 0], k1 = kj[k * 3 + 1], k2 = kj[k * 3 + 2];
    kj[k * 3 + 0] = g0 * Y[k];
    kj[k * 3 + 1] = g1 * Y[k];
    kj[k * 3 + 2] = g2 * Y[k];
    dY[k] = g0 * k0 + g1 * k1 + g2 * k2;
  }
  const float3 gd = sh_basis_backward(dx, dy, dz, dY);
  const float ddot = dx * gd.x + dy * gd.y + dz * gd.z;
  return make_float3(inv_len * (gd.x - dx * ddot), inv_len * (gd.y - dy * ddot),
                     inv_len * (gd.z - dz * ddot));
}

// sh_backward_inplace for one of several views: the coefficients kj are left unchanged and
// this view's dL/dk_j (the values sh_backward_inplace writes, each rounded as a product) is
// added to gkj, so that views summed in order give what one in-place call per view, summed
// into a buffer in the same order, gives.
__device__ __forceinline__ float3 sh_backward_accumulate(float3 gcol, float3 mu, float3 cam,
                                                         float3 A, const float* kj,
                                                         float* gkj, float3& gA) {
  const float vx = mu.x - cam.x, vy = mu.y - cam.y, vz = mu.z - cam.z;
  const float inv_len = rsqrtf(vx * vx + vy * vy + vz * vz + 1e-8f);
  const float dx = vx * inv_len, dy = vy * inv_len, dz = vz * inv_len;
  float Y[kShRest];
  sh_basis(dx, dy, dz, Y);
  const float3 rgb = sh_unclamped(Y, A, kj);
  const float g0 = (rgb.x < 0.0f || rgb.x > 1.0f) ? 0.0f : gcol.x;
  const float g1 = (rgb.y < 0.0f || rgb.y > 1.0f) ? 0.0f : gcol.y;
  const float g2 = (rgb.z < 0.0f || rgb.z > 1.0f) ? 0.0f : gcol.z;
  gA = make_float3(g0 * kShC0, g1 * kShC0, g2 * kShC0);
  float dY[kShRest];
#pragma unroll
  for (int k = 0; k < kShRest; ++k) {
    const float k0 = kj[k * 3 + 0], k1 = kj[k * 3 + 1], k2 = kj[k * 3 + 2];
    gkj[k * 3 + 0] = __fadd_rn(gkj[k * 3 + 0], __fmul_rn(g0, Y[k]));
    gkj[k * 3 + 1] = __fadd_rn(gkj[k * 3 + 1], __fmul_rn(g1, Y[k]));
    gkj[k * 3 + 2] = __fadd_rn(gkj[k * 3 + 2], __fmul_rn(g2, Y[k]));
    dY[k] = g0 * k0 + g1 * k1 + g2 * k2;
  }
  const float3 gd = sh_basis_backward(dx, dy, dz, dY);
  const float ddot = dx * gd.x + dy * gd.y + dz * gd.z;
  return make_float3(inv_len * (gd.x - dx * ddot), inv_len * (gd.y - dy * ddot),
                     inv_len * (gd.z - dz * ddot));
}

}  // namespace gs
