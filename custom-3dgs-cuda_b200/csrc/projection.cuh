// Per-Gaussian projection math (world -> camera -> screen, 3D -> 2D covariance) and its
// backward. Device functions shared by the stand-alone projection kernels and the fused
// render kernels.
#pragma once

#include "gs_common.cuh"

namespace gs {

struct Camera {
  float r[9];  // world->camera rotation, row-major
  float t[3];
  float fx, fy, cx, cy;
};

__device__ __forceinline__ void load_camera(const float* R, const float* t, float fx, float fy,
                                            float cx, float cy, Camera& cam) {
#pragma unroll
  for (int i = 0; i < 9; ++i) cam.r[i] = __ldg(R + i);
#pragma unroll
  for (int i = 0; i < 3; ++i) cam.t[i] = __ldg(t + i);
  cam.fx = fx;
  cam.fy = fy;
  cam.cx = cx;
  cam.cy = cy;
}

// Camera-space position R mu + t. Each row is evaluated as (r0*x + r1*y + r2*z) + t, the
// expression tree of a column-major mat3 * vec3 followed by a vec3 add
// (csrc/forward/projection.cu:44).
__device__ __forceinline__ float3 world_to_camera(const Camera& cam, float x, float y,
                                                  float z) {
  float3 c;
  c.x = cam.r[0] * x + cam.r[1] * y + cam.r[2] * z + cam.t[0];
  c.y = cam.r[3] * x + cam.r[4] * y + cam.r[5] * z + cam.t[1];
  c.z = cam.r[6] * x + cam.r[7] * y + cam.r[8] * z + cam.t[2];
  return c;
}

constexpr float kNearCull = 0.2f;  // csrc/forward/projection.cu:47

// Rotation matrix (row-major) of the normalised quaternion (w,x,y,z): the reference's
// glm::toMat3(glm::normalize(quat(w,x,y,z))) (csrc/forward/projection.cu:64-65). Normalisation
// multiplies by 1 / sqrt((w^2 + x^2) + (y^2 + z^2)) and maps a zero quaternion to the identity;
// the entries are the standard unit-quaternion rotation. Every rounding step is written with an
// explicit intrinsic, in the order the reference's build evaluates it (each sum of two products
// fuses its first product; the (0,0) entry adds the two rounded squares), so the compiler
// cannot re-associate or re-fuse them differently in different kernels: the rotation, and with
// it the 2D covariance, is bit-identical to the reference's.
__device__ __forceinline__ void quat_to_rotation(float qw, float qx, float qy, float qz,
                                                 float* Rq, float4& qn) {
  const float dot = __fadd_rn(__fmaf_rn(qw, qw, __fmul_rn(qx, qx)),
                              __fmaf_rn(qy, qy, __fmul_rn(qz, qz)));
  const float len = sqrtf(dot);
  float w, x, y, z;
  if (len <= 0.0f) {
    w = 1.0f; x = 0.0f; y = 0.0f; z = 0.0f;
  } else {
    const float inv = __fdiv_rn(1.0f, len);
    w = __fmul_rn(qw, inv); x = __fmul_rn(qx, inv); y = __fmul_rn(qy, inv); z = __fmul_rn(qz, inv);
  }
  qn = make_float4(w, x, y, z);
  const float yy = __fmul_rn(y, y), zz = __fmul_rn(z, z);
  const float wx = __fmul_rn(w, x), wy = __fmul_rn(w, y), wz = __fmul_rn(w, z);
  Rq[0] = __fmaf_rn(-2.0f, __fadd_rn(yy, zz), 1.0f);
  Rq[3] = 2.0f * __fmaf_rn(x, y, wz);
  Rq[6] = 2.0f * __fmaf_rn(x, z, -wy);
  Rq[1] = 2.0f * __fmaf_rn(x, y, -wz);
  Rq[4] = __fmaf_rn(-2.0f, __fmaf_rn(x, x, zz), 1.0f);
  Rq[7] = 2.0f * __fmaf_rn(y, z, wx);
  Rq[2] = 2.0f * __fmaf_rn(x, z, wy);
  Rq[5] = 2.0f * __fmaf_rn(y, z, -wx);
  Rq[8] = __fmaf_rn(-2.0f, __fmaf_rn(x, x, yy), 1.0f);
}

// C = A * B for row-major 3x3 matrices, each entry summed over k = 0, 1, 2 in order.
__device__ __forceinline__ void mat3_mul(const float* A, const float* B, float* C) {
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      C[r * 3 + c] = A[r * 3 + 0] * B[0 * 3 + c] + A[r * 3 + 1] * B[1 * 3 + c] +
                     A[r * 3 + 2] * B[2 * 3 + c];
}

// C = A * B^T for row-major 3x3 matrices.
__device__ __forceinline__ void mat3_mul_bt(const float* A, const float* B, float* C) {
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      C[r * 3 + c] = A[r * 3 + 0] * B[c * 3 + 0] + A[r * 3 + 1] * B[c * 3 + 1] +
                     A[r * 3 + 2] * B[c * 3 + 2];
}

struct Projected {
  float2 mean;
  float3 cov;  // (a, b, c)
  float depth;
};

// Forward projection of one Gaussian (csrc/forward/projection.cu:33-105). Returns false for
// Gaussians at z <= 0.2, whose outputs are all zero.
__device__ __forceinline__ bool project_gaussian(const Camera& cam, float mx, float my,
                                                 float mz, float4 q, float3 logs,
                                                 Projected& out) {
  float3 pc = world_to_camera(cam, mx, my, mz);
  if (pc.z <= kNearCull) {
    out.mean = make_float2(0.0f, 0.0f);
    out.cov = make_float3(0.0f, 0.0f, 0.0f);
    out.depth = 0.0f;
    return false;
  }
  out.depth = pc.z;
  out.mean = make_float2((cam.fx * pc.x) / pc.z + cam.cx, (cam.fy * pc.y) / pc.z + cam.cy);

  float Rq[9];
  float4 qn;
  quat_to_rotation(q.x, q.y, q.z, q.w, Rq, qn);
  const float sx = expf(logs.x), sy = expf(logs.y), sz = expf(logs.z);
  // M = Rq * diag(s): each column of Rq scaled (products with the zero entries of the
  // diagonal add signed zeros only, so they are left out).
  float M[9];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    M[r * 3 + 0] = Rq[r * 3 + 0] * sx;
    M[r * 3 + 1] = Rq[r * 3 + 1] * sy;
    M[r * 3 + 2] = Rq[r * 3 + 2] * sz;
  }
  float Sw[9], T[9], Sc[9];
  mat3_mul_bt(M, M, Sw);          // Sigma_world = M M^T
  mat3_mul(cam.r, Sw, T);         // R_cam Sigma_world
  mat3_mul_bt(T, cam.r, Sc);      // (R_cam Sigma_world) R_cam^T

  const float z = pc.z;
  const float z2 = z * z;
  const float J00 = cam.fx / z;
  const float J02 = -(cam.fx * pc.x) / z2;
  const float J11 = cam.fy / z;
  const float J12 = -(cam.fy * pc.y) / z2;
  // Row-major Sc[r*3+c]; the reference indexes the column-major Sigma_cam[c][r]
  // (csrc/forward/projection.cu:91-98).
  float a = J00 * (J00 * Sc[0] + J02 * Sc[2]) + J02 * (J00 * Sc[6] + J02 * Sc[8]);
  float b = J00 * (J11 * Sc[3] + J12 * Sc[6]) + J02 * (J11 * Sc[5] + J12 * Sc[8]);
  float c = J11 * (J11 * Sc[4] + J12 * Sc[7]) + J12 * (J11 * Sc[5] + J12 * Sc[8]);
  a += 0.3f;
  c += 0.3f;
  out.cov = make_float3(a, b, c);
  return true;
}

struct ProjectionGrad {
  float3 mu;
  float4 q;  // (w,x,y,z)
  float3 s;
};

// Backward of project_gaussian (csrc/backward/projection_backward.cu:33-138): chain rule
// through J, R_cam, M = R S, exp(s) and the quaternion normalisation
// (rsqrt(|q|^2 + 1e-8)). dL/dSigma2 arrives packed as (a, b, c) with b the shared
// off-diagonal, so the symmetric gradient is [[ga, gb/2], [gb/2, gc]].
// The quaternion gradient is the derivative of quat_to_rotation.
__device__ __forceinline__ void project_gaussian_backward(const Camera& cam, float mx,
                                                         float my, float mz, float4 q,
                                                         float3 logs, float2 gmean,
                                                         float3 gcov, ProjectionGrad& g) {
  float3 pc = world_to_camera(cam, mx, my, mz);
  if (pc.z <= kNearCull) {
    g.mu = make_float3(0.0f, 0.0f, 0.0f);
    g.q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    g.s = make_float3(0.0f, 0.0f, 0.0f);
    return;
  }
  const float z = pc.z, z2 = z * z, z3 = z2 * z;
  const float fx = cam.fx, fy = cam.fy;
  float dmc_x = (fx / z) * gmean.x;
  float dmc_y = (fy / z) * gmean.y;
  float dmc_z = (-fx * pc.x / z2) * gmean.x + (-fy * pc.y / z2) * gmean.y;

  const float J00 = fx / z, J02 = -(fx * pc.x) / z2;
  const float J11 = fy / z, J12 = -(fy * pc.y) / z2;
  const float G00 = gcov.x, G01 = 0.5f * gcov.y, G11 = gcov.z;

  float Rq[9];
  float4 qn;
  quat_to_rotation(q.x, q.y, q.z, q.w, Rq, qn);
  const float sx = expf(logs.x), sy = expf(logs.y), sz = expf(logs.z);
  const float sv[3] = {sx, sy, sz};
  float M[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) M[r * 3 + c] = Rq[r * 3 + c] * sv[c];
  float Sw[9], T[9], Sc[9];
  mat3_mul_bt(M, M, Sw);
  mat3_mul(cam.r, Sw, T);
  mat3_mul_bt(T, cam.r, Sc);

  // dSigma_cam = J^T G J with J = [[J00, 0, J02], [0, J11, J12]].
  float GJ[6];  // G J (2x3)
  GJ[0] = G00 * J00;               GJ[1] = G01 * J11;               GJ[2] = G00 * J02 + G01 * J12;
  GJ[3] = G01 * J00;               GJ[4] = G11 * J11;               GJ[5] = G01 * J02 + G11 * J12;
  const float Jc[6] = {J00, 0.0f, J02, 0.0f, J11, J12};
  float dSc[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) dSc[r * 3 + c] = Jc[r] * GJ[c] + Jc[3 + r] * GJ[3 + c];
  // dSigma_world = R_cam^T dSigma_cam R_cam
  float U[9], dSw[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      U[r * 3 + c] = cam.r[0 * 3 + r] * dSc[0 * 3 + c] + cam.r[1 * 3 + r] * dSc[1 * 3 + c] +
                     cam.r[2 * 3 + r] * dSc[2 * 3 + c];
  mat3_mul(U, cam.r, dSw);
  // dM = 2 dSigma_world M ; dRq = dM diag(s) ; dS_cc = (Rq^T dM)_cc
  float dM[9];
  mat3_mul(dSw, M, dM);
#pragma unroll
  for (int i = 0; i < 9; ++i) dM[i] *= 2.0f;
  float ds[3];
#pragma unroll
  for (int c = 0; c < 3; ++c)
    ds[c] = (Rq[0 * 3 + c] * dM[0 * 3 + c] + Rq[1 * 3 + c] * dM[1 * 3 + c] +
             Rq[2 * 3 + c] * dM[2 * 3 + c]) * sv[c];
  g.s = make_float3(ds[0], ds[1], ds[2]);
  float D[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) D[r * 3 + c] = dM[r * 3 + c] * sv[c];

  // dL/dJ = 2 G J Sigma_cam (2x3)
  float dJ[6];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      dJ[r * 3 + c] = 2.0f * (GJ[r * 3 + 0] * Sc[0 * 3 + c] + GJ[r * 3 + 1] * Sc[1 * 3 + c] +
                              GJ[r * 3 + 2] * Sc[2 * 3 + c]);
  const float dJ00 = dJ[0], dJ02 = dJ[2], dJ11 = dJ[4], dJ12 = dJ[5];
  dmc_x += dJ02 * (-fx / z2);
  dmc_y += dJ12 * (-fy / z2);
  dmc_z += dJ00 * (-fx / z2) + dJ11 * (-fy / z2) + dJ02 * (2.0f * fx * pc.x / z3) +
           dJ12 * (2.0f * fy * pc.y / z3);
  g.mu.x = cam.r[0] * dmc_x + cam.r[3] * dmc_y + cam.r[6] * dmc_z;
  g.mu.y = cam.r[1] * dmc_x + cam.r[4] * dmc_y + cam.r[7] * dmc_z;
  g.mu.z = cam.r[2] * dmc_x + cam.r[5] * dmc_y + cam.r[8] * dmc_z;

  // d rotation / d unit quaternion (w,x,y,z), rotation as in quat_to_rotation.
  const float w = qn.x, x = qn.y, y = qn.z, zq = qn.w;
  const float dw = 2.0f * (zq * (D[3] - D[1]) + y * (D[2] - D[6]) + x * (D[7] - D[5]));
  const float dx = 2.0f * (y * (D[1] + D[3]) + zq * (D[2] + D[6]) + w * (D[7] - D[5])) -
                   4.0f * x * (D[4] + D[8]);
  const float dy = 2.0f * (x * (D[1] + D[3]) + w * (D[2] - D[6]) + zq * (D[5] + D[7])) -
                   4.0f * y * (D[0] + D[8]);
  const float dz = 2.0f * (w * (D[3] - D[1]) + x * (D[2] + D[6]) + y * (D[5] + D[7])) -
                   4.0f * zq * (D[0] + D[4]);
  // through normalisation: (I - q q^T) / |q|
  const float inv_norm = rsqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w + 1e-8f);
  const float qdot = w * dw + x * dx + y * dy + zq * dz;
  g.q = make_float4(inv_norm * (dw - w * qdot), inv_norm * (dx - x * qdot),
                    inv_norm * (dy - y * qdot), inv_norm * (dz - zq * qdot));
}

}  // namespace gs
