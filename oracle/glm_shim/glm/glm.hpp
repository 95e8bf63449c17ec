// Minimal stand-in for the GLM (g-truc/glm) API subset that the reference's
// csrc/forward/projection.cu, csrc/forward/SH.cu, csrc/backward/projection_backward.cu and
// csrc/backward/delight_backward.cu use. TEST INFRASTRUCTURE ONLY: oracle/build_ref.py puts
// this directory on the include path so that those four files compile UNMODIFIED into the
// "ref+shim" build of the reference extension; nothing in the product includes it.
//
// GLM itself is header-only, not vendored by the reference, and pinned to no version
// (reference setup.py:18-28, README.md:60-75); it is absent from this image. This header is
// written from GLM's documented (GLSL-style) semantics, not from its sources:
//   * matCxR has C columns of R rows; constructors take the entries column by column;
//     m[c] is column c and m[c][r] its row-r entry;
//   * A * B is the linear-algebra product; every entry is a dot product summed over the
//     shared index in increasing order, left to right; mat * vec likewise;
//   * scalar op vec, vec op scalar and scalar * mat are component-wise;
//   * dot(a, b) sums the component products in index order; normalize(v) = v * (1 / sqrt(
//     dot(v, v)));
//   * quat(w, x, y, z) takes the real part first; dot(q, q) = (w*w + x*x) + (y*y + z*z);
//     normalize(q) multiplies every component by 1 / length(q) and maps a quaternion of
//     length <= 0 to the identity (1, 0, 0, 0); toMat3(q) is the rotation matrix of the
//     unit quaternion q (the standard formula, column by column).
// Results built against this header are labelled "ref+shim": the reference's own expressions
// with this restatement of the library underneath.
#pragma once

#include <cmath>
#include <type_traits>

#if defined(__CUDACC__)
#define GS_GLM_FN __host__ __device__ inline
#else
#define GS_GLM_FN inline
#endif

namespace glm {

// ---------------------------------------------------------------------------------------
// vectors
template <int L>
struct vec {
  float v[L];
  GS_GLM_FN vec() {
    for (int i = 0; i < L; ++i) v[i] = 0.0f;
  }
  GS_GLM_FN float& operator[](int i) { return v[i]; }
  GS_GLM_FN const float& operator[](int i) const { return v[i]; }
};

template <>
struct vec<2> {
  float x, y;
  GS_GLM_FN vec() : x(0.0f), y(0.0f) {}
  GS_GLM_FN explicit vec(float s) : x(s), y(s) {}
  GS_GLM_FN vec(float a, float b) : x(a), y(b) {}
  GS_GLM_FN float& operator[](int i) { return i == 0 ? x : y; }
  GS_GLM_FN const float& operator[](int i) const { return i == 0 ? x : y; }
};

template <>
struct vec<3> {
  float x, y, z;
  GS_GLM_FN vec() : x(0.0f), y(0.0f), z(0.0f) {}
  GS_GLM_FN explicit vec(float s) : x(s), y(s), z(s) {}
  GS_GLM_FN vec(float a, float b, float c) : x(a), y(b), z(c) {}
  GS_GLM_FN float& operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
  GS_GLM_FN const float& operator[](int i) const { return i == 0 ? x : (i == 1 ? y : z); }
  GS_GLM_FN vec& operator+=(const vec& o) {
    x += o.x;
    y += o.y;
    z += o.z;
    return *this;
  }
};

using vec2 = vec<2>;
using vec3 = vec<3>;

GS_GLM_FN vec3 operator+(const vec3& a, const vec3& b) { return vec3(a.x + b.x, a.y + b.y, a.z + b.z); }
GS_GLM_FN vec3 operator-(const vec3& a, const vec3& b) { return vec3(a.x - b.x, a.y - b.y, a.z - b.z); }
GS_GLM_FN vec3 operator*(const vec3& a, float s) { return vec3(a.x * s, a.y * s, a.z * s); }
GS_GLM_FN vec3 operator*(float s, const vec3& a) { return vec3(s * a.x, s * a.y, s * a.z); }
GS_GLM_FN vec3 operator+(float s, const vec3& a) { return vec3(s + a.x, s + a.y, s + a.z); }

GS_GLM_FN float dot(const vec3& a, const vec3& b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

GS_GLM_FN vec3 normalize(const vec3& a) {
  const float inv = 1.0f / std::sqrt(dot(a, a));
  return a * inv;
}

// ---------------------------------------------------------------------------------------
// matrices: C columns of R rows
template <int C, int R>
struct mat {
  vec<R> col[C];
  GS_GLM_FN mat() {}
  // C * R entries, column by column
  template <typename... F, typename = std::enable_if_t<sizeof...(F) == C * R && (C * R > 1)>>
  GS_GLM_FN mat(F... e) {
    const float flat[C * R] = {static_cast<float>(e)...};
    for (int c = 0; c < C; ++c)
      for (int r = 0; r < R; ++r) col[c][r] = flat[c * R + r];
  }
  GS_GLM_FN vec<R>& operator[](int c) { return col[c]; }
  GS_GLM_FN const vec<R>& operator[](int c) const { return col[c]; }
};

using mat2 = mat<2, 2>;
using mat3 = mat<3, 3>;
using mat3x2 = mat<3, 2>;
using mat2x3 = mat<2, 3>;

// (R x K) * (K x C): entry (row r, column c) = sum over k of a(r, k) * b(k, c), k ascending.
template <int K, int R, int C>
GS_GLM_FN mat<C, R> operator*(const mat<K, R>& a, const mat<C, K>& b) {
  mat<C, R> out;
  for (int c = 0; c < C; ++c)
    for (int r = 0; r < R; ++r) {
      float s = a[0][r] * b[c][0];
      for (int k = 1; k < K; ++k) s = s + a[k][r] * b[c][k];
      out[c][r] = s;
    }
  return out;
}

GS_GLM_FN vec3 operator*(const mat3& m, const vec3& x) {
  vec3 out;
  for (int r = 0; r < 3; ++r) out[r] = m[0][r] * x.x + m[1][r] * x.y + m[2][r] * x.z;
  return out;
}

template <int C, int R>
GS_GLM_FN mat<C, R> operator*(float s, const mat<C, R>& m) {
  mat<C, R> out;
  for (int c = 0; c < C; ++c)
    for (int r = 0; r < R; ++r) out[c][r] = s * m[c][r];
  return out;
}

template <int C, int R>
GS_GLM_FN mat<R, C> transpose(const mat<C, R>& m) {
  mat<R, C> out;
  for (int c = 0; c < C; ++c)
    for (int r = 0; r < R; ++r) out[r][c] = m[c][r];
  return out;
}

// ---------------------------------------------------------------------------------------
// quaternions
struct quat {
  float x, y, z, w;
  GS_GLM_FN quat() : x(0.0f), y(0.0f), z(0.0f), w(1.0f) {}
  GS_GLM_FN quat(float w_, float x_, float y_, float z_) : x(x_), y(y_), z(z_), w(w_) {}
};

GS_GLM_FN float dot(const quat& a, const quat& b) {
  return (a.w * b.w + a.x * b.x) + (a.y * b.y + a.z * b.z);
}

GS_GLM_FN quat normalize(const quat& q) {
  const float len = std::sqrt(dot(q, q));
  if (len <= 0.0f) return quat(1.0f, 0.0f, 0.0f, 0.0f);
  const float inv = 1.0f / len;
  return quat(q.w * inv, q.x * inv, q.y * inv, q.z * inv);
}

GS_GLM_FN mat3 toMat3(const quat& q) {
  const float xx = q.x * q.x, yy = q.y * q.y, zz = q.z * q.z;
  const float xz = q.x * q.z, xy = q.x * q.y, yz = q.y * q.z;
  const float wx = q.w * q.x, wy = q.w * q.y, wz = q.w * q.z;
  mat3 m;
  m[0][0] = 1.0f - 2.0f * (yy + zz);
  m[0][1] = 2.0f * (xy + wz);
  m[0][2] = 2.0f * (xz - wy);
  m[1][0] = 2.0f * (xy - wz);
  m[1][1] = 1.0f - 2.0f * (xx + zz);
  m[1][2] = 2.0f * (yz + wx);
  m[2][0] = 2.0f * (xz + wy);
  m[2][1] = 2.0f * (yz - wx);
  m[2][2] = 1.0f - 2.0f * (xx + yy);
  return m;
}

}  // namespace glm
