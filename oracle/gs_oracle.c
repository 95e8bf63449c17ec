/*
 * gs_oracle.c - CPU restatement of the reference rasterizer path (kmurungi/custom-3dgs-cuda:
 * the csrc/forward and csrc/backward kernels). TEST INFRASTRUCTURE ONLY: the parity tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg call it as the checker; the
 * product never links it.
 *
 * Arithmetic model. The reference is fp32 CUDA compiled with nvcc's default --fmad=true,
 * which contracts a*b + c into fused multiply-adds. This file is compiled with
 * -ffp-contract=off and writes the contraction out with fmaf() where nvcc forms one:
 *   x*y + z   -> fmaf(x, y, z)         z + x*y -> fmaf(x, y, z)
 *   a*b + c*d -> fmaf(a, b, c*d)       (the left product is fused)
 *   a*b - c*d -> fmaf(a, b, -(c*d))    x - y*z -> fmaf(-y, z, x)
 * IEEE division and square root are correctly rounded on both sides. __expf (an
 * approximate exponential on the GPU) is modelled by expf, so opacity-threshold and
 * transmittance-threshold decisions that fall within a few ulp of their thresholds are
 * reported per pixel in `ambiguous` instead of being trusted.
 *
 * Parity status: binning, sorting and blending are pinned against the reference's own
 * rasterize.cu / rasterize_backward.cu (built unmodified into oracle/_ref and run on a
 * B200 to produce tests/golden/). The projection and SH code of the reference needs GLM,
 * which is absent, so those forward values follow GLM's documented column-major semantics
 * and are pinned only by the reference's gradient checks and closed-form cases.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TILE 16

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------------------------------
 * Projection forward: csrc/forward/projection.cu:28-105 (GLM mat3 = column-major).
 * ------------------------------------------------------------------------------------- */
static void proj_camera(const float* R, const float* t, float x, float y, float z, float* c) {
  /* glm mat3 * vec3: ((m00 x + m10 y) + m20 z), then + t  (projection.cu:44) */
  for (int r = 0; r < 3; ++r)
    c[r] = fmaf(R[r * 3 + 2], z, fmaf(R[r * 3 + 0], x, R[r * 3 + 1] * y)) + t[r];
}

/* glm::toMat3(glm::normalize(quat(w,x,y,z))) as a row-major matrix (projection.cu:64-65). */
static void quat_rot(const float* q, float* Rq, float* qn) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  float dot = fmaf(w, w, x * x) + fmaf(y, y, z * z);
  float len = sqrtf(dot);
  if (len <= 0.0f) {
    w = 1.0f; x = y = z = 0.0f;
  } else {
    float inv = 1.0f / len;
    w *= inv; x *= inv; y *= inv; z *= inv;
  }
  qn[0] = w; qn[1] = x; qn[2] = y; qn[3] = z;
  /* glm mat3_cast as the reference's build evaluates it (measured against the ref+shim build
   * on a B200): sums of two products fuse the first product, except the (0,0) entry, which
   * adds the two rounded squares */
  float yy = y * y, zz = z * z, wx = w * x, wy = w * y, wz = w * z;
  Rq[0] = fmaf(-2.0f, yy + zz, 1.0f);
  Rq[3] = 2.0f * fmaf(x, y, wz);
  Rq[6] = 2.0f * fmaf(x, z, -wy);
  Rq[1] = 2.0f * fmaf(x, y, -wz);
  Rq[4] = fmaf(-2.0f, fmaf(x, x, zz), 1.0f);
  Rq[7] = 2.0f * fmaf(y, z, wx);
  Rq[2] = 2.0f * fmaf(x, z, wy);
  Rq[5] = 2.0f * fmaf(y, z, -wx);
  Rq[8] = fmaf(-2.0f, fmaf(x, x, yy), 1.0f);
}

/* C = A B (row-major), sum over k in order with the left products fused. */
static void mm(const float* A, const float* B, float* C) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c)
      C[r * 3 + c] = fmaf(A[r * 3 + 2], B[2 * 3 + c], fmaf(A[r * 3 + 0], B[0 * 3 + c], A[r * 3 + 1] * B[1 * 3 + c]));
}
/* C = A B^T */
static void mmt(const float* A, const float* B, float* C) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c)
      C[r * 3 + c] = fmaf(A[r * 3 + 2], B[c * 3 + 2], fmaf(A[r * 3 + 0], B[c * 3 + 0], A[r * 3 + 1] * B[c * 3 + 1]));
}

void oracle_project(int N, const float* mu, const float* q, const float* s, const float* R,
                    const float* t, float fx, float fy, float cx, float cy, float* mean2d,
                    float* cov2d, float* depths) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    float pc[3];
    proj_camera(R, t, mu[3 * i], mu[3 * i + 1], mu[3 * i + 2], pc);
    mean2d[2 * i] = mean2d[2 * i + 1] = 0.0f;
    cov2d[3 * i] = cov2d[3 * i + 1] = cov2d[3 * i + 2] = 0.0f;
    depths[i] = 0.0f;
    if (pc[2] <= 0.2f) continue; /* projection.cu:47 */
    depths[i] = pc[2];
    mean2d[2 * i] = (fx * pc[0]) / pc[2] + cx;
    mean2d[2 * i + 1] = (fy * pc[1]) / pc[2] + cy;
    float Rq[9], qn[4];
    quat_rot(q + 4 * i, Rq, qn);
    float sv[3] = {expf(s[3 * i]), expf(s[3 * i + 1]), expf(s[3 * i + 2])};
    float M[9], Sw[9], T[9], Sc[9];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) M[r * 3 + c] = Rq[r * 3 + c] * sv[c];
    mmt(M, M, Sw);
    mm(R, Sw, T);
    mmt(T, R, Sc);
    float z = pc[2], z2 = z * z;
    float J00 = fx / z, J02 = -(fx * pc[0]) / z2, J11 = fy / z, J12 = -(fy * pc[1]) / z2;
    /* projection.cu:91-98 with Sigma_cam[c][r] = Sc[r*3+c] */
    float a = fmaf(J00, fmaf(J00, Sc[0], J02 * Sc[2]), J02 * fmaf(J00, Sc[6], J02 * Sc[8]));
    float b = fmaf(J00, fmaf(J11, Sc[3], J12 * Sc[6]), J02 * fmaf(J11, Sc[5], J12 * Sc[8]));
    float c = fmaf(J11, fmaf(J11, Sc[4], J12 * Sc[7]), J12 * fmaf(J11, Sc[5], J12 * Sc[8]));
    cov2d[3 * i] = a + 0.3f;
    cov2d[3 * i + 1] = b;
    cov2d[3 * i + 2] = c + 0.3f;
  }
}

/* ---------------------------------------------------------------------------------------
 * SH forward: csrc/forward/SH.cu:31-91.
 * ------------------------------------------------------------------------------------- */
static const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
static const float C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                            -1.0925484305920792f, 0.5462742152960396f};
static const float C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                            0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                            -0.5900435899266435f};

static void sh_basis15(float x, float y, float z, float* Y) {
  float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  Y[0] = -C1 * y;
  Y[1] = C1 * z;
  Y[2] = -C1 * x;
  Y[3] = C2[0] * xy;
  Y[4] = C2[1] * yz;
  Y[5] = C2[2] * fmaf(-y, y, fmaf(2.0f, zz, -xx));
  Y[6] = C2[3] * xz;
  Y[7] = C2[4] * fmaf(x, x, -yy);
  Y[8] = (C3[0] * y) * fmaf(3.0f, xx, -yy);
  Y[9] = (C3[1] * xy) * z;
  Y[10] = (C3[2] * y) * fmaf(-y, y, fmaf(4.0f, zz, -xx));
  Y[11] = (C3[3] * z) * fmaf(-3.0f, yy, fmaf(2.0f, zz, -(3.0f * xx)));
  Y[12] = (C3[4] * x) * fmaf(-y, y, fmaf(4.0f, zz, -xx));
  Y[13] = (C3[5] * z) * fmaf(x, x, -yy);
  Y[14] = (C3[6] * x) * fmaf(x, x, -(3.0f * yy));
}

void oracle_sh(int N, const float* cam, const float* mu, const float* A, const float* kj,
               float* colors) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    float vx = mu[3 * i] - cam[0], vy = mu[3 * i + 1] - cam[1], vz = mu[3 * i + 2] - cam[2];
    float inv = 1.0f / sqrtf(fmaf(vz, vz, fmaf(vx, vx, vy * vy)));
    float Y[15];
    sh_basis15(vx * inv, vy * inv, vz * inv, Y);
    const float* k = kj + 45 * (size_t)i;
    for (int ch = 0; ch < 3; ++ch) {
      float v = fmaf(C0, A[3 * i + ch], 0.5f);
      for (int j = 0; j < 15; ++j) v = fmaf(Y[j], k[3 * j + ch], v);
      colors[3 * i + ch] = fminf(fmaxf(v, 0.0f), 1.0f);
    }
  }
}

/* ---------------------------------------------------------------------------------------
 * Binning: csrc/forward/rasterize.cu:19-59 (count), 79-135 (keys), 146-165 (ranges), and a
 * stable ascending sort of the 64-bit keys (rasterize.cu:416-435).
 * ------------------------------------------------------------------------------------- */
static int tile_rect(float mx, float my, float a, float b, float c, int W, int H, int* r) {
  float det = fmaf(a, c, -(b * b));
  if (det <= 0.0f) return 0;
  float mid = 0.5f * (a + c);
  float lambda = mid + sqrtf(fmaxf(0.1f, fmaf(mid, mid, -det)));
  float radius = ceilf(3.0f * sqrtf(lambda));
  int min_x = (int)floorf(mx - radius); if (min_x < 0) min_x = 0;
  int max_x = (int)ceilf(mx + radius);  if (max_x > W) max_x = W;
  int min_y = (int)floorf(my - radius); if (min_y < 0) min_y = 0;
  int max_y = (int)ceilf(my + radius);  if (max_y > H) max_y = H;
  int tx = (W + 15) / 16, ty = (H + 15) / 16;
  int x0 = min_x / 16, x1 = (max_x + 15) / 16, y0 = min_y / 16, y1 = (max_y + 15) / 16;
#define CL(v, hi) ((v) < 0 ? 0 : ((v) > (hi) ? (hi) : (v)))
  r[0] = CL(x0, tx); r[1] = CL(x1, tx); r[2] = CL(y0, ty); r[3] = CL(y1, ty);
#undef CL
  int w = r[1] - r[0], h = r[3] - r[2];
  return (w > 0 ? w : 0) * (h > 0 ? h : 0);
}

/* Per-Gaussian tile counts; returns M. `counts` may be NULL. */
long long oracle_count(int N, int H, int W, const float* mean2d, const float* cov2d,
                       int* counts) {
  long long M = 0;
#pragma omp parallel for reduction(+ : M) schedule(static)
  for (int i = 0; i < N; ++i) {
    int r[4];
    int cnt = tile_rect(mean2d[2 * i], mean2d[2 * i + 1], cov2d[3 * i], cov2d[3 * i + 1],
                        cov2d[3 * i + 2], W, H, r);
    if (counts) counts[i] = cnt;
    M += cnt;
  }
  return M;
}

/* Stable LSD radix sort of (key, id) by 64-bit key, 16-bit digits. */
static void radix_sort64(uint64_t* keys, int* ids, long long M) {
  if (M <= 1) return;
  uint64_t* k2 = (uint64_t*)malloc((size_t)M * sizeof(uint64_t));
  int* i2 = (int*)malloc((size_t)M * sizeof(int));
  long long* cnt = (long long*)malloc(65536 * sizeof(long long));
  for (int pass = 0; pass < 4; ++pass) {
    int shift = 16 * pass;
    memset(cnt, 0, 65536 * sizeof(long long));
    for (long long j = 0; j < M; ++j) cnt[(keys[j] >> shift) & 0xffff]++;
    long long run = 0;
    for (int d = 0; d < 65536; ++d) { long long c = cnt[d]; cnt[d] = run; run += c; }
    for (long long j = 0; j < M; ++j) {
      long long pos = cnt[(keys[j] >> shift) & 0xffff]++;
      k2[pos] = keys[j];
      i2[pos] = ids[j];
    }
    memcpy(keys, k2, (size_t)M * sizeof(uint64_t));
    memcpy(ids, i2, (size_t)M * sizeof(int));
  }
  free(k2); free(i2); free(cnt);
}

/* Keys, ids and ranges. keys/ids hold M entries (from oracle_count); ranges T*2. */
void oracle_bin(int N, int H, int W, const float* mean2d, const float* cov2d,
                const float* depths, long long M, uint64_t* keys, int* ids, int* ranges) {
  int tx = (W + 15) / 16, ty = (H + 15) / 16;
  long long T = (long long)tx * ty;
  int* counts = (int*)malloc((size_t)(N > 0 ? N : 1) * sizeof(int));
  long long* offs = (long long*)malloc((size_t)(N > 0 ? N : 1) * sizeof(long long));
  oracle_count(N, H, W, mean2d, cov2d, counts);
  long long run = 0;
  for (int i = 0; i < N; ++i) { offs[i] = run; run += counts[i]; }
#pragma omp parallel for schedule(dynamic, 1024)
  for (int i = 0; i < N; ++i) {
    if (!counts[i]) continue;
    int r[4];
    tile_rect(mean2d[2 * i], mean2d[2 * i + 1], cov2d[3 * i], cov2d[3 * i + 1], cov2d[3 * i + 2],
              W, H, r);
    uint32_t dbits;
    memcpy(&dbits, depths + i, 4);
    long long slot = offs[i];
    for (int y = r[2]; y < r[3]; ++y)
      for (int x = r[0]; x < r[1]; ++x) {
        keys[slot] = ((uint64_t)(uint32_t)(y * tx + x) << 32) | (uint64_t)dbits;
        ids[slot] = i;
        ++slot;
      }
  }
  (void)M;
  radix_sort64(keys, ids, run);
  memset(ranges, 0, (size_t)T * 2 * sizeof(int));
  for (long long j = 0; j < run; ++j) {
    uint32_t cur = (uint32_t)(keys[j] >> 32);
    if (j == 0) ranges[2 * cur] = 0;
    else {
      uint32_t prev = (uint32_t)(keys[j - 1] >> 32);
      if (cur != prev) { ranges[2 * prev + 1] = (int)j; ranges[2 * cur] = (int)j; }
    }
    if (j == run - 1) ranges[2 * cur + 1] = (int)run;
  }
  free(counts); free(offs);
}

/* ---------------------------------------------------------------------------------------
 * Blend forward: csrc/forward/rasterize.cu:188-280.
 * ------------------------------------------------------------------------------------- */
static void conic_of(float a, float b, float c, float* v) {
  float det = fmaf(a, c, -(b * b));
  float inv = det > 0.0f ? 1.0f / det : 0.0f;
  v[0] = c * inv; v[1] = -b * inv; v[2] = a * inv;
}

static float power_of(const float* v, float dx, float dy, float* mag) {
  /* -0.5 * (v0 dx dx + 2 v1 dx dy + v2 dy dy)  (rasterize.cu:249-251) */
  float t2 = ((2.0f * v[1]) * dx) * dy;
  float s1 = fmaf(v[0] * dx, dx, t2);
  float s = fmaf(v[2] * dy, dy, s1);
  if (mag) *mag = fabsf(v[0] * dx * dx) + fabsf(t2) + fabsf(v[2] * dy * dy);
  return -0.5f * s;
}

#define AMB_REL_ALPHA 4e-6f
#define AMB_REL_T 1e-4f

void oracle_blend(int N, int H, int W, const int* ranges, const int* ids, const float* mean2d,
                  const float* cov2d, const float* colors, const float* alpha, float* img,
                  float* final_T, int* n_contrib, unsigned char* ambiguous) {
  int tx = (W + 15) / 16, ty = (H + 15) / 16;
  (void)N;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < tx * ty; ++tile) {
    int x0 = (tile % tx) * 16, y0 = (tile / tx) * 16;
    int start = ranges[2 * tile], end = ranges[2 * tile + 1];
    for (int py = y0; py < y0 + 16 && py < H; ++py)
      for (int px = x0; px < x0 + 16 && px < W; ++px) {
        float T = 1.0f, C[3] = {0.0f, 0.0f, 0.0f};
        int contributor = 0, last = 0;
        unsigned char amb = 0;
        for (int j = start; j < end; ++j) {
          ++contributor;
          int g = ids[j];
          float v[3], mag;
          conic_of(cov2d[3 * g], cov2d[3 * g + 1], cov2d[3 * g + 2], v);
          float dx = (float)px - mean2d[2 * g], dy = (float)py - mean2d[2 * g + 1];
          float power = power_of(v, dx, dy, &mag);
          if (fabsf(2.0f * power) <= 1e-6f * mag && mag > 0.0f) amb = 1;
          if (power > 0.0f) continue;
          float a = fminf(0.99f, alpha[g] * expf(power));
          if (fabsf(a * 255.0f - 1.0f) <= AMB_REL_ALPHA) amb = 1;
          if (a < (1.0f / 255.0f)) continue;
          float wgt = a * T;
          for (int ch = 0; ch < 3; ++ch) C[ch] = fmaf(colors[3 * g + ch], wgt, C[ch]);
          T = T * (1.0f - a);
          last = contributor;
          if (fabsf(T - 1e-4f) <= AMB_REL_T * 1e-4f) amb = 1;
          if (T < 1e-4f) break;
        }
        int pix = py * W + px;
        img[3 * pix] = C[0]; img[3 * pix + 1] = C[1]; img[3 * pix + 2] = C[2];
        final_T[pix] = T;
        n_contrib[pix] = last;
        if (ambiguous) ambiguous[pix] = amb;
      }
  }
}

/* ---------------------------------------------------------------------------------------
 * Blend backward: csrc/backward/rasterize_backward.cu:60-235. Per-tile slot sums and the
 * global sums are accumulated in double; `amb_g` (optional, N bytes) flags Gaussians that
 * received a contribution whose opacity or clamp decision was within a few ulp.
 * ------------------------------------------------------------------------------------- */
void oracle_blend_backward(int N, int H, int W, const float* grad_img, const float* mean2d,
                           const float* cov2d, const float* colors, const float* alpha,
                           const int* ids, const int* ranges, const float* final_T,
                           const int* n_contrib, float* g_mean2d, float* g_cov2d,
                           float* g_colors, float* g_alpha, unsigned char* amb_g) {
  int tx = (W + 15) / 16, ty = (H + 15) / 16;
  double* acc = (double*)calloc((size_t)(N > 0 ? N : 1) * 9, sizeof(double));
  if (amb_g) memset(amb_g, 0, (size_t)N);
#pragma omp parallel
  {
    double* slot = NULL;
    int slot_cap = 0;
    double* mine = (double*)calloc((size_t)(N > 0 ? N : 1) * 9, sizeof(double));
#pragma omp for schedule(dynamic, 1)
    for (int tile = 0; tile < tx * ty; ++tile) {
      int x0 = (tile % tx) * 16, y0 = (tile / tx) * 16;
      int start = ranges[2 * tile], end = ranges[2 * tile + 1], K = end - start;
      if (K <= 0) continue;
      if (K > slot_cap) { free(slot); slot_cap = K; slot = (double*)malloc((size_t)K * 9 * sizeof(double)); }
      memset(slot, 0, (size_t)K * 9 * sizeof(double));
      for (int py = y0; py < y0 + 16 && py < H; ++py)
        for (int px = x0; px < x0 + 16 && px < W; ++px) {
          int pix = py * W + px;
          float g[3] = {grad_img[3 * pix], grad_img[3 * pix + 1], grad_img[3 * pix + 2]};
          float T = final_T[pix];
          int last = n_contrib[pix];
          if (last > K) last = K;
          float acc_c[3] = {0.0f, 0.0f, 0.0f};
          for (int k = last - 1; k >= 0; --k) {
            int gid = ids[start + k];
            if (gid < 0 || gid >= N) continue;
            float v[3];
            conic_of(cov2d[3 * gid], cov2d[3 * gid + 1], cov2d[3 * gid + 2], v);
            float dx = (float)px - mean2d[2 * gid], dy = (float)py - mean2d[2 * gid + 1];
            float power = power_of(v, dx, dy, NULL);
            if (power > 0.0f) continue;
            float G = expf(power);
            float araw = alpha[gid] * G;
            float a = fminf(0.99f, araw);
            if (a < (1.0f / 255.0f)) continue;
            if (amb_g && (fabsf(a * 255.0f - 1.0f) <= AMB_REL_ALPHA ||
                          fabsf(araw / 0.99f - 1.0f) <= AMB_REL_ALPHA))
              amb_g[gid] = 1;
            float om = 1.0f - a;
            float Tb = T / fmaxf(om, 1e-4f);
            const float* c = colors + 3 * gid;
            double* sl = slot + (size_t)k * 9;
            for (int ch = 0; ch < 3; ++ch) sl[5 + ch] += (double)(a * Tb * g[ch]);
            float dLda = ((c[0] - acc_c[0]) * g[0] + (c[1] - acc_c[1]) * g[1] +
                          (c[2] - acc_c[2]) * g[2]) * Tb;
            float dLdp = 0.0f;
            if (araw < 0.99f) {
              sl[8] += (double)(G * dLda);
              dLdp = a * dLda;
            }
            sl[0] += (double)(dLdp * (v[0] * dx + v[1] * dy));
            sl[1] += (double)(dLdp * (v[1] * dx + v[2] * dy));
            sl[2] += (double)(-0.5f * dLdp * dx * dx);
            sl[3] += (double)(-dLdp * dx * dy);
            sl[4] += (double)(-0.5f * dLdp * dy * dy);
            for (int ch = 0; ch < 3; ++ch) acc_c[ch] = a * c[ch] + om * acc_c[ch];
            T = Tb;
          }
        }
      for (int k = 0; k < K; ++k) {
        int gid = ids[start + k];
        if (gid < 0 || gid >= N) continue;
        double* sl = slot + (size_t)k * 9;
        double* o = mine + (size_t)gid * 9;
        float v[3];
        conic_of(cov2d[3 * gid], cov2d[3 * gid + 1], cov2d[3 * gid + 2], v);
        double vx = v[0], vy = v[1], vz = v[2], gx = sl[2], gy = 0.5 * sl[3], gz = sl[4];
        o[0] += sl[0];
        o[1] += sl[1];
        o[2] += -(vx * vx * gx + 2.0 * vx * vy * gy + vy * vy * gz);
        o[3] += -2.0 * (vx * vy * gx + (vx * vz + vy * vy) * gy + vy * vz * gz);
        o[4] += -(vy * vy * gx + 2.0 * vy * vz * gy + vz * vz * gz);
        o[5] += sl[5]; o[6] += sl[6]; o[7] += sl[7]; o[8] += sl[8];
      }
    }
#pragma omp critical
    for (size_t j = 0; j < (size_t)N * 9; ++j) acc[j] += mine[j];
    free(mine);
    free(slot);
  }
  for (int i = 0; i < N; ++i) {
    const double* o = acc + (size_t)i * 9;
    g_mean2d[2 * i] = (float)o[0]; g_mean2d[2 * i + 1] = (float)o[1];
    g_cov2d[3 * i] = (float)o[2]; g_cov2d[3 * i + 1] = (float)o[3]; g_cov2d[3 * i + 2] = (float)o[4];
    g_colors[3 * i] = (float)o[5]; g_colors[3 * i + 1] = (float)o[6]; g_colors[3 * i + 2] = (float)o[7];
    g_alpha[i] = (float)o[8];
  }
  free(acc);
}

/* ---------------------------------------------------------------------------------------
 * SH backward: csrc/backward/delight_backward.cu:121-173.
 * ------------------------------------------------------------------------------------- */
static void sh_dY_ddir(float x, float y, float z, const float* dY, float* g) {
  float xx = x * x, yy = y * y, zz = z * z;
  g[0] = g[1] = g[2] = 0.0f;
  g[1] += dY[0] * (-C1);
  g[2] += dY[1] * C1;
  g[0] += dY[2] * (-C1);
  g[0] += dY[3] * (C2[0] * y);          g[1] += dY[3] * (C2[0] * x);
  g[1] += dY[4] * (C2[1] * z);          g[2] += dY[4] * (C2[1] * y);
  g[0] += dY[5] * (-2.0f * C2[2] * x);  g[1] += dY[5] * (-2.0f * C2[2] * y);
  g[2] += dY[5] * (4.0f * C2[2] * z);
  g[0] += dY[6] * (C2[3] * z);          g[2] += dY[6] * (C2[3] * x);
  g[0] += dY[7] * (2.0f * C2[4] * x);   g[1] += dY[7] * (-2.0f * C2[4] * y);
  g[0] += dY[8] * (C3[0] * y * 6.0f * x);
  g[1] += dY[8] * (C3[0] * (3.0f * xx - 3.0f * yy));
  g[0] += dY[9] * (C3[1] * y * z); g[1] += dY[9] * (C3[1] * x * z); g[2] += dY[9] * (C3[1] * x * y);
  g[0] += dY[10] * (C3[2] * y * (-2.0f * x));
  g[1] += dY[10] * (C3[2] * (4.0f * zz - xx - 3.0f * yy));
  g[2] += dY[10] * (C3[2] * y * 8.0f * z);
  g[0] += dY[11] * (C3[3] * z * (-6.0f * x));
  g[1] += dY[11] * (C3[3] * z * (-6.0f * y));
  g[2] += dY[11] * (C3[3] * (6.0f * zz - 3.0f * xx - 3.0f * yy));
  g[0] += dY[12] * (C3[4] * (4.0f * zz - 3.0f * xx - yy));
  g[1] += dY[12] * (C3[4] * x * (-2.0f * y));
  g[2] += dY[12] * (C3[4] * x * 8.0f * z);
  g[0] += dY[13] * (C3[5] * z * 2.0f * x);
  g[1] += dY[13] * (C3[5] * z * (-2.0f * y));
  g[2] += dY[13] * (C3[5] * (xx - yy));
  g[0] += dY[14] * (C3[6] * (3.0f * xx - 3.0f * yy));
  g[1] += dY[14] * (C3[6] * x * (-6.0f * y));
}

void oracle_sh_backward(int N, const float* gcol, const float* mu, const float* A,
                        const float* kj, const float* cam, float* gA, float* gkj, float* gmu) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    float vx = mu[3 * i] - cam[0], vy = mu[3 * i + 1] - cam[1], vz = mu[3 * i + 2] - cam[2];
    float inv = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz + 1e-8f);
    float d[3] = {vx * inv, vy * inv, vz * inv};
    float Y[15];
    sh_basis15(d[0], d[1], d[2], Y);
    const float* k = kj + 45 * (size_t)i;
    float g[3];
    for (int ch = 0; ch < 3; ++ch) {
      float v = fmaf(C0, A[3 * i + ch], 0.5f);
      for (int j = 0; j < 15; ++j) v = fmaf(Y[j], k[3 * j + ch], v);
      g[ch] = (v < 0.0f || v > 1.0f) ? 0.0f : gcol[3 * i + ch];
      gA[3 * i + ch] = g[ch] * C0;
    }
    float dY[15];
    for (int j = 0; j < 15; ++j) {
      for (int ch = 0; ch < 3; ++ch) gkj[45 * (size_t)i + 3 * j + ch] = g[ch] * Y[j];
      dY[j] = g[0] * k[3 * j] + g[1] * k[3 * j + 1] + g[2] * k[3 * j + 2];
    }
    float gd[3];
    sh_dY_ddir(d[0], d[1], d[2], dY, gd);
    float dd = d[0] * gd[0] + d[1] * gd[1] + d[2] * gd[2];
    for (int c = 0; c < 3; ++c) gmu[3 * i + c] = inv * (gd[c] - d[c] * dd);
  }
}

/* ---------------------------------------------------------------------------------------
 * Projection backward: csrc/backward/projection_backward.cu:33-138, with the quaternion
 * gradient taken as the derivative of quat_rot (the reading of the reference's
 * dL_dRt-indexed formula under which its own gradcheck,
 * tests/test_cuda_backward.py:53-113, holds).
 * ------------------------------------------------------------------------------------- */
void oracle_project_backward(int N, const float* gm, const float* gc, const float* mu,
                             const float* q, const float* s, const float* R, const float* t,
                             float fx, float fy, float cx, float cy, float* gmu, float* gq,
                             float* gs) {
  (void)cx; (void)cy;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    float pc[3];
    proj_camera(R, t, mu[3 * i], mu[3 * i + 1], mu[3 * i + 2], pc);
    for (int c = 0; c < 3; ++c) { gmu[3 * i + c] = 0.0f; gs[3 * i + c] = 0.0f; }
    for (int c = 0; c < 4; ++c) gq[4 * i + c] = 0.0f;
    if (pc[2] <= 0.2f) continue;
    float z = pc[2], z2 = z * z, z3 = z2 * z;
    float dmc[3] = {(fx / z) * gm[2 * i], (fy / z) * gm[2 * i + 1],
                    (-fx * pc[0] / z2) * gm[2 * i] + (-fy * pc[1] / z2) * gm[2 * i + 1]};
    float G00 = gc[3 * i], G01 = 0.5f * gc[3 * i + 1], G11 = gc[3 * i + 2];
    float J[6] = {fx / z, 0.0f, -(fx * pc[0]) / z2, 0.0f, fy / z, -(fy * pc[1]) / z2};
    float Rq[9], qn[4];
    quat_rot(q + 4 * i, Rq, qn);
    float sv[3] = {expf(s[3 * i]), expf(s[3 * i + 1]), expf(s[3 * i + 2])};
    float M[9], Sw[9], T[9], Sc[9];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) M[r * 3 + c] = Rq[r * 3 + c] * sv[c];
    mmt(M, M, Sw); mm(R, Sw, T); mmt(T, R, Sc);
    float G[4] = {G00, G01, G01, G11};
    float GJ[6];
    for (int r = 0; r < 2; ++r)
      for (int c = 0; c < 3; ++c) GJ[r * 3 + c] = G[r * 2] * J[c] + G[r * 2 + 1] * J[3 + c];
    float dSc[9];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) dSc[r * 3 + c] = J[r] * GJ[c] + J[3 + r] * GJ[3 + c];
    float U[9], dSw[9], dM[9];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c)
        U[r * 3 + c] = R[r] * dSc[c] + R[3 + r] * dSc[3 + c] + R[6 + r] * dSc[6 + c];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c)
        dSw[r * 3 + c] = U[r * 3] * R[c] + U[r * 3 + 1] * R[3 + c] + U[r * 3 + 2] * R[6 + c];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c)
        dM[r * 3 + c] = 2.0f * (dSw[r * 3] * M[c] + dSw[r * 3 + 1] * M[3 + c] + dSw[r * 3 + 2] * M[6 + c]);
    for (int c = 0; c < 3; ++c)
      gs[3 * i + c] = (Rq[c] * dM[c] + Rq[3 + c] * dM[3 + c] + Rq[6 + c] * dM[6 + c]) * sv[c];
    float D[9];
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) D[r * 3 + c] = dM[r * 3 + c] * sv[c];
    float dJ[6];
    for (int r = 0; r < 2; ++r)
      for (int c = 0; c < 3; ++c)
        dJ[r * 3 + c] = 2.0f * (GJ[r * 3] * Sc[c] + GJ[r * 3 + 1] * Sc[3 + c] + GJ[r * 3 + 2] * Sc[6 + c]);
    dmc[0] += dJ[2] * (-fx / z2);
    dmc[1] += dJ[5] * (-fy / z2);
    dmc[2] += dJ[0] * (-fx / z2) + dJ[4] * (-fy / z2) + dJ[2] * (2.0f * fx * pc[0] / z3) +
              dJ[5] * (2.0f * fy * pc[1] / z3);
    for (int c = 0; c < 3; ++c) gmu[3 * i + c] = R[c] * dmc[0] + R[3 + c] * dmc[1] + R[6 + c] * dmc[2];
    float w = qn[0], x = qn[1], y = qn[2], zq = qn[3];
    float dq[4];
    dq[0] = 2.0f * (zq * (D[3] - D[1]) + y * (D[2] - D[6]) + x * (D[7] - D[5]));
    dq[1] = 2.0f * (y * (D[1] + D[3]) + zq * (D[2] + D[6]) + w * (D[7] - D[5])) - 4.0f * x * (D[4] + D[8]);
    dq[2] = 2.0f * (x * (D[1] + D[3]) + w * (D[2] - D[6]) + zq * (D[5] + D[7])) - 4.0f * y * (D[0] + D[8]);
    dq[3] = 2.0f * (w * (D[3] - D[1]) + x * (D[2] + D[6]) + y * (D[5] + D[7])) - 4.0f * zq * (D[0] + D[4]);
    const float* qr = q + 4 * i;
    float inv_norm = 1.0f / sqrtf(qr[0] * qr[0] + qr[1] * qr[1] + qr[2] * qr[2] + qr[3] * qr[3] + 1e-8f);
    float qd = w * dq[0] + x * dq[1] + y * dq[2] + zq * dq[3];
    for (int c = 0; c < 4; ++c) gq[4 * i + c] = inv_norm * (dq[c] - qn[c] * qd);
  }
}
