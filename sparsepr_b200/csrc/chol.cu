// Batched Cholesky solve of small symmetric positive definite systems
// A X = B (A: m x m, m <= 128; B: m x nrhs), one CTA per system, fp32.
// Used for the dual ridge solve of the probe repair fit, (Xw Xw^T + l I) D = Yw.
// A matrix that is not positive definite yields non-finite X, which the
// caller's per-head recovery replaces (no device assert).
#include "common.cuh"

namespace spr {

constexpr int kCholMax = 128;
constexpr int kCholLd = kCholMax + 1;

__global__ void __launch_bounds__(256)
chol_solve_kernel(const float* __restrict__ a, const float* __restrict__ rhs, int m, int nrhs,
                  float* __restrict__ x) {
  extern __shared__ float sh_l[];  // [m][kCholLd], lower triangle = L
  const int64_t b = blockIdx.x;
  const float* A = a + b * (int64_t)m * m;
  for (int idx = threadIdx.x; idx < m * m; idx += blockDim.x) {
    const int i = idx / m, j = idx % m;
    sh_l[i * kCholLd + j] = A[idx];
  }
  __syncthreads();
  // Cholesky-Banachiewicz, one column per step: L[j][j], then L[i][j] for i > j in parallel.
  for (int j = 0; j < m; ++j) {
    if (threadIdx.x == 0) {
      float s = sh_l[j * kCholLd + j];
      for (int kk = 0; kk < j; ++kk) s -= sh_l[j * kCholLd + kk] * sh_l[j * kCholLd + kk];
      sh_l[j * kCholLd + j] = sqrtf(s);  // NaN when A is not positive definite
    }
    __syncthreads();
    const float djj = sh_l[j * kCholLd + j];
    for (int i = j + 1 + threadIdx.x; i < m; i += blockDim.x) {
      float s = sh_l[i * kCholLd + j];
      for (int kk = 0; kk < j; ++kk) s -= sh_l[i * kCholLd + kk] * sh_l[j * kCholLd + kk];
      sh_l[i * kCholLd + j] = s / djj;
    }
    __syncthreads();
  }
  // One right-hand-side column per thread: L y = b, then L^T x = y (in place).
  for (int col = threadIdx.x; col < nrhs; col += blockDim.x) {
    const float* B = rhs + b * (int64_t)m * nrhs + col;
    float* X = x + b * (int64_t)m * nrhs + col;
    for (int i = 0; i < m; ++i) {
      float s = B[(int64_t)i * nrhs];
      for (int kk = 0; kk < i; ++kk) s -= sh_l[i * kCholLd + kk] * X[(int64_t)kk * nrhs];
      X[(int64_t)i * nrhs] = s / sh_l[i * kCholLd + i];
    }
    for (int i = m - 1; i >= 0; --i) {
      float s = X[(int64_t)i * nrhs];
      for (int kk = i + 1; kk < m; ++kk) s -= sh_l[kk * kCholLd + i] * X[(int64_t)kk * nrhs];
      X[(int64_t)i * nrhs] = s / sh_l[i * kCholLd + i];
    }
  }
}

// In-place Cholesky of the m x m matrix in shared memory (row stride ld; the
// lower triangle becomes L).  Returns false (for every thread) when a pivot is
// not positive and finite.  Block-wide: every thread of the CTA calls it.
__device__ bool chol_factor_smem(float* L, int m, int ld) {
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int j = 0; j < m; ++j) {
    if (threadIdx.x == 0) {
      float s = L[j * ld + j];
      for (int kk = 0; kk < j; ++kk) s -= L[j * ld + kk] * L[j * ld + kk];
      if (!(s > 0.f) || !isfinite(s)) {
        s_bad = 1;
        s = 1.f;
      }
      L[j * ld + j] = sqrtf(s);
    }
    __syncthreads();
    const float djj = L[j * ld + j];
    for (int i = j + 1 + threadIdx.x; i < m; i += blockDim.x) {
      float s = L[i * ld + j];
      for (int kk = 0; kk < j; ++kk) s -= L[i * ld + kk] * L[j * ld + kk];
      L[i * ld + j] = s / djj;
    }
    __syncthreads();
  }
  const bool ok = s_bad == 0;
  __syncthreads();
  return ok;
}

// Cholesky-QR of x [n][r] (n, r <= 128): columns normalised to unit length,
// Gram G = X^T X plus mean(diag G) * ridge on the diagonal, G = L L^T, and
// out = X L^{-T} (orthonormal columns up to the ridge).  A Gram matrix that is
// not positive definite gives L = I (out = the normalised X) and failed = 1.
// (operator_kmeans.py:332-364 of the reference.)
__global__ void __launch_bounds__(256)
cholesky_qr_kernel(const float* __restrict__ x, int n, int r, float ridge, float* __restrict__ out,
                   int32_t* __restrict__ failed) {
  extern __shared__ float sh[];
  float* X = sh;                   // [n][kCholLd]
  float* G = sh + n * kCholLd;     // [r][kCholLd]
  const int64_t b = blockIdx.x;
  const float* src = x + b * (int64_t)n * r;
  for (int idx = threadIdx.x; idx < n * r; idx += blockDim.x) X[(idx / r) * kCholLd + idx % r] = src[idx];
  __syncthreads();
  for (int j = threadIdx.x; j < r; j += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s = fmaf(X[i * kCholLd + j], X[i * kCholLd + j], s);
    const float inv = 1.f / fmaxf(sqrtf(s), 1e-12f);
    for (int i = 0; i < n; ++i) X[i * kCholLd + j] *= inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < r * r; idx += blockDim.x) {
    const int a = idx / r, c = idx % r;
    float s = 0.f;
    for (int i = 0; i < n; ++i) s = fmaf(X[i * kCholLd + a], X[i * kCholLd + c], s);
    G[a * kCholLd + c] = s;
  }
  __syncthreads();
  __shared__ float s_jit;
  if (threadIdx.x == 0) {
    float d = 0.f;
    for (int j = 0; j < r; ++j) d += G[j * kCholLd + j];
    s_jit = fmaxf(d / (float)r, 1e-12f) * ridge;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < r; j += blockDim.x) G[j * kCholLd + j] += s_jit;
  __syncthreads();
  const bool ok = chol_factor_smem(G, r, kCholLd);
  if (threadIdx.x == 0) failed[b] = ok ? 0 : 1;
  float* dst = out + b * (int64_t)n * r;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {  // row i: y L^T = x_i by forward substitution
    for (int j = 0; j < r; ++j) {
      float s = X[i * kCholLd + j];
      if (ok) {
        for (int kk = 0; kk < j; ++kk) s -= dst[(int64_t)i * r + kk] * G[j * kCholLd + kk];
        s /= G[j * kCholLd + j];
      }
      dst[(int64_t)i * r + j] = s;
    }
  }
}

// Batched Cholesky with the reference's ridge fallback (operator_kmeans.py:154-218):
// L of A + scale*ridge*I; when that fails, of A + scale*fallback*I; when that
// fails too, L = I and failed = 1.  L is written as a full matrix (zero upper).
__global__ void __launch_bounds__(256)
ridge_cholesky_kernel(const float* __restrict__ a, const float* __restrict__ scale, int m, float ridge,
                      float fallback, float* __restrict__ lout, int32_t* __restrict__ failed) {
  extern __shared__ float sh[];  // [m][kCholLd]
  const int64_t b = blockIdx.x;
  const float* A = a + b * (int64_t)m * m;
  bool ok = false;
  for (int attempt = 0; attempt < 2 && !ok; ++attempt) {
    const float shift = scale[b] * (attempt == 0 ? ridge : fallback);
    for (int idx = threadIdx.x; idx < m * m; idx += blockDim.x) {
      const int i = idx / m, j = idx % m;
      sh[i * kCholLd + j] = A[idx] + (i == j ? shift : 0.f);
    }
    __syncthreads();
    ok = chol_factor_smem(sh, m, kCholLd);
  }
  if (threadIdx.x == 0) failed[b] = ok ? 0 : 1;
  float* L = lout + b * (int64_t)m * m;
  for (int idx = threadIdx.x; idx < m * m; idx += blockDim.x) {
    const int i = idx / m, j = idx % m;
    L[idx] = ok ? (j <= i ? sh[i * kCholLd + j] : 0.f) : (i == j ? 1.f : 0.f);
  }
}

}  // namespace spr

using namespace spr;

extern "C" int spr_cholesky_qr(const float* x, int64_t batch, int n, int r, float relative_ridge, float* out,
                               int32_t* failed, void* stream) {
  if (batch <= 0 || batch > 65535 || n < 1 || n > kCholMax || r < 1 || r > kCholMax)
    return fail(SPR_ERR_SHAPE, "cholesky_qr: need 0 < batch <= 65535, 1 <= n, r <= 128 (n=%d r=%d)", n, r);
  if (!(relative_ridge > 0.f)) return fail(SPR_ERR_ARG, "cholesky_qr: relative_ridge must be positive");
  if (x == out) return fail(SPR_ERR_ARG, "cholesky_qr: out must not alias x");
  const int smem = (n + r) * kCholLd * (int)sizeof(float);
  cudaFuncSetAttribute(cholesky_qr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kCholMax * kCholLd * 4);
  cholesky_qr_kernel<<<(unsigned)batch, 256, smem, (cudaStream_t)stream>>>(x, n, r, relative_ridge, out, failed);
  return check_launch("cholesky_qr");
}

extern "C" int spr_ridge_cholesky(const float* a, const float* scale, int64_t batch, int m, float relative_ridge,
                                  float fallback_ridge, float* l, int32_t* failed, void* stream) {
  if (batch <= 0 || batch > 65535 || m < 1 || m > kCholMax)
    return fail(SPR_ERR_SHAPE, "ridge_cholesky: need 0 < batch <= 65535, 1 <= m <= 128 (m=%d)", m);
  if (!(relative_ridge > 0.f) || !(fallback_ridge > 0.f))
    return fail(SPR_ERR_ARG, "ridge_cholesky: ridge values must be positive");
  const int smem = m * kCholLd * (int)sizeof(float);
  cudaFuncSetAttribute(ridge_cholesky_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kCholMax * kCholLd * 4);
  ridge_cholesky_kernel<<<(unsigned)batch, 256, smem, (cudaStream_t)stream>>>(
      a, scale, m, relative_ridge, fmaxf(fallback_ridge, relative_ridge), l, failed);
  return check_launch("ridge_cholesky");
}

extern "C" int spr_chol_solve(const float* a, const float* b, int64_t batch, int m, int nrhs, float* x,
                              void* stream) {
  if (batch <= 0 || batch > 65535 || m < 1 || m > kCholMax || nrhs < 1)
    return fail(SPR_ERR_SHAPE, "chol_solve: need 0 < batch <= 65535, 1 <= m <= 128, nrhs >= 1 (batch=%lld m=%d nrhs=%d)",
                (long long)batch, m, nrhs);
  if (x == b) return fail(SPR_ERR_ARG, "chol_solve: x must not alias b");
  const int smem = m * kCholLd * (int)sizeof(float);
  cudaFuncSetAttribute(chol_solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kCholMax * kCholLd * 4);
  chol_solve_kernel<<<(unsigned)batch, 256, smem, (cudaStream_t)stream>>>(a, b, m, nrhs, x);
  return check_launch("chol_solve");
}
