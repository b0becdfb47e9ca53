// Batched Cholesky solve of small symmetric positive definite systems
// A X = B (A: m x m, m <= 128; B: m x nrhs), one CTA per system, fp32.
// Used for the dual ridge solve of the probe repair fit, (Xw Xw^T + l I) D = Yw.
// A matrix that is not positive definite yields non-finite X, which the
// caller's per-head recovery replaces (no device assert).
#include "common.cuh"

namespace spr {

constexpr int kCholMax = 128;
constexpr int kCholLd = kCholMax + 1;

// In-place Cholesky of the m x m matrix in shared memory (row stride ld; the
// lower triangle becomes L), right-looking: per column j the pivot s = a_jj,
// then the trailing lower triangle a_ik -= a_ij a_kj / s (k in (j, i]) in
// parallel, and column j is divided by sqrt(s) one step later (the next
// update no longer reads it): two barriers per column.  A pivot that is not
// positive and finite makes the result false; with nan_on_fail the pivot
// stays sqrt(s) (NaN for s < 0, which then propagates into a solve),
// otherwise it becomes 1.  Block-wide: every thread of the CTA calls it.
__device__ bool chol_factor_smem(float* L, int m, int ld, bool nan_on_fail = false) {
  __shared__ int s_bad;
  __shared__ float s_inv_piv;
  if (threadIdx.x == 0) s_bad = 0;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5, ny = blockDim.x >> 5;
  for (int j = 0; j < m; ++j) {
    if (threadIdx.x == 0) {
      float s = L[j * ld + j];
      if (!(s > 0.f) || !isfinite(s)) {
        s_bad = 1;
        if (!nan_on_fail) s = 1.f;
      }
      L[j * ld + j] = sqrtf(s);
      s_inv_piv = 1.f / s;
    }
    __syncthreads();
    const float inv_s = s_inv_piv;
    // Trailing update (rows i > j, columns j < k <= i) with the unscaled column j.
    for (int i = j + 1 + ty; i < m; i += ny) {
      const float lij = L[i * ld + j] * inv_s;
      for (int k = j + 1 + tx; k <= i; k += 32) L[i * ld + k] = fmaf(-lij, L[k * ld + j], L[i * ld + k]);
    }
    if (j > 0) {  // scale the previous column, which this update did not read
      const float pd = L[(j - 1) * ld + (j - 1)];
      for (int i = j + threadIdx.x; i < m; i += blockDim.x) L[i * ld + (j - 1)] /= pd;
    }
    __syncthreads();
  }
  const bool ok = s_bad == 0;
  __syncthreads();
  return ok;
}

// A X = B per system: L in shared memory, then forward and back substitution
// with the right-hand sides staged in shared memory (one column per thread,
// in blocks of blockDim.x columns).
__global__ void __launch_bounds__(256)
chol_solve_kernel(const float* __restrict__ a, const float* __restrict__ rhs, int m, int nrhs,
                  float* __restrict__ x) {
  extern __shared__ float sh_l[];  // [m][kCholLd] L, then [m][blockDim.x] right-hand sides
  const int nt = blockDim.x;
  float* XS = sh_l + m * kCholLd;
  const int64_t b = blockIdx.x;
  const float* A = a + b * (int64_t)m * m;
  for (int idx = threadIdx.x; idx < m * m; idx += nt) {
    const int i = idx / m, j = idx % m;
    sh_l[i * kCholLd + j] = A[idx];
  }
  __syncthreads();
  chol_factor_smem(sh_l, m, kCholLd, /*nan_on_fail=*/true);
  for (int c0 = 0; c0 < nrhs; c0 += nt) {
    const int nc = min(nt, nrhs - c0);
    const float* B = rhs + b * (int64_t)m * nrhs + c0;
    float* X = x + b * (int64_t)m * nrhs + c0;
    for (int idx = threadIdx.x; idx < m * nc; idx += nt) {
      const int i = idx / nc, c = idx % nc;
      XS[i * nt + c] = B[(int64_t)i * nrhs + c];
    }
    __syncthreads();
    const int col = threadIdx.x;
    if (col < nc) {
      // Rows in blocks of 8: the earlier rows' contributions first (eight
      // independent accumulators per loaded value), then the 8 x 8 triangle.
      constexpr int RB = 8;
      for (int i0 = 0; i0 < m; i0 += RB) {  // L y = b
        const int nb = min(RB, m - i0);
        float acc[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) acc[r] = r < nb ? XS[(i0 + r) * nt + col] : 0.f;
        for (int kk = 0; kk < i0; ++kk) {
          const float xk = XS[kk * nt + col];
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < nb) acc[r] = fmaf(-sh_l[(i0 + r) * kCholLd + kk], xk, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (r < nb) {
#pragma unroll
            for (int q = 0; q < r; ++q) acc[r] = fmaf(-sh_l[(i0 + r) * kCholLd + i0 + q], acc[q], acc[r]);
            acc[r] /= sh_l[(i0 + r) * kCholLd + i0 + r];
            XS[(i0 + r) * nt + col] = acc[r];
          }
        }
      }
      for (int i1 = m; i1 > 0; i1 -= RB) {  // L^T x = y
        const int i0 = max(0, i1 - RB), nb = i1 - i0;
        float acc[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) acc[r] = r < nb ? XS[(i0 + r) * nt + col] : 0.f;
        for (int kk = i1; kk < m; ++kk) {
          const float xk = XS[kk * nt + col];
#pragma unroll
          for (int r = 0; r < RB; ++r)
            if (r < nb) acc[r] = fmaf(-sh_l[kk * kCholLd + i0 + r], xk, acc[r]);
        }
#pragma unroll
        for (int r = RB - 1; r >= 0; --r) {
          if (r < nb) {
#pragma unroll
            for (int q = r + 1; q < RB; ++q)
              if (q < nb) acc[r] = fmaf(-sh_l[(i0 + q) * kCholLd + i0 + r], acc[q], acc[r]);
            acc[r] /= sh_l[(i0 + r) * kCholLd + i0 + r];
            XS[(i0 + r) * nt + col] = acc[r];
          }
        }
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < m * nc; idx += nt) {
      const int i = idx / nc, c = idx % nc;
      X[(int64_t)i * nrhs + c] = XS[i * nt + c];
    }
    __syncthreads();
  }
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
  const int smem = (m * kCholLd + m * 256) * (int)sizeof(float);
  const cudaError_t e = cudaFuncSetAttribute(chol_solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (kCholMax * kCholLd + kCholMax * 256) * 4);
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "chol_solve: shared-memory opt-in: %s", cudaGetErrorString(e));
  chol_solve_kernel<<<(unsigned)batch, 256, smem, (cudaStream_t)stream>>>(a, b, m, nrhs, x);
  return check_launch("chol_solve");
}
