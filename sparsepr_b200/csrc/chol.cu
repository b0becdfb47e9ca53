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

}  // namespace spr

using namespace spr;

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
