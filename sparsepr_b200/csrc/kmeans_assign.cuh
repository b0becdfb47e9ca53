// k-means assignment: per point, argmin over centroids of
// max(|x|^2 + |c|^2 - 2 x.c, 0), ties to the lowest centroid index.
#pragma once
#include "common.cuh"

namespace spr {

inline bool assign_supported_dim(int d) {
  return d == 16 || d == 32 || d == 48 || d == 64 || d == 96 || d == 128;
}

constexpr int kAssignPoints = 128;   // points (threads) per block
constexpr int kAssignTileK = 64;     // centroids per shared-memory tile

// Exact fp32 FFMA assignment.  Each thread keeps its point in registers and
// streams centroid tiles from shared memory (broadcast reads).
template <int D, typename T>
__global__ void __launch_bounds__(kAssignPoints)
assign_simt_kernel(const T* __restrict__ x, int64_t n, int k, const float* __restrict__ centroids,
                   int32_t* __restrict__ labels, const int* __restrict__ done) {
  if (done && *done) return;
  __shared__ __align__(16) float sh_c[kAssignTileK * D];
  __shared__ float sh_csq[kAssignTileK];
  const int64_t b = blockIdx.y;
  const int64_t p = (int64_t)blockIdx.x * kAssignPoints + threadIdx.x;
  const bool valid = p < n;
  float xr[D];
  float xsq = 0.f;
  const T* xp = x + (b * n + (valid ? p : 0)) * D;
#pragma unroll
  for (int e = 0; e < D; ++e) {
    xr[e] = valid ? to_f32(xp[e]) : 0.f;
    xsq = fmaf(xr[e], xr[e], xsq);
  }
  float best = 3.4e38f;
  int best_idx = 0;
  const float* cb = centroids + b * (int64_t)k * D;
  for (int k0 = 0; k0 < k; k0 += kAssignTileK) {
    const int tk = min(kAssignTileK, k - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < tk * D / 4; i += kAssignPoints)
      reinterpret_cast<float4*>(sh_c)[i] = reinterpret_cast<const float4*>(cb + (int64_t)k0 * D)[i];
    __syncthreads();
    if (threadIdx.x < tk) {
      float s = 0.f;
      const float* cc = sh_c + threadIdx.x * D;
      for (int e = 0; e < D; ++e) s = fmaf(cc[e], cc[e], s);
      sh_csq[threadIdx.x] = s;
    }
    __syncthreads();
    for (int j = 0; j < tk; ++j) {
      const float4* c4 = reinterpret_cast<const float4*>(sh_c + j * D);
      float dot0 = 0.f, dot1 = 0.f;
#pragma unroll
      for (int e = 0; e < D / 4; e += 2) {
        const float4 a = c4[e];
        dot0 = fmaf(xr[4 * e + 0], a.x, dot0);
        dot0 = fmaf(xr[4 * e + 1], a.y, dot0);
        dot0 = fmaf(xr[4 * e + 2], a.z, dot0);
        dot0 = fmaf(xr[4 * e + 3], a.w, dot0);
        if (e + 1 < D / 4) {
          const float4 bq = c4[e + 1];
          dot1 = fmaf(xr[4 * e + 4], bq.x, dot1);
          dot1 = fmaf(xr[4 * e + 5], bq.y, dot1);
          dot1 = fmaf(xr[4 * e + 6], bq.z, dot1);
          dot1 = fmaf(xr[4 * e + 7], bq.w, dot1);
        }
      }
      const float dist = fmaxf(xsq + sh_csq[j] - 2.f * (dot0 + dot1), 0.f);
      if (dist < best) {
        best = dist;
        best_idx = k0 + j;
      }
    }
  }
  if (valid) labels[b * n + p] = best_idx;
}

template <int D>
static int launch_assign_d(const void* x, int x_dtype, int64_t bh, int64_t n, int k, const float* c,
                           int32_t* labels, const int* done, cudaStream_t st) {
  dim3 grid((unsigned)((n + kAssignPoints - 1) / kAssignPoints), (unsigned)bh);
  if (x_dtype == SPR_F32)
    assign_simt_kernel<D, float><<<grid, kAssignPoints, 0, st>>>((const float*)x, n, k, c, labels, done);
  else if (x_dtype == SPR_BF16)
    assign_simt_kernel<D, __nv_bfloat16><<<grid, kAssignPoints, 0, st>>>((const __nv_bfloat16*)x, n, k, c, labels, done);
  else
    assign_simt_kernel<D, __half><<<grid, kAssignPoints, 0, st>>>((const __half*)x, n, k, c, labels, done);
  return check_launch("k-means assign");
}

inline int launch_assign(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k, const float* c,
                         int32_t* labels, const int* done, cudaStream_t st) {
  switch (d) {
    case 16: return launch_assign_d<16>(x, x_dtype, bh, n, k, c, labels, done, st);
    case 32: return launch_assign_d<32>(x, x_dtype, bh, n, k, c, labels, done, st);
    case 48: return launch_assign_d<48>(x, x_dtype, bh, n, k, c, labels, done, st);
    case 64: return launch_assign_d<64>(x, x_dtype, bh, n, k, c, labels, done, st);
    case 96: return launch_assign_d<96>(x, x_dtype, bh, n, k, c, labels, done, st);
    case 128: return launch_assign_d<128>(x, x_dtype, bh, n, k, c, labels, done, st);
    default: return fail(SPR_ERR_SHAPE, "k-means assign: unsupported d=%d", d);
  }
}

}  // namespace spr
