// Row-level HBM kernels: permute / inverse permute, repair apply with the
// exact probe-row overwrite, and the library's error/version plumbing.
#include "common.cuh"

namespace spr {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

// Each warp moves rows with 16-byte accesses; `cpr` chunks per row.
__global__ void permute_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ idx,
                                    uint4* __restrict__ y, int64_t n, int cpr, int inverse, int64_t total_rows) {
  const int lane = threadIdx.x & 31;
  const int rpw = 32 / cpr;
  const int sub = lane / cpr, ch = lane % cpr;
  if (sub >= rpw) return;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp * rpw + sub; r < total_rows; r += nwarps * rpw) {
    const int64_t b = r / n;
    const int64_t t = idx[r];
    const int64_t src = inverse ? r : b * n + t;
    const int64_t dst = inverse ? b * n + t : r;
    y[dst * cpr + ch] = x[src * cpr + ch];
  }
}

// Repair: out = bf16(base + alpha*((((base - xm)/xs) L) B^T + ym))
// (kernels/triton/residual_repair.py:96-160, wrapper 478-562; one rounding).  One thread per row.  Per head the block
// folds the standardisation into the left factor, L'[d][j] = L[d][j] / xs[d]
// and c0[j] = -sum_d (xm[d] / xs[d]) L[d][j], so coords = v L' + c0; the row
// streams in 16-byte chunks twice (coords, then the output; the second read
// hits L1/L2) and the weights are shared-memory broadcasts (every lane of a
// warp reads the same address).  ~4k FMAs per row, no shuffles.
template <int D, int R>
__global__ void __launch_bounds__(256)
repair_apply_kernel(const __nv_bfloat16* __restrict__ base, const float* __restrict__ xm,
                    const float* __restrict__ xs, const float* __restrict__ ym, const float* __restrict__ left,
                    const float* __restrict__ basis, int64_t n, float alpha, __nv_bfloat16* __restrict__ out) {
  static_assert(R % 4 == 0 && D % 8 == 0, "repair apply tiling");
  __shared__ float4 sh_l[D][R / 4], sh_b[D][R / 4];
  __shared__ float sh_c0[R], sh_ym[D];
  const int64_t b = blockIdx.y;
  for (int i = threadIdx.x; i < D; i += blockDim.x) sh_ym[i] = ym[b * D + i];
  float* lf = reinterpret_cast<float*>(sh_l);
  float* bf = reinterpret_cast<float*>(sh_b);
  for (int i = threadIdx.x; i < D * R; i += blockDim.x) {  // [d][j] layout, as stored
    lf[i] = __fdiv_rn(left[b * D * R + i], xs[b * D + i / R]);
    bf[i] = basis[b * D * R + i];
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float c = 0.f;
    for (int d = 0; d < D; ++d) c = fmaf(-xm[b * D + d], lf[d * R + threadIdx.x], c);
    sh_c0[threadIdx.x] = c;
  }
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const uint4* row = reinterpret_cast<const uint4*>(base + (b * n + r) * D);
  float coord[R];
#pragma unroll
  for (int j = 0; j < R; ++j) coord[j] = sh_c0[j];
#pragma unroll 2
  for (int c = 0; c < D / 8; ++c) {
    const uint4 u = row[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 v = __bfloat1622float2(h[e]);
#pragma unroll
      for (int q = 0; q < R / 4; ++q) {
        const float4 l0 = sh_l[8 * c + 2 * e][q], l1 = sh_l[8 * c + 2 * e + 1][q];
        coord[4 * q] = fmaf(v.y, l1.x, fmaf(v.x, l0.x, coord[4 * q]));
        coord[4 * q + 1] = fmaf(v.y, l1.y, fmaf(v.x, l0.y, coord[4 * q + 1]));
        coord[4 * q + 2] = fmaf(v.y, l1.z, fmaf(v.x, l0.z, coord[4 * q + 2]));
        coord[4 * q + 3] = fmaf(v.y, l1.w, fmaf(v.x, l0.w, coord[4 * q + 3]));
      }
    }
  }
  uint4* orow = reinterpret_cast<uint4*>(out + (b * n + r) * D);
#pragma unroll 2
  for (int c = 0; c < D / 8; ++c) {
    const uint4 u = row[c];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 v = __bfloat1622float2(h[e]);
      float c0 = sh_ym[8 * c + 2 * e], c1 = sh_ym[8 * c + 2 * e + 1];
#pragma unroll
      for (int q = 0; q < R / 4; ++q) {
        const float4 b0 = sh_b[8 * c + 2 * e][q], b1 = sh_b[8 * c + 2 * e + 1][q];
        c0 = fmaf(coord[4 * q + 3], b0.w, fmaf(coord[4 * q + 2], b0.z, fmaf(coord[4 * q + 1], b0.y, fmaf(coord[4 * q], b0.x, c0))));
        c1 = fmaf(coord[4 * q + 3], b1.w, fmaf(coord[4 * q + 2], b1.z, fmaf(coord[4 * q + 1], b1.y, fmaf(coord[4 * q], b1.x, c1))));
      }
      oh[e] = __floats2bfloat162_rn(fmaf(alpha, c0, v.x), fmaf(alpha, c1, v.y));
    }
    orow[c] = o;
  }
}

// Overwrite probe rows with their exact dense attention output.
__global__ void probe_scatter_kernel(const int32_t* __restrict__ rows, const uint4* __restrict__ dense, int m,
                                     int64_t n, int cpr, uint4* __restrict__ out) {
  const int64_t b = blockIdx.y;
  const int j = blockIdx.x;
  const int64_t r = rows[b * m + j];
  for (int c = threadIdx.x; c < cpr; c += blockDim.x) out[(b * n + r) * cpr + c] = dense[(b * m + j) * (int64_t)cpr + c];
}

}  // namespace spr

using namespace spr;

// Role-equal probe representatives (models/cosmos3/residual_repair.py:118-208, the heavy
// token pass): per (head, cluster) the mean of the cluster's role features
// and the token nearest to it (squared distance, ties to the lowest token
// index; n for an empty cluster).  One warp per cluster walks the cluster's
// tokens in sorted order (ascending token index within a cluster).  Mean:
// 16-byte loads, r/4 lanes per row and 32/(r/4) rows per warp instruction,
// eight rows per lane in flight; each lane sums its chunk over its rows in
// sorted order, then the row groups are added in a fixed order (shuffles).
// Distances: lane j takes tokens j, j + 32, ... of the cluster (two per
// iteration) and computes each full distance against the mean in shared
// memory (no shuffles per token); one warp argmin at the end.
constexpr int kProbeWarps = 8;

__global__ void __launch_bounds__(kProbeWarps * 32)
probe_representatives_kernel(const float* __restrict__ feat, const int32_t* __restrict__ order,
                             const int32_t* __restrict__ offsets, int64_t n, int r, int k, int64_t total,
                             int32_t* __restrict__ best) {
  __shared__ __align__(16) float sh_mean[kProbeWarps][64];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t w = (int64_t)blockIdx.x * kProbeWarps + wib;
  if (w >= total) return;  // warp-uniform; no block-wide barrier below
  const int64_t b = w / k;
  const int c = (int)(w % k);
  const int32_t beg = offsets[b * (k + 1) + c], end = offsets[b * (k + 1) + c + 1];
  if (end <= beg) {
    if (lane == 0) best[w] = (int32_t)n;
    return;
  }
  const int32_t* ob = order + b * n;
  const float* fb = feat + b * n * r;
  const int cpr = r / 4;                  // float4 chunks per row
  const int rpw = 32 / cpr;               // rows per warp instruction (r <= 64: at least 2)
  const int q = lane % cpr, sub = lane / cpr;
  const bool act = sub < rpw;
  float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
  if (act) {
    constexpr int U = 8;
    for (int32_t i = beg + sub; i < end; i += U * rpw) {
      float4 a[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int32_t ii = i + u * rpw;
        a[u] = ii < end ? reinterpret_cast<const float4*>(fb + (int64_t)ob[ii] * r)[q]
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        m.x += a[u].x; m.y += a[u].y; m.z += a[u].z; m.w += a[u].w;
      }
    }
  }
  // Row groups sub = 0 .. rpw-1 added in order into group 0.
  for (int g = 1; g < rpw; ++g) {
    const float4 o = make_float4(__shfl_sync(0xffffffffu, m.x, g * cpr + q), __shfl_sync(0xffffffffu, m.y, g * cpr + q),
                                 __shfl_sync(0xffffffffu, m.z, g * cpr + q), __shfl_sync(0xffffffffu, m.w, g * cpr + q));
    if (sub == 0) { m.x += o.x; m.y += o.y; m.z += o.z; m.w += o.w; }
  }
  const float cnt = (float)(end - beg);
  if (sub == 0)
    reinterpret_cast<float4*>(sh_mean[wib])[q] =
        make_float4(__fdiv_rn(m.x, cnt), __fdiv_rn(m.y, cnt), __fdiv_rn(m.z, cnt), __fdiv_rn(m.w, cnt));
  __syncwarp();
  float best_d = INFINITY;
  int32_t best_t = (int32_t)n;
  const float4* mu = reinterpret_cast<const float4*>(sh_mean[wib]);
  // Squared distance of token t's row to the mean, in a fixed order (two chains).
  auto dist = [&](int32_t t) {
    const float4* row = reinterpret_cast<const float4*>(fb + (int64_t)t * r);
    float d0 = 0.f, d1 = 0.f;
    for (int qq = 0; qq < cpr; qq += 2) {
      const float4 x0 = row[qq], c0 = mu[qq];
      d0 = fmaf(x0.x - c0.x, x0.x - c0.x, d0);
      d0 = fmaf(x0.y - c0.y, x0.y - c0.y, d0);
      d0 = fmaf(x0.z - c0.z, x0.z - c0.z, d0);
      d0 = fmaf(x0.w - c0.w, x0.w - c0.w, d0);
      if (qq + 1 < cpr) {
        const float4 x1 = row[qq + 1], c1 = mu[qq + 1];
        d1 = fmaf(x1.x - c1.x, x1.x - c1.x, d1);
        d1 = fmaf(x1.y - c1.y, x1.y - c1.y, d1);
        d1 = fmaf(x1.z - c1.z, x1.z - c1.z, d1);
        d1 = fmaf(x1.w - c1.w, x1.w - c1.w, d1);
      }
    }
    return d0 + d1;
  };
  for (int32_t i = beg + lane; i < end; i += 64) {  // tokens i and i + 32 of this lane, ascending
    const int32_t t0 = ob[i];
    const bool two = i + 32 < end;
    const int32_t t1 = two ? ob[i + 32] : t0;
    const float da = dist(t0), db = dist(t1);
    if (da < best_d) {  // tokens of a lane ascend: strict keeps the lower one
      best_d = da;
      best_t = t0;
    }
    if (two && db < best_d) {
      best_d = db;
      best_t = t1;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float od = __shfl_xor_sync(0xffffffffu, best_d, o);
    const int32_t ot = __shfl_xor_sync(0xffffffffu, best_t, o);
    if (od < best_d || (od == best_d && ot < best_t)) {
      best_d = od;
      best_t = ot;
    }
  }
  if (lane == 0) best[w] = best_t;
}

extern "C" int spr_probe_representatives(const float* feat, const int32_t* order, const int32_t* offsets, int64_t bh,
                                         int64_t n, int r, int k, int32_t* best, void* stream) {
  if (bh <= 0 || n <= 0 || n > INT32_MAX || k <= 0 || r <= 0 || r > 64)
    return fail(SPR_ERR_SHAPE, "probe representatives: bh=%lld n=%lld r=%d k=%d unsupported (r <= 64)",
                (long long)bh, (long long)n, r, k);
  if (r % 4) return fail(SPR_ERR_SHAPE, "probe representatives: r=%d must be a multiple of 4", r);
  if (!aligned(feat, 16)) return fail(SPR_ERR_ALIGN, "probe representatives: features must be 16-byte aligned");
  const int64_t total = bh * k;
  probe_representatives_kernel<<<(unsigned)((total + kProbeWarps - 1) / kProbeWarps), kProbeWarps * 32, 0,
                                 (cudaStream_t)stream>>>(feat, order, offsets, n, r, k, total, best);
  return check_launch("probe representatives");
}

extern "C" int spr_version(void) { return 100; }
extern "C" const char* spr_last_error(void) { return g_last_error; }

extern "C" int spr_permute_rows(const void* x, const int32_t* idx, void* y, int64_t bh, int64_t n, int d,
                                int elem_bytes, int inverse, void* stream) {
  const int64_t rb = (int64_t)d * elem_bytes;
  if (bh <= 0 || n <= 0 || rb % 16 != 0 || rb / 16 > 32)
    return fail(SPR_ERR_SHAPE, "permute: row of %lld bytes unsupported", (long long)rb);
  if (!aligned(x, 16) || !aligned(y, 16)) return fail(SPR_ERR_ALIGN, "permute: 16-byte alignment required");
  const int64_t rows = bh * n;
  const int blocks = (int)std::min<int64_t>((rows + 7) / 8, 148 * 16);
  permute_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint4*)x, idx, (uint4*)y, n, (int)(rb / 16),
                                                                inverse, rows);
  return check_launch("permute");
}

extern "C" int spr_repair_apply(const void* base, const float* x_mean, const float* x_scale, const float* y_mean,
                                const float* left, const float* basis, int64_t bh, int64_t n, int d, int r,
                                float alpha, const int32_t* rows, const void* dense, int m, void* out, void* stream) {
  if (d != 128 || r != 16) return fail(SPR_ERR_SHAPE, "repair apply: requires d=128, r=16 (got d=%d r=%d)", d, r);
  if (bh <= 0 || n <= 0 || bh > 65535) return fail(SPR_ERR_SHAPE, "repair apply: bad shape");
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)((n + 255) / 256), (unsigned)bh);  // one thread per row
  repair_apply_kernel<128, 16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)base, x_mean, x_scale, y_mean, left, basis,
                                                     n, alpha, (__nv_bfloat16*)out);
  int s = check_launch("repair apply");
  if (s) return s;
  if (rows && dense && m > 0) {
    probe_scatter_kernel<<<dim3((unsigned)m, (unsigned)bh), 32, 0, st>>>(rows, (const uint4*)dense, m, n, 16, (uint4*)out);
    return check_launch("probe scatter");
  }
  return SPR_OK;
}
