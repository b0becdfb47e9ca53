// Routing kernels: attention-mass selector scores and the budgeted
// cluster selector (sort + prefix budget + crossing cluster + compaction).
#include "common.cuh"

namespace spr {

constexpr int kScoreTok = 16;  // key rows staged per step

// One block per (key cluster, problem); each thread owns query centroids and
// keeps an online log-sum-exp over the cluster's key rows (exact fp32 dots).
__global__ void __launch_bounds__(256)
attention_mass_scores_kernel(const float* __restrict__ qc, const __nv_bfloat16* __restrict__ ks,
                             const int32_t* __restrict__ koff, int cq, int ck, int64_t n,
                             float* __restrict__ scores) {
  constexpr int D = 128;
  __shared__ __align__(16) float sh_k[kScoreTok][D];
  const int c = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int32_t beg = koff[b * (ck + 1) + c], end = koff[b * (ck + 1) + c + 1];
  const float scale = rsqrtf((float)D);
  const float* qb = qc + b * (int64_t)cq * D;
  const __nv_bfloat16* kb = ks + b * n * D;
  // Up to 2 query centroids per thread (cq <= 512).
  float m[2] = {-INFINITY, -INFINITY}, s[2] = {0.f, 0.f};
  for (int32_t t0 = beg; t0 < end; t0 += kScoreTok) {
    const int nt = min(kScoreTok, end - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < kScoreTok * D / 8; i += blockDim.x) {
      const int r = i / (D / 8), cidx = i % (D / 8);
      float f[8];
      if (r < nt) {
        const uint4 v = reinterpret_cast<const uint4*>(kb + (int64_t)(t0 + r) * D)[cidx];
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __bfloat162float(h[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) sh_k[r][cidx * 8 + e] = f[e];
    }
    __syncthreads();
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int q = threadIdx.x + slot * blockDim.x;
      if (q >= cq) continue;
      const float4* q4 = reinterpret_cast<const float4*>(qb + (int64_t)q * D);
      float dots[kScoreTok];
#pragma unroll
      for (int j = 0; j < kScoreTok; ++j) dots[j] = 0.f;
      for (int e4 = 0; e4 < D / 4; ++e4) {
        const float4 qv = __ldg(q4 + e4);
#pragma unroll
        for (int j = 0; j < kScoreTok; ++j) {
          const float4 kv = reinterpret_cast<const float4*>(sh_k[j])[e4];
          dots[j] = fmaf(qv.x, kv.x, dots[j]);
          dots[j] = fmaf(qv.y, kv.y, dots[j]);
          dots[j] = fmaf(qv.z, kv.z, dots[j]);
          dots[j] = fmaf(qv.w, kv.w, dots[j]);
        }
      }
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < kScoreTok; ++j)
        if (j < nt) cm = fmaxf(cm, dots[j] * scale);
      const float nm = fmaxf(m[slot], cm);
      float acc = s[slot] * __expf(m[slot] - nm);
#pragma unroll
      for (int j = 0; j < kScoreTok; ++j)
        if (j < nt) acc += __expf(dots[j] * scale - nm);
      s[slot] = acc;
      m[slot] = nm;
    }
  }
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int q = threadIdx.x + slot * blockDim.x;
    if (q >= cq) continue;
    const float v = end > beg ? logf(fmaxf(s[slot], 1e-30f)) + m[slot] : -INFINITY;
    scores[(b * cq + q) * (int64_t)ck + c] = v;
  }
}

__device__ __forceinline__ uint32_t float_order_desc(float f) {
  uint32_t u = __float_as_uint(f);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending-orderable
  return ~u;                                         // descending
}

// Block-wide exclusive scan (blockDim multiple of 32); *total = block sum.
__device__ int32_t block_exclusive_scan(int32_t v, int32_t* sh_warp, int32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < nw ? sh_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) sh_warp[lane] = w;
  }
  __syncthreads();
  const int32_t warp_base = warp > 0 ? sh_warp[warp - 1] : 0;
  *total = sh_warp[nw - 1];
  __syncthreads();
  return warp_base + x - v;
}

// One block (1024 threads) per (problem, query cluster) row; ck <= 2048.
__global__ void __launch_bounds__(1024)
select_budget_kernel(const float* __restrict__ scores, const int32_t* __restrict__ sizes,
                     const int32_t* __restrict__ budgets, int cq, int ck, uint8_t* __restrict__ routed,
                     int32_t* __restrict__ sel_ids, int32_t* __restrict__ sel_counts) {
  __shared__ unsigned long long sh_key[2048];
  __shared__ uint8_t sh_flag[2048];
  __shared__ int32_t sh_warp[32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / cq;
  const int q = (int)(row % cq);
  int P = 1;
  while (P < ck) P <<= 1;
  const float* sr = scores + row * ck;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    unsigned long long key = ~0ull;
    if (i < ck) key = ((unsigned long long)float_order_desc(sr[i]) << 32) | (uint32_t)i;
    sh_key[i] = key;
  }
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) sh_flag[i] = 0;
  __syncthreads();
  // Bitonic sort ascending on (descending score, ascending id).
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = sh_key[i], c = sh_key[j];
          if ((a > c) == up) { sh_key[i] = c; sh_key[j] = a; }
        }
      }
      __syncthreads();
    }
  }
  const int32_t budget = budgets[row];
  const int32_t* sz = sizes + b * ck;
  // Prefix of positive costs in sorted order: two positions per thread.
  const int i0 = 2 * threadIdx.x, i1 = i0 + 1;
  const int32_t c0 = i0 < ck ? sz[(uint32_t)sh_key[i0]] : 0;
  const int32_t c1 = i1 < ck ? sz[(uint32_t)sh_key[i1]] : 0;
  const int32_t p0 = c0 > 0 ? c0 : 0, p1 = c1 > 0 ? c1 : 0;
  int32_t tot;
  const int32_t ex = block_exclusive_scan(p0 + p1, sh_warp, &tot);
  const int32_t cum0 = ex + p0, cum1 = ex + p0 + p1;
  const bool k0 = c0 > 0 && cum0 <= budget, k1 = c1 > 0 && cum1 <= budget;
  int32_t cnt_total, cost_total, valid_total;
  block_exclusive_scan((int)k0 + (int)k1, sh_warp, &cnt_total);
  block_exclusive_scan((k0 ? c0 : 0) + (k1 ? c1 : 0), sh_warp, &cost_total);
  block_exclusive_scan((int)(c0 > 0) + (int)(c1 > 0), sh_warp, &valid_total);
  const bool need = budget > 0 && cost_total < budget && cnt_total < valid_total;
  if (i0 < ck) sh_flag[(uint32_t)sh_key[i0]] = k0 || (need && i0 == cnt_total);
  if (i1 < ck) sh_flag[(uint32_t)sh_key[i1]] = k1 || (need && i1 == cnt_total);
  __syncthreads();
  if (routed) {
    uint8_t* rr = routed + (b * (cq + 1) + q + 1) * (int64_t)(ck + 1);
    for (int i = threadIdx.x; i <= ck; i += blockDim.x) rr[i] = i == 0 ? 1 : sh_flag[i - 1];
    if (q == 0) {
      uint8_t* r0 = routed + b * (cq + 1) * (int64_t)(ck + 1);
      for (int i = threadIdx.x; i <= ck; i += blockDim.x) r0[i] = i == 0 ? 1 : 0;
    }
  }
  // Compact selected ids in ascending cluster order.
  const int32_t f0 = i0 < ck ? sh_flag[i0] : 0, f1 = i1 < ck ? sh_flag[i1] : 0;
  int32_t nsel;
  const int32_t pos = block_exclusive_scan(f0 + f1, sh_warp, &nsel);
  int32_t* ids = sel_ids + row * ck;
  if (f0) ids[pos] = i0;
  if (f1) ids[pos + f0] = i1;
  for (int i = nsel + threadIdx.x; i < ck; i += blockDim.x) ids[i] = -1;
  if (threadIdx.x == 0) sel_counts[row] = nsel;
}

}  // namespace spr

using namespace spr;

extern "C" int spr_attention_mass_scores(const float* q_centroids, const void* k_sorted, const int32_t* k_offsets,
                                         int64_t bh, int cq, int ck, int64_t n, int d, float* scores, void* stream) {
  if (d != 128) return fail(SPR_ERR_SHAPE, "attention-mass scores require d=128, got %d", d);
  if (bh <= 0 || cq <= 0 || ck <= 0 || cq > 512 || bh > 65535)
    return fail(SPR_ERR_SHAPE, "attention-mass scores: bad shape bh=%lld cq=%d ck=%d", (long long)bh, cq, ck);
  if (!aligned(q_centroids, 16) || !aligned(k_sorted, 16))
    return fail(SPR_ERR_ALIGN, "attention-mass scores: 16-byte alignment required");
  dim3 grid((unsigned)ck, (unsigned)bh);
  attention_mass_scores_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      q_centroids, (const __nv_bfloat16*)k_sorted, k_offsets, cq, ck, n, scores);
  return check_launch("attention-mass scores");
}

extern "C" int spr_select_budget(const float* scores, const int32_t* k_sizes, const int32_t* budgets, int64_t bh,
                                 int cq, int ck, uint8_t* routed, int32_t* sel_ids, int32_t* sel_counts, void* stream) {
  if (bh <= 0 || cq <= 0 || ck <= 0 || ck > 2048)
    return fail(SPR_ERR_SHAPE, "selector: need 0 < ck <= 2048, got ck=%d", ck);
  select_budget_kernel<<<(unsigned)(bh * cq), 1024, 0, (cudaStream_t)stream>>>(scores, k_sizes, budgets, cq, ck,
                                                                                routed, sel_ids, sel_counts);
  return check_launch("selector");
}
