// Routing kernel: the budgeted cluster selector (sort + prefix budget +
// crossing cluster + compaction).  The attention-mass scores are in scores.cu.
#include "common.cuh"

namespace spr {


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

// Warp-per-row selector for ck <= 1024 (same keys, order and rule as
// select_budget_kernel, so the result is identical).  Position i = e * 32 +
// lane of the padded row (P = 32 E entries) lives in register e of `lane`; the
// bitonic network's strides >= 32 compare two registers of one lane, strides
// < 32 two lanes (shuffles).  The sorted positions' costs are scanned e-major
// with warp scans; per-id flags go through shared memory for the ascending
// compaction.  No block barriers.
constexpr int kSelWarps = 8;

template <int E>
__global__ void __launch_bounds__(kSelWarps * 32)
select_budget_warp_kernel(const float* __restrict__ scores, const int32_t* __restrict__ sizes,
                          const int32_t* __restrict__ budgets, int64_t rows, int cq, int ck,
                          uint8_t* __restrict__ routed, int32_t* __restrict__ sel_ids,
                          int32_t* __restrict__ sel_counts) {
  constexpr int P = 32 * E;
  __shared__ uint8_t sh_flag[kSelWarps][P];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * kSelWarps + w;
  if (row >= rows) return;  // warp-uniform; no block barrier below
  const int64_t b = row / cq;
  const int q = (int)(row % cq);
  const float* sr = scores + row * ck;
  unsigned long long key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 32 + lane;
    key[e] = i < ck ? (((unsigned long long)float_order_desc(sr[i]) << 32) | (uint32_t)i) : ~0ull;
  }
  // Bitonic sort ascending on (descending score, ascending id).
#pragma unroll
  for (int size = 2; size <= P; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int es = stride / 32;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & es) == 0) {
            const bool up = (((e * 32 + lane) & size) == 0);
            const unsigned long long a = key[e], c = key[e | es];
            if ((a > c) == up) { key[e] = c; key[e | es] = a; }
          }
        }
      } else {
        const bool lo = (lane & stride) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const bool up = (((e * 32 + lane) & size) == 0);
          const unsigned long long v = key[e];
          const uint32_t whi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), stride);
          const uint32_t wlo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, stride);
          const unsigned long long o = ((unsigned long long)whi << 32) | wlo;
          const unsigned long long mn = v < o ? v : o, mx = v < o ? o : v;
          key[e] = (lo == up) ? mn : mx;
        }
      }
    }
  }
  const int32_t budget = budgets[row];
  const int32_t* sz = sizes + b * ck;
  // Costs in sorted order, inclusive prefix of the positive ones, e-major.
  int32_t cost[E];
  bool keep[E];
  int32_t carry = 0, cnt_total = 0, cost_total = 0, valid_total = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const uint32_t id = (uint32_t)key[e];
    const int32_t c = id < (uint32_t)ck ? sz[id] : 0;
    cost[e] = c;
    int32_t x = c > 0 ? c : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    const int32_t cum = carry + x;
    carry += __shfl_sync(0xffffffffu, x, 31);
    keep[e] = c > 0 && cum <= budget;
    cnt_total += __popc(__ballot_sync(0xffffffffu, keep[e]));
    valid_total += __popc(__ballot_sync(0xffffffffu, c > 0));
    int32_t kc = keep[e] ? c : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kc += __shfl_xor_sync(0xffffffffu, kc, o);
    cost_total += kc;
  }
  const bool need = budget > 0 && cost_total < budget && cnt_total < valid_total;
  uint8_t* fl = sh_flag[w];
#pragma unroll
  for (int e = 0; e < E; ++e) fl[e * 32 + lane] = 0;
  __syncwarp();
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const uint32_t id = (uint32_t)key[e];
    if (id < (uint32_t)ck) fl[id] = keep[e] || (need && e * 32 + lane == cnt_total);
  }
  __syncwarp();
  if (routed) {
    uint8_t* rr = routed + (b * (cq + 1) + q + 1) * (int64_t)(ck + 1);
    for (int i = lane; i <= ck; i += 32) rr[i] = i == 0 ? 1 : fl[i - 1];
    if (q == 0) {
      uint8_t* r0 = routed + b * (cq + 1) * (int64_t)(ck + 1);
      for (int i = lane; i <= ck; i += 32) r0[i] = i == 0 ? 1 : 0;
    }
  }
  // Compact selected ids in ascending cluster order.
  int32_t* ids = sel_ids + row * ck;
  int32_t nsel = 0;
  for (int i0 = 0; i0 < ck; i0 += 32) {
    const int i = i0 + lane;
    const bool f = i < ck && fl[i];
    const unsigned m = __ballot_sync(0xffffffffu, f);
    if (f) ids[nsel + __popc(m & ((1u << lane) - 1u))] = i;
    nsel += __popc(m);
  }
  for (int i = nsel + lane; i < ck; i += 32) ids[i] = -1;
  if (lane == 0) sel_counts[row] = nsel;
}

}  // namespace spr

using namespace spr;

extern "C" int spr_select_budget(const float* scores, const int32_t* k_sizes, const int32_t* budgets, int64_t bh,
                                 int cq, int ck, uint8_t* routed, int32_t* sel_ids, int32_t* sel_counts, void* stream) {
  if (bh <= 0 || cq <= 0 || ck <= 0 || ck > 2048)
    return fail(SPR_ERR_SHAPE, "selector: need 0 < ck <= 2048, got ck=%d", ck);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t rows = bh * cq;
  const unsigned wgrid = (unsigned)((rows + kSelWarps - 1) / kSelWarps);
  if (ck <= 1024) {  // one warp per row, keys in registers
    int e = 1;
    while (32 * e < ck) e <<= 1;
    switch (e) {
#define SPR_SEL_CASE(EE)                                                                                        \
  case EE:                                                                                                      \
    select_budget_warp_kernel<EE><<<wgrid, kSelWarps * 32, 0, st>>>(scores, k_sizes, budgets, rows, cq, ck,    \
                                                                    routed, sel_ids, sel_counts);              \
    break;
      SPR_SEL_CASE(1) SPR_SEL_CASE(2) SPR_SEL_CASE(4) SPR_SEL_CASE(8) SPR_SEL_CASE(16) SPR_SEL_CASE(32)
#undef SPR_SEL_CASE
    }
    return check_launch("selector");
  }
  select_budget_kernel<<<(unsigned)rows, 1024, 0, st>>>(scores, k_sizes, budgets, cq, ck, routed, sel_ids,
                                                        sel_counts);
  return check_launch("selector");
}
