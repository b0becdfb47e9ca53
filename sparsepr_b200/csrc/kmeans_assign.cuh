// k-means assignment on the tensor cores: per point, argmin over centroids of
// max(|x|^2 + |c|^2 - 2 x.c, 0), ties to the lowest centroid index.
//
// The cross term x.c is a tcgen05 GEMM (kind::tf32, fp32 accumulation in
// TMEM): 128 points x 128 centroids per MMA tile, the feature dimension padded
// with zeros to a multiple of 32.  Precision SPR_KMEANS_TF32 matches the
// reference's TF32 `tl.dot`; SPR_KMEANS_FP32 splits both operands as
// hi = tf32(v), lo = v - hi and accumulates hi.hi + hi.lo + lo.hi (3xTF32),
// which reproduces fp32 dot products to ~2^-22 relative.
//
// Persistent kernel: one CTA per SM loops over (problem, 128-point tile)
// items.  Warp roles (416 threads): warps 0-7 argmin epilogue (warp w reads
// TMEM lanes 32*(w%4).. and columns 64*(w/4).. of each tile: two threads per
// point, merged per item), warp 8 MMA issuer, warps 9-12 loaders (thread =
// row: the point tile of each item into a double buffer, |x|^2, and a
// continuous stream of centroid tiles with |c|^2 into a 2-stage ring).  TMEM
// holds two 128-column accumulators so the argmin of one tile overlaps the
// next GEMM, across item boundaries too.
#pragma once
#include "tc_common.cuh"

namespace spr {

inline bool assign_supported_dim(int d) { return d >= 4 && d <= 128 && d % 4 == 0; }

constexpr int kAsgM = 128;   // points per item
constexpr int kAsgN = 128;   // centroids per tile
constexpr int kAsgThreads = 416;
constexpr int kAsgLoaders = 128;
constexpr int kAsgEpilogue = 256;
constexpr uint32_t kIdescAsg = tc::idesc_tf32_f32(128, 128);

template <int DP, bool SPLIT>
struct AsgSmem {
  static constexpr int kRowBytes = DP * 4;
  static constexpr int kXBytes = kAsgM * kRowBytes;
  static constexpr int kCBytes = kAsgN * kRowBytes;
  static constexpr int kParts = SPLIT ? 2 : 1;
  static constexpr int kBudget = 200 * 1024;
  static constexpr int kNX = (1024 + 2 * kParts * kXBytes + 2 * kParts * kCBytes <= kBudget) ? 2 : 1;
  // Centroid stages: as many as fit (2..4).
  static constexpr int kNC = (1024 + kNX * kParts * kXBytes + 4 * kParts * kCBytes <= kBudget)   ? 4
                             : (1024 + kNX * kParts * kXBytes + 3 * kParts * kCBytes <= kBudget) ? 3
                                                                                                 : 2;
  static constexpr int kTotal = 1024 + kNX * kParts * kXBytes + kNC * kParts * kCBytes;
};

// |c|^2 per centroid row (one warp per row), skipped once the run has converged.
__global__ void row_sq_kernel(const float* __restrict__ c, int64_t rows, int d, float* __restrict__ out,
                              const int* __restrict__ done) {
  if (done && *done) return;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  float s = 0.f;
  for (int e = lane; e < d; e += 32) s = fmaf(c[w * d + e], c[w * d + e], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[w] = s;
}

__device__ __forceinline__ float tf32_hi(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
  const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}

// Store a float4 (optionally split into tf32 hi/lo parts) at a swizzled chunk.
template <bool SPLIT>
__device__ __forceinline__ void put4(uint32_t hi_base, uint32_t lo_base, uint32_t off, float4 v) {
  if constexpr (SPLIT) {
    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
    const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(hi_base + off), "f"(h.x), "f"(h.y), "f"(h.z), "f"(h.w)
                 : "memory");
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(lo_base + off), "f"(l.x), "f"(l.y), "f"(l.z), "f"(l.w)
                 : "memory");
  } else {
    (void)lo_base;
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(hi_base + off), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
  }
}

template <int DP, bool SPLIT, typename T>
__global__ void __launch_bounds__(kAsgThreads, 1)
assign_tc_kernel(const T* __restrict__ x, int64_t n, int d, int k, int64_t items, const float* __restrict__ centroids,
                 const float* __restrict__ xsq_g, const float* __restrict__ csq_g, int32_t* __restrict__ labels,
                 const int* __restrict__ done, int* __restrict__ err) {
  using L = AsgSmem<DP, SPLIT>;
  constexpr int NX = L::kNX;
  constexpr int NC = L::kNC;
  // fp32 points without the split are copied to shared memory as they are
  // (cp.async, many tiles in flight); other cases go through registers.
  constexpr bool kAsync = !SPLIT && sizeof(T) == 4;
  constexpr int kChunks = DP / 4;  // 16-byte chunks per row
  if (done && *done) return;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_x_full[2], bar_x_empty[2], bar_x_read[2];
  // c_read[s]: the argmin warps are done with |c|^2 of stage s (one completion
  // per stage use, so a parity wait on it can never alias a later use).
  __shared__ uint64_t bar_c_full[NC], bar_c_empty[NC], bar_c_read[NC], bar_d_full[2], bar_d_free[2];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(16) float s_csq[NC][kAsgN];  // read as float2 by the epilogue
  __shared__ __align__(16) float s_xsq[2][kAsgM];
  __shared__ float s_best[kAsgM];
  __shared__ int s_best_idx[kAsgM];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sx0 = tc::smem_addr(smem);                       // X buffer i: hi at sx0 + i*parts*X
  const uint32_t sc0 = sx0 + NX * L::kParts * L::kXBytes;         // C stage s: hi at sc0 + s*parts*C
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ctiles = (k + kAsgN - 1) / kAsgN;
  const int64_t ptiles = (n + kAsgM - 1) / kAsgM;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_x_full[i], kAsgLoaders);
      tc::mbar_init(&bar_x_empty[i], 1);
      tc::mbar_init(&bar_x_read[i], kAsgEpilogue);
      tc::mbar_init(&bar_d_full[i], 1);
      tc::mbar_init(&bar_d_free[i], kAsgEpilogue);
    }
    for (int i = 0; i < NC; ++i) {
      tc::mbar_init(&bar_c_full[i], kAsgLoaders);
      tc::mbar_init(&bar_c_empty[i], 1);
      tc::mbar_init(&bar_c_read[i], kAsgEpilogue);
    }
    tc::mbar_fence_init();
  }
  if (warp == 8) tc::tmem_alloc<256>(&s_tmem);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp >= 9) {
    // ---------------------------------------------------------- loaders
    const int r = tid - 9 * 32;  // register path: thread = row; async path: flat index
    int64_t gt = 0;  // global centroid-tile counter of this CTA
    int il = 0;      // item counter of this CTA
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x, ++il) {
      const int64_t b = it / ptiles;
      const int64_t p0 = (it % ptiles) * kAsgM;
      const int xb = il % NX;
      if (il >= NX) {  // the GEMMs and the epilogue's |x|^2 read of item il-NX are done
        tc::mbar_wait(&bar_x_empty[xb], ((il / NX) - 1) & 1, err, 21);
        tc::mbar_wait(&bar_x_read[xb], ((il / NX) - 1) & 1, err, 21);
      }
      const uint32_t xhi = sx0 + xb * L::kParts * L::kXBytes;
      if constexpr (kAsync) {
        const float* xg = reinterpret_cast<const float*>(x) + (b * n + p0) * d;
        for (int idx = r; idx < kAsgM * kChunks; idx += kAsgLoaders) {
          const int row = idx / kChunks, ch = idx % kChunks;
          const bool ok = p0 + row < n && ch * 4 < d;
          tc::cp_async16(xhi + tc::sw128_off(row, ch, kAsgM), ok ? xg + (int64_t)row * d + ch * 4 : xg, ok);
        }
        {  // |x|^2 of row r (4-byte copies: b*n need not be a multiple of 4)
          const bool ok = p0 + r < n;
          tc::cp_async4(tc::smem_addr(&s_xsq[xb][r]), ok ? xsq_g + b * n + p0 + r : xsq_g, ok);
        }
        tc::cp_async_arrive(&bar_x_full[xb]);
      } else {
        const uint32_t xlo = xhi + (SPLIT ? L::kXBytes : 0);
        const T* xr = x + (b * n + p0 + r) * d;
        const bool row_ok = p0 + r < n;
        float sq = 0.f;
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (row_ok && ch * 4 < d) v = load4<T>(xr + ch * 4);
          sq = fmaf(v.x, v.x, sq);
          sq = fmaf(v.y, v.y, sq);
          sq = fmaf(v.z, v.z, sq);
          sq = fmaf(v.w, v.w, sq);
          put4<SPLIT>(xhi, xlo, tc::sw128_off(r, ch, kAsgM), v);
        }
        s_xsq[xb][r] = sq;
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&bar_x_full[xb]);
      }
      const float* cb = centroids + b * (int64_t)k * d;
      for (int t = 0; t < ctiles; ++t, ++gt) {
        const int st = (int)(gt % NC);
        const int use = (int)(gt / NC);
        const uint32_t hi = sc0 + st * L::kParts * L::kCBytes;
        if constexpr (kAsync) {
          if (gt >= NC) {  // the GEMM and the argmin of tile gt-NC are both done with this stage
            tc::mbar_wait(&bar_c_empty[st], (use - 1) & 1, err, 11);
            tc::mbar_wait(&bar_c_read[st], (use - 1) & 1, err, 11);
          }
          const int k0 = t * kAsgN;
          for (int idx = r; idx < kAsgN * kChunks; idx += kAsgLoaders) {
            const int row = idx / kChunks, ch = idx % kChunks;
            const bool ok = k0 + row < k && ch * 4 < d;
            tc::cp_async16(hi + tc::sw128_off(row, ch, kAsgN), ok ? cb + (int64_t)(k0 + row) * d + ch * 4 : cb, ok);
          }
          {  // |c|^2 of centroid k0 + r
            const bool ok = k0 + r < k;
            tc::cp_async4(tc::smem_addr(&s_csq[st][r]), ok ? csq_g + b * (int64_t)k + k0 + r : csq_g, ok);
          }
          tc::cp_async_arrive(&bar_c_full[st]);
        } else {
          const int kc = t * kAsgN + r;
          float4 v[kChunks];
          float sq = 0.f;
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) {
            v[ch] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kc < k && ch * 4 < d) v[ch] = *reinterpret_cast<const float4*>(cb + (int64_t)kc * d + ch * 4);
            sq = fmaf(v[ch].x, v[ch].x, sq);
            sq = fmaf(v[ch].y, v[ch].y, sq);
            sq = fmaf(v[ch].z, v[ch].z, sq);
            sq = fmaf(v[ch].w, v[ch].w, sq);
          }
          if (gt >= NC) {
            tc::mbar_wait(&bar_c_empty[st], (use - 1) & 1, err, 11);
            tc::mbar_wait(&bar_c_read[st], (use - 1) & 1, err, 11);
          }
          const uint32_t lo = hi + (SPLIT ? L::kCBytes : 0);
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) put4<SPLIT>(hi, lo, tc::sw128_off(r, ch, kAsgN), v[ch]);
          s_csq[st][r] = sq;
          tc::fence_proxy_async_smem();
          tc::mbar_arrive(&bar_c_full[st]);
        }
      }
    }
    if constexpr (kAsync) tc::cp_async_wait_all();
  } else if (warp == 8) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int64_t gt = 0;
      int il = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < items; it += gridDim.x, ++il) {
        const int xb = il % NX;
        if (!(ok = tc::mbar_wait(&bar_x_full[xb], (il / NX) & 1, err, 12))) break;
        const uint32_t xhi = sx0 + xb * L::kParts * L::kXBytes;
        const uint32_t xlo = xhi + (SPLIT ? L::kXBytes : 0);
        for (int t = 0; t < ctiles; ++t, ++gt) {
          const int st = (int)(gt % NC);
          const int db = (int)(gt & 1);
          if (!(ok = tc::mbar_wait(&bar_c_full[st], (int)((gt / NC) & 1), err, 12))) break;
          if (gt >= 2 && !(ok = tc::mbar_wait(&bar_d_free[db], (int)(((gt >> 1) - 1) & 1), err, 12))) break;
          tc::tc_fence_after();
          const uint32_t chi = sc0 + st * L::kParts * L::kCBytes;
          const uint32_t clo = chi + (SPLIT ? L::kCBytes : 0);
          const uint32_t dt = tmem + db * 128;
#pragma unroll
          for (int kk = 0; kk < DP / 8; ++kk) {  // 8 tf32 = 32 bytes per MMA K step
            const uint32_t kb = kk * 32;
            const uint32_t oa = (kb >> 7) * (kAsgM * 128) + (kb & 127);
            const uint32_t ob = (kb >> 7) * (kAsgN * 128) + (kb & 127);
            tc::mma_tf32(dt, tc::sw128_desc(xhi + oa, 16, 1024), tc::sw128_desc(chi + ob, 16, 1024), kIdescAsg,
                         kk > 0);
            if constexpr (SPLIT) {
              tc::mma_tf32(dt, tc::sw128_desc(xhi + oa, 16, 1024), tc::sw128_desc(clo + ob, 16, 1024), kIdescAsg, 1);
              tc::mma_tf32(dt, tc::sw128_desc(xlo + oa, 16, 1024), tc::sw128_desc(chi + ob, 16, 1024), kIdescAsg, 1);
            }
          }
          tc::mma_commit(&bar_d_full[db]);
          tc::mma_commit(&bar_c_empty[st]);
          if (t == ctiles - 1) tc::mma_commit(&bar_x_empty[xb]);
        }
      }
    }
  } else {
    // ---------------------------------------------------------- argmin epilogue
    const int row = tid & 127;
    const int colh = tid >> 7;  // 64-column half of each tile scanned by this thread
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int64_t gt = 0;
    int il = 0;
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x, ++il) {
      const int64_t b = it / ptiles;
      const int64_t p = (it % ptiles) * kAsgM + row;
      const int xb = il % NX;
      ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_x_full[xb], (il / NX) & 1, err, 13));
      const float xsq = s_xsq[xb][row];
      tc::mbar_arrive(&bar_x_read[xb]);
      float best = 3.4e38f;
      int best_idx = 0x7fffffff;
      for (int t = 0; t < ctiles; ++t, ++gt) {
        const int st = (int)(gt & 1);   // TMEM buffer
        const int cs = (int)(gt % NC);  // centroid stage (|c|^2)
        ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_d_full[st], (int)((gt >> 1) & 1), err, 13));
        tc::tc_fence_after();
        const int k0 = t * kAsgN;
        if (ok) {
          // dist = max(|x|^2 + |c|^2 - 2 x.c, 0) is compared as
          // t = max(|c|^2 - 2 x.c, -|x|^2): the same order and the same
          // clamp, one FFMA + one FMNMX per column.
          const float floor_t = -xsq;
          const bool full = k0 + kAsgN <= k;  // only the last centroid tile is partial
#pragma unroll 1
          for (int cb = 2 * colh; cb < 2 * colh + 2; ++cb) {
            float acc[32];
            tc::tmem_ld32(tmem + lane_base + st * 128 + cb * 32, acc);
            const float* cq = &s_csq[cs][cb * 32];
            // Two interleaved first-minimum chains (even / odd columns) with
            // column offsets as immediates; merged with the lower index on ties.
            float b0 = 3.4e38f, b1 = 3.4e38f;
            int j0 = 0, j1 = 1;
            if (full) {
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float2 c2 = *reinterpret_cast<const float2*>(cq + j);
                const float t0 = fmaxf(fmaf(-2.f, acc[j], c2.x), floor_t);
                const float t1 = fmaxf(fmaf(-2.f, acc[j + 1], c2.y), floor_t);
                if (t0 < b0) { b0 = t0; j0 = j; }
                if (t1 < b1) { b1 = t1; j1 = j + 1; }
              }
            } else {
              const int lim = k - (k0 + cb * 32);  // valid columns in this block (may be <= 0)
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                const float2 c2 = *reinterpret_cast<const float2*>(cq + j);
                const float t0 = fmaxf(fmaf(-2.f, acc[j], c2.x), floor_t);
                const float t1 = fmaxf(fmaf(-2.f, acc[j + 1], c2.y), floor_t);
                if (j < lim && t0 < b0) { b0 = t0; j0 = j; }
                if (j + 1 < lim && t1 < b1) { b1 = t1; j1 = j + 1; }
              }
            }
            if (b1 < b0 || (b1 == b0 && j1 < j0)) { b0 = b1; j0 = j1; }
            if (b0 < best) { best = b0; best_idx = k0 + cb * 32 + j0; }
          }
        }
        tc::tc_fence_before();
        tc::mbar_arrive(&bar_d_free[st]);
        tc::mbar_arrive(&bar_c_read[cs]);
      }
      // Merge the two column halves of each point (equal distances: lower index).
      if (colh == 1) { s_best[row] = best; s_best_idx[row] = best_idx; }
      tc::named_bar(1, kAsgEpilogue);
      if (colh == 0) {
        const float ob = s_best[row];
        const int oi = s_best_idx[row];
        if (ob < best || (ob == best && oi < best_idx)) { best = ob; best_idx = oi; }
        if (best_idx == 0x7fffffff) best_idx = 0;
        if (p < n) labels[b * n + p] = best_idx;
      }
      tc::named_bar(1, kAsgEpilogue);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc<256>(tmem);
  }
}

template <int DP, bool SPLIT, typename T>
static int launch_assign_tc(const void* x, int64_t bh, int64_t n, int d, int k, const float* c, const float* xsq,
                            const float* csq, int32_t* labels, const int* done, int* err, cudaStream_t st) {
  constexpr int smem = AsgSmem<DP, SPLIT>::kTotal;
  auto kern = assign_tc_kernel<DP, SPLIT, T>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = bh * ((n + kAsgM - 1) / kAsgM);
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);  // persistent: one CTA per SM
  kern<<<grid, kAsgThreads, smem, st>>>((const T*)x, n, d, k, items, c, xsq, csq, labels, done, err);
  return check_launch("k-means assign (tcgen05)");
}

template <bool SPLIT, typename T>
static int launch_assign_dp(const void* x, int64_t bh, int64_t n, int d, int k, const float* c, const float* xsq,
                            const float* csq, int32_t* labels, const int* done, int* err, cudaStream_t st) {
  if (d <= 32) return launch_assign_tc<32, SPLIT, T>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
  if (d <= 64) return launch_assign_tc<64, SPLIT, T>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
  if constexpr (!SPLIT) {
    if (d <= 96) return launch_assign_tc<96, SPLIT, T>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
    return launch_assign_tc<128, SPLIT, T>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
  } else {
    return fail(SPR_ERR_UNIMPLEMENTED, "k-means assign: fp32 (3xTF32) precision supports d <= 64, got d=%d", d);
  }
}

// |x|^2 for fp32 points (call once per k-means run: x does not change).
inline int launch_point_sq(const void* x, int x_dtype, int64_t bh, int64_t n, int d, float* xsq, cudaStream_t st) {
  if (x_dtype != SPR_F32) return SPR_OK;  // other dtypes compute |x|^2 inside the assignment kernel
  const int64_t rows = bh * n;
  row_sq_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>((const float*)x, rows, d, xsq, nullptr);
  return check_launch("point norms");
}

// |c|^2 of the current centroids, then the assignment GEMM (xsq from launch_point_sq).
inline int launch_assign(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k, const float* c,
                         const float* xsq, float* csq, int precision, int32_t* labels, const int* done, int* err,
                         cudaStream_t st) {
  const int64_t crows = bh * k;
  row_sq_kernel<<<(unsigned)((crows * 32 + 255) / 256), 256, 0, st>>>(c, crows, d, csq, done);
  int s = check_launch("centroid norms");
  if (s) return s;
  const bool split = precision == SPR_KMEANS_FP32;
  if (x_dtype == SPR_F32)
    return split ? launch_assign_dp<true, float>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st)
                 : launch_assign_dp<false, float>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
  if (x_dtype == SPR_BF16)
    return split ? launch_assign_dp<true, __nv_bfloat16>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st)
                 : launch_assign_dp<false, __nv_bfloat16>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
  return split ? launch_assign_dp<true, __half>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st)
               : launch_assign_dp<false, __half>(x, bh, n, d, k, c, xsq, csq, labels, done, err, st);
}

}  // namespace spr
