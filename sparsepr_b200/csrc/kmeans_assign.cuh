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
#include "tmap.cuh"

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

// ---------------------------------------------------------------------------
// TMA variant for fp32 points at TF32 precision (the routing path).
//
// One thread streams tiles with tiled TMA loads (128-byte swizzle, zero fill
// past the last point / centroid / feature), so the loads cost a handful of
// instructions per tile instead of one cp.async per 16 bytes.  For d <= 64 an
// item is 256 points (two 128-row M tiles): each centroid tile feeds two MMAs,
// halving centroid traffic and the per-tile barrier round trips; TMEM holds
// 2 buffers x 2 M tiles x 128 columns (all 512 columns).
//
// Argmin as one integer minimum per column.  Per problem b the host-side
// prologue (point_sqmax_kernel, centroid_bias_kernel) provides a bias
// B >= max|x|^2 and the biased norms |c|^2 + B, so that per column
//     s = (|c|^2 + B) - 2 x.c = dist + (B - |x|^2)
// is one FFMA, strictly positive and within 2^12 of base = B / 256.  For
// positive floats the bit pattern orders like the value, so
//     key = 32 * (bits(s) - bits(base)) + j      (j = column within 32)
// is exact (fp32 order, ties to the lower column) and fits 32 bits: one IMAD
// and one unsigned min per column.  Columns with dist <= 0 (s <= B - |x|^2)
// are clamped to distance 0 as the reference does, lowest index first, on a
// warp-uniform slow path that only runs when such a column exists.
//
// |x|^2 is computed by the argmin threads from the staged point tile.
//
// Folded bias (FOLD, when round_up(d, 8) + 8 <= DP): the FFMA and the |c|^2
// shared-memory reads leave the epilogue.  The centroid operand is the
// augmented row [-2c | 0.. | hi, lo, 0 x 6] (centroid_bias_kernel writes it,
// feature dh = round_up(d, 8) holds hi = tf32(|c|^2 + B), dh + 1 the
// remainder lo), and one extra K step multiplies those 8 features by a
// constant all-ones A tile in shared memory, so the accumulator is s itself.
// Scaling by -2 is exact; hi + lo carry |c|^2 + B to ~2^-21 relative, far
// inside the TF32 error of the dot product.
//
// Warps 0-7: argmin (thread = point when MT == 2; two threads per point, one
// per 64-column half, when MT == 1), warp 8: MMA issuer, warp 9: TMA producer.
constexpr int kTmaAsgThreads = 320;

// Features before the folded-bias columns, and the augmented row length.
inline int fold_head(int d) { return (d + 7) / 8 * 8; }
__device__ __forceinline__ int fold_head_dev(int d) { return (d + 7) / 8 * 8; }
inline int fold_row(int d) { return fold_head(d) + 8; }
template <int DP>
inline bool assign_folds(int d) { return fold_row(d) <= DP; }

// BF: bf16 points and bf16 centroid operands, kind::f16 MMAs (the standalone
// flash_kmeans path, whose centroids are rounded to the input dtype); else
// fp32 operands at TF32.  Both use 32-byte MMA K steps over 128-byte
// swizzled row blocks (8 tf32 or 16 bf16 features per step).
template <int DP, bool FOLD = false, bool BF = false>
struct TmaAsg {
  static constexpr int kElem = BF ? 2 : 4;
  static constexpr int kRowBytes = DP * kElem;
  static constexpr int kMT = kRowBytes <= 256 ? 2 : 1;  // 128-point M tiles per item
  static constexpr int kBlocks = kRowBytes / 128;       // 128-byte column blocks per row
  static constexpr int kBlockElems = 128 / kElem;       // features per 128-byte block
  static constexpr int kTileBytes = 128 * kRowBytes;    // one 128-row tile of points or centroids
  static constexpr int kXBytes = kMT * kTileBytes;
  static constexpr int kOnesBytes = FOLD ? 128 * 128 : 0;  // all-ones A tile (128 rows x 128 bytes)
  static constexpr int kBudget = 216 * 1024 - kOnesBytes;
  static constexpr int kNX = (1024 + 2 * kXBytes + 2 * kTileBytes <= kBudget) ? 2 : 1;
  static constexpr int kNC = (1024 + kNX * kXBytes + 4 * kTileBytes <= kBudget)   ? 4
                             : (1024 + kNX * kXBytes + 3 * kTileBytes <= kBudget) ? 3
                                                                                  : 2;
  static constexpr int kTotal = 1024 + kNX * kXBytes + kNC * kTileBytes + kOnesBytes;
  static constexpr int kCG = 2 / kMT;  // argmin threads per point
  static constexpr int kNQ = 8;        // |c|^2 ring slots
};

// max over the points of problem b of |x|^2 into xmax[b] (zeroed by the caller).
template <typename T>
__global__ void point_sqmax_kernel(const T* __restrict__ x, int64_t n, int d, float* __restrict__ xmax) {
  __shared__ float s_max[8];
  const int64_t b = blockIdx.y;
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float s = 0.f;
  if (p < n) {
    const T* r = x + (b * n + p) * d;
    for (int e = 0; e < d / 4; ++e) {
      const float4 v = load4<T>(r + 4 * e);
      s = fmaf(v.x, v.x, s);
      s = fmaf(v.y, v.y, s);
      s = fmaf(v.z, v.z, s);
      s = fmaf(v.w, v.w, s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) s = fmaxf(s, s_max[w]);
    atomicMax(reinterpret_cast<int*>(xmax + b), __float_as_int(s));  // non-negative floats order as ints
  }
}

// Per problem b: csqb[b][j] = |c_j|^2 + B for j < k (0 in the padding up to
// kpad = 128 * centroid tiles) and bias[b] = (B, base) with
//   B = max|x|^2 * (1 + 2^-7) + max|c|^2 / 4,   base = B / 256.
// Then s = |c|^2 + B - 2 x.c lies in (2^-7 B - e, 10 B] for every point of b
// (e = TF32 error of 2 x.c, at most 2^-9 B), i.e. above base and below
// 2^12 base.
//
// Grid (centroid blocks of 128, bh); thread = centroid.  Each block folds its
// maximum into cmax[b]; the last block of a problem (ticket counter) adds B to
// the whole row and resets cmax[b] and the counter to 0 for the next call.
// cmax and count must be zero before the first call.
//
// With caug (folded bias), row i of caug[b] ([k][fold_row(d)]) becomes
// [-2c_i | 0 | hi_i, lo_i, 0 x 6], hi_i = tf32(|c_i|^2 + B) (low 13 bits
// cleared) and lo_i = |c_i|^2 + B - hi_i; the last block writes hi and lo.
//
// With cbf (the bf16 path), the centroids are rounded to bf16 into cbf[b][k][d]
// and |c|^2 is taken of the rounded values (the MMA operand itself).
__global__ void __launch_bounds__(128) centroid_bias_kernel(const float* __restrict__ c, int k, int d, int kpad,
                                                            const float* __restrict__ xmax, float* __restrict__ csqb,
                                                            float* __restrict__ bias, float* __restrict__ cmax,
                                                            unsigned* __restrict__ count, const int* __restrict__ done,
                                                            float* __restrict__ caug, __nv_bfloat16* __restrict__ cbf) {
  if (done && *done) return;
  __shared__ float s_max[4];
  __shared__ bool s_last;
  const int64_t b = blockIdx.y;
  const int i = blockIdx.x * 128 + threadIdx.x;
  float* out = csqb + b * kpad;
  float s = 0.f;
  if (i < k) {
    const float4* r = reinterpret_cast<const float4*>(c + (b * k + i) * d);
    for (int e = 0; e < d / 4; ++e) {
      float4 v = r[e];
      if (cbf) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        v = make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&lo);
        u.y = *reinterpret_cast<const uint32_t*>(&hi);
        reinterpret_cast<uint2*>(cbf + (b * k + i) * d)[e] = u;
      }
      s = fmaf(v.x, v.x, s);
      s = fmaf(v.y, v.y, s);
      s = fmaf(v.z, v.z, s);
      s = fmaf(v.w, v.w, s);
    }
    out[i] = s;
    if (caug) {
      const int dh = fold_head_dev(d);
      float4* w = reinterpret_cast<float4*>(caug + (b * k + i) * (dh + 8));
      for (int e = 0; e < d / 4; ++e) {
        const float4 v = r[e];
        w[e] = make_float4(-2.f * v.x, -2.f * v.y, -2.f * v.z, -2.f * v.w);
      }
      for (int e = d / 4; e < dh / 4; ++e) w[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float m = s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    m = fmaxf(fmaxf(s_max[0], s_max[1]), fmaxf(s_max[2], s_max[3]));
    atomicMax(reinterpret_cast<int*>(cmax + b), __float_as_int(m));
    __threadfence();
    s_last = atomicAdd(count + b, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float cm = __int_as_float(atomicAdd(reinterpret_cast<int*>(cmax + b), 0));
  const float B = fmaf(__ldcg(xmax + b), 1.0078125f, 0.25f * cm) + 1e-30f;
  for (int j = threadIdx.x; j < kpad; j += blockDim.x) {
    const float v = j < k ? __ldcg(out + j) + B : 0.f;
    out[j] = v;
    if (caug && j < k) {
      const int dh = fold_head_dev(d);
      const float hi = __uint_as_float(__float_as_uint(v) & 0xffffe000u);
      float4* w = reinterpret_cast<float4*>(caug + (b * k + j) * (dh + 8) + dh);
      w[0] = make_float4(hi, v - hi, 0.f, 0.f);
      w[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (threadIdx.x == 0) {
    bias[2 * b] = B;
    bias[2 * b + 1] = B * 0.00390625f;
    cmax[b] = 0.f;
    count[b] = 0u;
  }
}

template <int DP, bool FOLD, bool BF>
__global__ void __launch_bounds__(kTmaAsgThreads, 1)
assign_tma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap cmap, int64_t n,
                  int d, int k, int64_t items, const float* __restrict__ csqb, const float* __restrict__ bias,
                  int32_t* __restrict__ labels, const int* __restrict__ done, int* __restrict__ err) {
  using L = TmaAsg<DP, FOLD, BF>;
  static_assert(!(FOLD && BF), "the folded bias is a TF32-path option");
  constexpr int MT = L::kMT, NX = L::kNX, NC = L::kNC, NQ = L::kNQ, CG = L::kCG;
  constexpr int kBlocksPerThread = 4 / CG;  // 32-column TMEM blocks scanned per tile
  if (done && *done) return;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_x_full[NX], bar_x_empty[NX], bar_x_read[NX];
  __shared__ uint64_t bar_c_full[NC], bar_c_empty[NC], bar_q_full[NQ], bar_q_read[NQ];
  __shared__ uint64_t bar_d_full[2], bar_d_free[2], bar_mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ __align__(128) float s_csq[NQ][kAsgN];
  __shared__ float s_best[kAsgM];
  __shared__ int s_best_idx[kAsgM];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sx0 = tc::smem_addr(smem);
  const uint32_t sc0 = sx0 + NX * L::kXBytes;
  const uint32_t sones = sc0 + NC * L::kTileBytes;  // FOLD: all-ones A tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if constexpr (FOLD) {
    float4* o = reinterpret_cast<float4*>(smem + NX * L::kXBytes + NC * L::kTileBytes);
    for (int i = tid; i < L::kOnesBytes / 16; i += kTmaAsgThreads) o[i] = make_float4(1.f, 1.f, 1.f, 1.f);
    tc::fence_proxy_async_smem();  // the MMAs read the tile through the async proxy
  }
  const int ctiles = (k + kAsgN - 1) / kAsgN;
  const int64_t ptiles = (n + MT * kAsgM - 1) / (MT * kAsgM);

  if (tid == 0) {
    for (int i = 0; i < NX; ++i) {
      tc::mbar_init(&bar_x_full[i], 1);
      tc::mbar_init(&bar_x_empty[i], 1);
      tc::mbar_init(&bar_x_read[i], kAsgEpilogue);
    }
    for (int i = 0; i < NC; ++i) {
      tc::mbar_init(&bar_c_full[i], 1);
      tc::mbar_init(&bar_c_empty[i], 1);
    }
    for (int i = 0; i < NQ; ++i) {
      tc::mbar_init(&bar_q_full[i], 1);
      tc::mbar_init(&bar_q_read[i], kAsgEpilogue);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_d_full[i], 1);
      tc::mbar_init(&bar_d_free[i], kAsgEpilogue);
    }
    tc::mbar_init(&bar_mma_done, 1);
    tc::mbar_fence_init();
  }
  if (warp == 9 && lane == 0) {
    tc::prefetch_tmap(&xmap);
    tc::prefetch_tmap(&cmap);
  }
  if (warp == 8) tc::tmem_alloc<256 * MT>(&s_tmem);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 9) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      int64_t nc = 0;  // centroid tiles issued
      int nx = 0;      // point items issued
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < items; it += gridDim.x) {
        const int b = (int)(it / ptiles);
        const int64_t p0 = (it % ptiles) * (MT * kAsgM);
        const int xb = nx % NX;
        if (nx >= NX) {  // the GEMMs and the |x|^2 reads of item nx-NX are done with this buffer
          const uint32_t par = ((nx / NX) - 1) & 1;
          if (!(ok = tc::mbar_wait(&bar_x_empty[xb], par, err, 31) && tc::mbar_wait(&bar_x_read[xb], par, err, 31)))
            break;
        }
        const uint32_t xbase = sx0 + xb * L::kXBytes;
        const int mts = p0 + kAsgM < n ? MT : 1;  // an M tile wholly past the last point is not loaded
        tc::mbar_expect_tx(&bar_x_full[xb], (uint32_t)(mts * L::kTileBytes));
        for (int mt = 0; mt < mts; ++mt)
#pragma unroll
          for (int j = 0; j < L::kBlocks; ++j)
            tc::tma_load_3d(xbase + mt * L::kTileBytes + j * (kAsgM * 128), &xmap, L::kBlockElems * j,
                            (int)(p0 + mt * kAsgM), b, &bar_x_full[xb]);
        ++nx;
        for (int t = 0; t < ctiles; ++t) {
          const int st = (int)(nc % NC), q = (int)(nc % NQ);
          if (nc >= NC && !(ok = tc::mbar_wait(&bar_c_empty[st], (uint32_t)(((nc / NC) - 1) & 1), err, 32))) break;
          if (!FOLD && nc >= NQ && !(ok = tc::mbar_wait(&bar_q_read[q], (uint32_t)(((nc / NQ) - 1) & 1), err, 32)))
            break;
          const uint32_t cbase = sc0 + st * L::kTileBytes;
          tc::mbar_expect_tx(&bar_c_full[st], (uint32_t)L::kTileBytes);
#pragma unroll
          for (int j = 0; j < L::kBlocks; ++j)
            tc::tma_load_3d(cbase + j * (kAsgN * 128), &cmap, L::kBlockElems * j, t * kAsgN, b, &bar_c_full[st]);
          if constexpr (!FOLD) {
            tc::mbar_expect_tx(&bar_q_full[q], kAsgN * 4);
            tc::bulk_load(tc::smem_addr(&s_csq[q][0]), csqb + ((int64_t)b * ctiles + t) * kAsgN, kAsgN * 4,
                          &bar_q_full[q]);
          }
          ++nc;
        }
      }
      // Let every copy issued here land before the CTA exits (matters only
      // when a wait gave up and the consumers stopped early).
      for (int u = nx > NX ? nx - NX : 0; u < nx; ++u) tc::mbar_drain(&bar_x_full[u % NX], (u / NX) & 1);
      for (int64_t u = nc > NC ? nc - NC : 0; u < nc; ++u)
        tc::mbar_drain(&bar_c_full[u % NC], (uint32_t)((u / NC) & 1));
      if constexpr (!FOLD)
        for (int64_t u = nc > NQ ? nc - NQ : 0; u < nc; ++u)
          tc::mbar_drain(&bar_q_full[u % NQ], (uint32_t)((u / NQ) & 1));
    }
  } else if (warp == 8) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const int ksteps = BF ? (d + 15) / 16 : (d + 7) / 8;  // 32-byte K steps
      // FOLD: the K step over features [dh, dh + 8) of the centroid row (hi, lo, zeros) against ones.
      const uint32_t kbf = (uint32_t)ksteps * 32;
      const uint32_t offf = (kbf >> 7) * (kAsgN * 128) + (kbf & 127);
      int64_t gt = 0;
      int il = 0;
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < items; it += gridDim.x, ++il) {
        const int xb = il % NX;
        if (!(ok = tc::mbar_wait(&bar_x_full[xb], (il / NX) & 1, err, 33))) break;
        const uint32_t xbase = sx0 + xb * L::kXBytes;
        for (int t = 0; t < ctiles; ++t, ++gt) {
          const int st = (int)(gt % NC);
          const int db = (int)(gt & 1);
          if (!(ok = tc::mbar_wait(&bar_c_full[st], (uint32_t)((gt / NC) & 1), err, 33))) break;
          if (gt >= 2 && !(ok = tc::mbar_wait(&bar_d_free[db], (uint32_t)(((gt >> 1) - 1) & 1), err, 33))) break;
          tc::tc_fence_after();
          const uint32_t cbase = sc0 + st * L::kTileBytes;
          // The last centroid tile is only as wide as its centroids (rounded up
          // to 16): its MMAs read fewer B rows; columns past it are masked.
          const int nt = t == ctiles - 1 ? min(kAsgN, (k - t * kAsgN + 15) & ~15) : kAsgN;
          const uint32_t idesc_t = tc::idesc_tf32_f32(128, nt), idesc_bf_t = tc::idesc_bf16_f32(128, nt, 0);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint32_t dt = tmem + (uint32_t)(db * MT + mt) * 128;
            if constexpr (FOLD)
              tc::mma_tf32(dt, tc::sw128_desc(sones, 16, 1024), tc::sw128_desc(cbase + offf, 16, 1024), idesc_t,
                           false);
            // 8 tf32 or 16 bf16 (32 bytes) per MMA K step; steps wholly inside
            // the zero padding past d are skipped.
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint32_t kb = kk * 32;
              const uint32_t off = (kb >> 7) * (kAsgM * 128) + (kb & 127);
              if constexpr (BF)
                tc::mma_f16(dt, tc::sw128_desc(xbase + mt * L::kTileBytes + off, 16, 1024),
                            tc::sw128_desc(cbase + off, 16, 1024), idesc_bf_t, kk > 0);
              else
                tc::mma_tf32(dt, tc::sw128_desc(xbase + mt * L::kTileBytes + off, 16, 1024),
                             tc::sw128_desc(cbase + off, 16, 1024), idesc_t, FOLD || kk > 0);
            }
          }
          tc::mma_commit(&bar_d_full[db]);
          tc::mma_commit(&bar_c_empty[st]);
          if (t == ctiles - 1) tc::mma_commit(&bar_x_empty[xb]);
        }
      }
      tc::mma_commit(&bar_mma_done);  // every MMA issued above has finished before TMEM is freed
      tc::mbar_drain(&bar_mma_done, 0);
    }
  } else {
    // ---------------------------------------------------------- argmin epilogue
    const int row = tid & 127;  // TMEM lane = point row within its M tile
    const int sub = tid >> 7;
    const int mt = MT == 2 ? sub : 0;
    const int cg = MT == 2 ? 0 : sub;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    int64_t gt = 0;
    int il = 0;
    bool ok = true;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x, ++il) {
      const int64_t b = it / ptiles;
      const int64_t p = (it % ptiles) * (MT * kAsgM) + mt * kAsgM + row;
      const int xb = il % NX;
      ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_x_full[xb], (il / NX) & 1, err, 34));
      // |x|^2 of this point from the staged tile (zero padding adds nothing).
      float xsq = 0.f;
      if (ok) {
        const uint8_t* xt = smem + xb * L::kXBytes + mt * L::kTileBytes;
#pragma unroll
        for (int ch = 0; ch < L::kRowBytes / 16; ++ch) {
          if constexpr (BF) {
            const uint4 u = *reinterpret_cast<const uint4*>(xt + tc::sw128_off(row, ch, kAsgM));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
              xsq = fmaf(__low2float(h), __low2float(h), xsq);
              xsq = fmaf(__high2float(h), __high2float(h), xsq);
            }
          } else {
            const float4 v = *reinterpret_cast<const float4*>(xt + tc::sw128_off(row, ch, kAsgM));
            xsq = fmaf(v.x, v.x, xsq);
            xsq = fmaf(v.y, v.y, xsq);
            xsq = fmaf(v.z, v.z, xsq);
            xsq = fmaf(v.w, v.w, xsq);
          }
        }
      }
      tc::mbar_arrive(&bar_x_read[xb]);
      const float B = __ldg(bias + 2 * b), base = __ldg(bias + 2 * b + 1);
      // key = 32 * (bits(s) - bits(base)) + j, computed mod 2^32 as bits(s) * 32 + kj[j].
      const uint32_t koff = 0u - 32u * __float_as_uint(base);
      uint32_t kj[32];  // per-column key offsets, kept in registers for the item
#pragma unroll
      for (int j = 0; j < 32; ++j) kj[j] = koff + j;
      // Columns with s <= thr have dist <= 0 (clamped to 0 by the reference).
      const uint32_t thrq = __float_as_uint(B - xsq) - __float_as_uint(base);
      uint32_t best_q = 0xffffffffu;  // bits(s) - bits(base) of the best column so far
      int best_idx = 0;
      for (int t = 0; t < ctiles; ++t, ++gt) {
        const int db = (int)(gt & 1);
        const int q = (int)(gt % NQ);
        ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_d_full[db], (uint32_t)((gt >> 1) & 1), err, 34));
        if constexpr (!FOLD)
          ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_q_full[q], (uint32_t)((gt / NQ) & 1), err, 34));
        tc::tc_fence_after();
        const int k0 = t * kAsgN;
        if (ok) {
          const bool full = k0 + kAsgN <= k;  // only the last centroid tile is partial
          const uint32_t tbase = tmem + lane_base + (uint32_t)(db * MT + mt) * 128 + cg * kBlocksPerThread * 32;
          // Double-buffered TMEM reads: block i+1 is in flight while block i is scanned.
          float accv[2][32];
          tc::tmem_ld32_async(tbase, accv[0]);
          tc::tmem_wait_ld();
          tc::reg_fence32(accv[0]);
#pragma unroll
          for (int i = 0; i < kBlocksPerThread; ++i) {
            float* acc = accv[i & 1];
            if (i + 1 < kBlocksPerThread) tc::tmem_ld32_async(tbase + (i + 1) * 32, accv[(i + 1) & 1]);
            const int cb = cg * kBlocksPerThread + i;
            const float* cq = &s_csq[q][cb * 32];
            const int lim = full ? 32 : k - (k0 + cb * 32);  // valid columns in this block (may be <= 0)
            // Four independent minimum chains (columns j mod 4); keys are
            // distinct per column, so the merged minimum is the same.
            uint32_t m0 = 0xffffffffu, m1 = 0xffffffffu, m2 = 0xffffffffu, m3 = 0xffffffffu;
            if (FOLD && full) {  // s is the accumulator itself
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                m0 = min(m0, __float_as_uint(acc[j]) * 32u + kj[j]);
                m1 = min(m1, __float_as_uint(acc[j + 1]) * 32u + kj[j + 1]);
                m2 = min(m2, __float_as_uint(acc[j + 2]) * 32u + kj[j + 2]);
                m3 = min(m3, __float_as_uint(acc[j + 3]) * 32u + kj[j + 3]);
              }
            } else if (FOLD) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const uint32_t key = __float_as_uint(acc[j]) * 32u + kj[j];
                m0 = j < lim ? min(m0, key) : m0;
              }
            } else if (full) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 c4 = *reinterpret_cast<const float4*>(cq + j);
                m0 = min(m0, __float_as_uint(fmaf(-2.f, acc[j], c4.x)) * 32u + kj[j]);
                m1 = min(m1, __float_as_uint(fmaf(-2.f, acc[j + 1], c4.y)) * 32u + kj[j + 1]);
                m2 = min(m2, __float_as_uint(fmaf(-2.f, acc[j + 2], c4.z)) * 32u + kj[j + 2]);
                m3 = min(m3, __float_as_uint(fmaf(-2.f, acc[j + 3], c4.w)) * 32u + kj[j + 3]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const uint32_t key = __float_as_uint(fmaf(-2.f, acc[j], cq[j])) * 32u + kj[j];
                m0 = j < lim ? min(m0, key) : m0;
              }
            }
            const uint32_t kmin = min(min(m0, m1), min(m2, m3));
            uint32_t qv = kmin >> 5;
            int jj = (int)(kmin & 31u);
            if (__any_sync(0xffffffffu, qv <= thrq && lim > 0)) {
              // Rare: a column at distance <= 0.  All such columns tie at 0;
              // the lowest one wins.
              if (qv <= thrq && lim > 0) {
                int first = 31;
#pragma unroll
                for (int j = 31; j >= 0; --j) {
                  const uint32_t sq = __float_as_uint(FOLD ? acc[j] : fmaf(-2.f, acc[j], cq[j])) -
                                      __float_as_uint(base);
                  if (j < lim && sq <= thrq) first = j;
                }
                jj = first;
                qv = thrq;
              }
            }
            if (lim > 0 && qv < best_q) {  // strict: an earlier column keeps a tie
              best_q = qv;
              best_idx = k0 + cb * 32 + jj;
            }
            if (i + 1 < kBlocksPerThread) {
              tc::tmem_wait_ld();
              tc::reg_fence32(accv[(i + 1) & 1]);
            }
          }
        }
        tc::tc_fence_before();
        tc::mbar_arrive(&bar_d_free[db]);
        if constexpr (!FOLD) tc::mbar_arrive(&bar_q_read[q]);
      }
      if constexpr (CG == 2) {
        // Merge the two column halves of each point (equal values: lower index).
        if (cg == 1) { s_best[row] = __uint_as_float(best_q); s_best_idx[row] = best_idx; }
        tc::named_bar(1, kAsgEpilogue);
        if (cg == 0) {
          const uint32_t ob = __float_as_uint(s_best[row]);
          const int oi = s_best_idx[row];
          if (ob < best_q || (ob == best_q && oi < best_idx)) best_idx = oi;
          if (p < n) labels[b * n + p] = best_idx;
        }
        tc::named_bar(1, kAsgEpilogue);
      } else {
        if (p < n) labels[b * n + p] = best_idx;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc<256 * MT>(tmem);
  }
}

// 3-D map over [bh][rows][d] rows: box of one 128-byte block (32 fp32 or 64 bf16
// features) x 128 rows x 1, 128-byte swizzle.
inline int encode_row_map(CUtensorMap* m, const void* base, bool bf16, int d, int64_t rows, int64_t bh,
                          const char* what) {
  return bf16 ? encode_map_3d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, d, rows, bh, 64, kAsgM, what)
              : encode_map_3d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, d, rows, bh, 32, kAsgM, what);
}

template <int DP, bool FOLD, bool BF = false>
static int launch_assign_tma_as(const void* x, int64_t bh, int64_t n, int d, int k, const void* c,
                                const float* csqb, const float* bias, int32_t* labels, const int* done, int* err,
                                cudaStream_t st) {
  using L = TmaAsg<DP, FOLD, BF>;
  CUtensorMap xmap, cmap;
  int s = encode_row_map(&xmap, x, BF, d, n, bh, "points");
  // FOLD: c is the augmented centroid array [bh][k][fold_row(d)]; BF: the bf16 centroid copy.
  if (!s) s = encode_row_map(&cmap, c, BF, FOLD ? fold_row(d) : d, k, bh, "centroids");
  if (s) return s;
  auto kern = assign_tma_kernel<DP, FOLD, BF>;
  const cudaError_t ae = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (ae != cudaSuccess)
    return fail(SPR_ERR_LAUNCH, "k-means assign: shared-memory opt-in (%d B): %s", L::kTotal, cudaGetErrorString(ae));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = bh * ((n + L::kMT * kAsgM - 1) / (L::kMT * kAsgM));
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);  // persistent: one CTA per SM
  kern<<<grid, kTmaAsgThreads, L::kTotal, st>>>(xmap, cmap, n, d, k, items, csqb, bias, labels, done, err);
  return check_launch("k-means assign (tcgen05, TMA)");
}

template <int DP>
static int launch_assign_tma(const float* x, int64_t bh, int64_t n, int d, int k, const float* c, const float* caug,
                             const float* csqb, const float* bias, int32_t* labels, const int* done, int* err,
                             cudaStream_t st) {
  if (caug && assign_folds<DP>(d))
    return launch_assign_tma_as<DP, true>(x, bh, n, d, k, caug, csqb, bias, labels, done, err, st);
  return launch_assign_tma_as<DP, false>(x, bh, n, d, k, c, csqb, bias, labels, done, err, st);
}

// Whether the TMA path folds the bias into the MMA for width d (the augmented
// centroid rows are then needed), and their float count.  Only where the 8
// extra features fit the tile width d already uses: widening the tile (d = 64
// -> 96, one M tile per item) costs more than the fold saves.
inline int assign_dp(int d) { return d <= 32 ? 32 : d <= 64 ? 64 : d <= 96 ? 96 : 128; }
inline bool assign_fold_for(int d) { return fold_row(d) <= assign_dp(d); }
inline size_t centroid_aug_count(int64_t bh, int d, int k) {
  return assign_fold_for(d) ? (size_t)bh * (size_t)k * (size_t)fold_row(d) : 0;
}

// Padded |c|^2 entries needed by the TMA path: [bh][128 * centroid tiles].
inline size_t centroid_sq_pad_count(int64_t bh, int k) { return (size_t)bh * (size_t)((k + kAsgN - 1) / kAsgN) * kAsgN; }

// The TMA path serves fp32 points at TF32 precision, and bf16 points when the
// caller keeps its centroids in bf16 (cbf_ok: the standalone flash_kmeans
// path rounds every update to the input dtype, so bf16 MMAs see the exact
// centroids); other cases use the register-staged kernel above.
inline bool assign_uses_tma(int x_dtype, int precision, bool cbf_ok = false) {
  return precision == SPR_KMEANS_TF32 && (x_dtype == SPR_F32 || (x_dtype == SPR_BF16 && cbf_ok));
}

// Per-run point statistics (call once per k-means run: x does not change):
// |x|^2 per point for the register path, max |x|^2 per problem for the TMA
// path (which computes |x|^2 itself).
inline int launch_point_sq(const void* x, int x_dtype, int precision, int64_t bh, int64_t n, int d, float* xsq,
                           float* xmax, cudaStream_t st, bool cbf_ok = false) {
  if (assign_uses_tma(x_dtype, precision, cbf_ok)) {
    // xmax and the bias scratch that follows it (4 * bh words) start at 0.
    cudaMemsetAsync(xmax, 0, (size_t)bh * 5 * sizeof(float), st);
    const dim3 grid((unsigned)((n + 255) / 256), (unsigned)bh);
    if (x_dtype == SPR_BF16)
      point_sqmax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, n, d, xmax);
    else
      point_sqmax_kernel<float><<<grid, 256, 0, st>>>((const float*)x, n, d, xmax);
    return check_launch("point norm maxima");
  }
  if (x_dtype != SPR_F32) return SPR_OK;  // other dtypes compute |x|^2 inside the assignment kernel
  const int64_t rows = bh * n;
  row_sq_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>((const float*)x, rows, d, xsq, nullptr);
  return check_launch("point norms");
}

// Centroid norms of the current centroids, then the assignment GEMM (point
// statistics from launch_point_sq).  csq holds centroid_sq_pad_count floats,
// bias 4 * bh: (B, base) pairs, then the centroid-norm maxima and counters of
// centroid_bias_kernel (zeroed once per run by launch_point_sq).
// caug: augmented centroid rows for the folded-bias TMA path
// (centroid_aug_count floats; nullptr when that count is 0).
// cbf: bf16 centroid scratch [bh][k][d] for the bf16 TMA path (cbf_ok).
inline int launch_assign(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k, const float* c,
                         const float* xsq, const float* xmax, float* csq, float* bias, float* caug, int precision,
                         int32_t* labels, const int* done, int* err, cudaStream_t st, __nv_bfloat16* cbf = nullptr) {
  const bool cbf_ok = cbf != nullptr;
  if (assign_uses_tma(x_dtype, precision, cbf_ok)) {
    const int kpad = (k + kAsgN - 1) / kAsgN * kAsgN;
    const bool bf = x_dtype == SPR_BF16;
    if (!assign_fold_for(d) || bf) caug = nullptr;
    centroid_bias_kernel<<<dim3((unsigned)(kpad / kAsgN), (unsigned)bh), 128, 0, st>>>(
        c, k, d, kpad, xmax, csq, bias, bias + 2 * bh, reinterpret_cast<unsigned*>(bias + 3 * bh), done, caug,
        bf ? cbf : nullptr);
    int s = check_launch("centroid norms");
    if (s) return s;
    if (bf) {
      if (d <= 64) return launch_assign_tma_as<64, false, true>(x, bh, n, d, k, cbf, csq, bias, labels, done, err, st);
      return launch_assign_tma_as<128, false, true>(x, bh, n, d, k, cbf, csq, bias, labels, done, err, st);
    }
    const float* xf = (const float*)x;
    if (d <= 32) return launch_assign_tma<32>(xf, bh, n, d, k, c, caug, csq, bias, labels, done, err, st);
    if (d <= 64) return launch_assign_tma<64>(xf, bh, n, d, k, c, caug, csq, bias, labels, done, err, st);
    if (d <= 96) return launch_assign_tma<96>(xf, bh, n, d, k, c, caug, csq, bias, labels, done, err, st);
    return launch_assign_tma<128>(xf, bh, n, d, k, c, caug, csq, bias, labels, done, err, st);
  }
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
