// Attention-mass routing scores on the tensor cores:
//   scores[b, c, j] = log sum_{t in key cluster j} exp(q_c . k_t / sqrt(D))
// (-inf for an empty cluster), D = 128, query centroids q_c fp32, keys bf16
// sorted by cluster (k_offsets gives each cluster's token range).
//
// The dots are a [Cq x D] x [D x N] GEMM per problem.  Keys are exact in
// bf16; each fp32 centroid is split into three bf16 parts
// (q = q1 + q2 + q3, |q - q1 - q2 - q3| <= 2^-24 |q|), so three kind::f16
// MMAs with fp32 accumulation reproduce the fp32 dot products.
//
// Work items: (problem b, 128-centroid M tile, chunk of kChunk key clusters).
// Each CTA takes a contiguous range of items, so consecutive items share the
// staged centroid tile (re-staged only when (b, M tile) changes).  Per item the
// chunk's tokens stream through in 128-token tiles: one thread issues tiled
// TMA loads of the key rows, one thread issues the MMAs into a double-buffered
// TMEM accumulator, and four warps (thread = centroid = TMEM lane) walk the
// columns with an online log-sum-exp per cluster.  Cluster boundaries are the
// same for every row, so the walk is warp-uniform.
#include "tc_common.cuh"
#include "tmap.cuh"

namespace spr {

namespace {

constexpr int kSD = 128;            // head dim
constexpr int kSM = 128;            // centroids per M tile
constexpr int kSN = 128;            // tokens per tile
constexpr int kChunk = 16;          // key clusters per work item
constexpr int kSplits = 3;          // bf16 parts of each centroid
constexpr int kSTile = kSM * kSD * 2;  // one bf16 128 x 128 tile (32 KB)
constexpr int kSStages = 3;            // key-tile ring
constexpr int kSThreads = 192;         // warps 0-3 epilogue, 4 MMA, 5 TMA
constexpr int kSEpi = 128;
constexpr int kSSmem = 1024 + kSplits * kSTile + kSStages * kSTile;
constexpr uint32_t kIdescS = tc::idesc_bf16_f32(128, 128, 0);

struct ScoreItems {
  int mtiles, chunks;
  int64_t items;
};

__host__ __device__ inline ScoreItems score_items(int64_t bh, int cq, int ck) {
  ScoreItems s;
  s.mtiles = (cq + kSM - 1) / kSM;
  s.chunks = (ck + kChunk - 1) / kChunk;
  s.items = bh * s.mtiles * s.chunks;
  return s;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Stage centroid row r of M tile mt as three bf16 parts (K-major, 128-byte
// swizzle: two 64-column blocks per part).  Rows past cq are zero.
__device__ void stage_centroid_row(const float* __restrict__ qrow, bool valid, uint32_t a0, int r) {
#pragma unroll 1
  for (int ch = 0; ch < kSD / 8; ++ch) {  // 8 values = one 16-byte chunk per part
    float x[8];
    if (valid) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(qrow) + 2 * ch);
      const float4 w = __ldg(reinterpret_cast<const float4*>(qrow) + 2 * ch + 1);
      x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w; x[4] = w.x; x[5] = w.y; x[6] = w.z; x[7] = w.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = 0.f;
    }
    uint32_t p[kSplits][4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float r0 = x[e], r1 = x[e + 1];
#pragma unroll
      for (int s = 0; s < kSplits; ++s) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(r0), h1 = __float2bfloat16_rn(r1);
        __nv_bfloat162 hh;
        hh.x = h0;
        hh.y = h1;
        p[s][e / 2] = *reinterpret_cast<const uint32_t*>(&hh);
        r0 -= __bfloat162float(h0);  // exact: the residual of a round-to-nearest split
        r1 -= __bfloat162float(h1);
      }
    }
    const uint32_t off = tc::sw128_off(r, ch, kSM);
#pragma unroll
    for (int s = 0; s < kSplits; ++s) st_shared_v4(a0 + s * kSTile + off, p[s][0], p[s][1], p[s][2], p[s][3]);
  }
}

__global__ void __launch_bounds__(kSThreads, 1)
scores_tc_kernel(const __grid_constant__ CUtensorMap kmap, const float* __restrict__ qc,
                 const int32_t* __restrict__ koff, int cq, int ck, int64_t n, int64_t items,
                 float* __restrict__ scores, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_a_full, bar_a_empty, bar_b_full[kSStages], bar_b_empty[kSStages], bar_d_full[2],
      bar_d_free[2], bar_mma_done;
  __shared__ uint32_t s_tmem;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = tc::smem_addr(smem);
  const uint32_t sb = sa + kSplits * kSTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScoreItems si = score_items(1, cq, ck);
  const int per_b = si.mtiles * si.chunks;
  // Contiguous item range of this CTA.
  const int64_t it0 = items * blockIdx.x / gridDim.x, it1 = items * (blockIdx.x + 1) / gridDim.x;

  if (tid == 0) {
    tc::mbar_init(&bar_a_full, kSEpi);
    tc::mbar_init(&bar_a_empty, 1);
    for (int i = 0; i < kSStages; ++i) {
      tc::mbar_init(&bar_b_full[i], 1);
      tc::mbar_init(&bar_b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bar_d_full[i], 1);
      tc::mbar_init(&bar_d_free[i], kSEpi);
    }
    tc::mbar_init(&bar_mma_done, 1);
    tc::mbar_fence_init();
  }
  if (warp == 5 && lane == 0) tc::prefetch_tmap(&kmap);
  if (warp == 4) tc::tmem_alloc<256>(&s_tmem);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;

  // Item decomposition shared by all roles.
  auto decode = [&](int64_t it, int64_t& b, int& mt, int& c0, int& c1, int32_t& t0, int32_t& t1) {
    b = it / per_b;
    const int r = (int)(it % per_b);
    mt = r / si.chunks;
    const int chunk = r % si.chunks;
    c0 = chunk * kChunk;
    c1 = min(ck, c0 + kChunk);
    t0 = __ldg(koff + b * (ck + 1) + c0);
    t1 = __ldg(koff + b * (ck + 1) + c1);
  };

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int64_t nt = 0;  // key tiles issued
      bool ok = true;
      for (int64_t it = it0; ok && it < it1; ++it) {
        int64_t b;
        int mt, c0, c1;
        int32_t t0, t1;
        decode(it, b, mt, c0, c1, t0, t1);
        for (int32_t tt = t0; tt < t1; tt += kSN, ++nt) {
          const int st = (int)(nt % kSStages);
          if (nt >= kSStages && !(ok = tc::mbar_wait(&bar_b_empty[st], (uint32_t)(((nt / kSStages) - 1) & 1), err, 41)))
            break;
          const uint32_t dst = sb + st * kSTile;
          tc::mbar_expect_tx(&bar_b_full[st], kSTile);
          tc::tma_load_3d(dst, &kmap, 0, tt, (int)b, &bar_b_full[st]);
          tc::tma_load_3d(dst + kSN * 128, &kmap, 64, tt, (int)b, &bar_b_full[st]);
        }
      }
      for (int64_t u = nt > kSStages ? nt - kSStages : 0; u < nt; ++u)
        tc::mbar_drain(&bar_b_full[u % kSStages], (uint32_t)((u / kSStages) & 1));
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int64_t nt = 0;
      int na = 0;            // centroid tiles staged so far
      int64_t akey = -1;     // (b, mt) of the staged tile
      bool ok = true;
      for (int64_t it = it0; ok && it < it1; ++it) {
        int64_t b;
        int mt, c0, c1;
        int32_t t0, t1;
        decode(it, b, mt, c0, c1, t0, t1);
        const int64_t key = b * si.mtiles + mt;
        if (key != akey) {
          if (na > 0) tc::mma_commit(&bar_a_empty);  // the previous tile is free once its MMAs finish
          if (!(ok = tc::mbar_wait(&bar_a_full, (uint32_t)(na & 1), err, 42))) break;
          akey = key;
          ++na;
        }
        for (int32_t tt = t0; tt < t1; tt += kSN, ++nt) {
          const int st = (int)(nt % kSStages);
          const int db = (int)(nt & 1);
          if (!(ok = tc::mbar_wait(&bar_b_full[st], (uint32_t)((nt / kSStages) & 1), err, 42))) break;
          if (nt >= 2 && !(ok = tc::mbar_wait(&bar_d_free[db], (uint32_t)(((nt >> 1) - 1) & 1), err, 42))) break;
          tc::tc_fence_after();
          const uint32_t bt = sb + st * kSTile;
          const uint32_t dt = tmem + db * kSN;
#pragma unroll
          for (int s = 0; s < kSplits; ++s) {
#pragma unroll
            for (int kk = 0; kk < kSD / 16; ++kk) {  // 16 bf16 = 32 bytes per K step
              const uint32_t kb = kk * 32;
              const uint32_t off = (kb >> 7) * (kSM * 128) + (kb & 127);
              tc::mma_f16(dt, tc::sw128_desc(sa + s * kSTile + off, 16, 1024), tc::sw128_desc(bt + off, 16, 1024),
                          kIdescS, (s | kk) != 0);
            }
          }
          tc::mma_commit(&bar_d_full[db]);
          tc::mma_commit(&bar_b_empty[st]);
        }
      }
      tc::mma_commit(&bar_mma_done);
      tc::mbar_drain(&bar_mma_done, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int r = tid;  // TMEM lane = centroid row within the M tile
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sc = 1.4426950408889634f * rsqrtf((float)kSD);  // log2(e) / sqrt(D)
    const float ln2 = 0.6931471805599453f;
    int64_t nt = 0;
    int na = 0;
    int64_t akey = -1;
    bool ok = true;
    for (int64_t it = it0; it < it1; ++it) {
      int64_t b;
      int mt, c0, c1;
      int32_t t0, t1;
      decode(it, b, mt, c0, c1, t0, t1);
      const int c = mt * kSM + r;
      const bool row_ok = c < cq;
      const int64_t key = b * si.mtiles + mt;
      if (key != akey) {
        if (na > 0) ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_a_empty, (uint32_t)((na - 1) & 1), err, 43));
        if (ok) stage_centroid_row(qc + (b * cq + (row_ok ? c : 0)) * (int64_t)kSD, row_ok, sa, r);
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&bar_a_full);
        akey = key;
        ++na;
      }
      float* out = scores + (b * cq + (row_ok ? c : 0)) * (int64_t)ck;
      // Cluster walk state: current cluster j ends at token jend.
      int j = c0;
      int32_t jend = t0;
      float m = -INFINITY, sum = 0.f;
      // Emit -inf for empty clusters until one with tokens starts.
      auto advance = [&]() {
        while (j < c1) {
          jend = __ldg(koff + b * (ck + 1) + j + 1);
          if (jend > __ldg(koff + b * (ck + 1) + j)) return;
          if (row_ok) out[j] = -INFINITY;
          ++j;
        }
      };
      advance();
      for (int32_t tt = t0; tt < t1; tt += kSN, ++nt) {
        const int db = (int)(nt & 1);
        ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_d_full[db], (uint32_t)((nt >> 1) & 1), err, 44));
        tc::tc_fence_after();
        if (ok) {
#pragma unroll 1
          for (int blk = 0; blk < kSN / 32; ++blk) {
            const int32_t bt = tt + blk * 32;
            if (bt >= t1) break;
            float acc[32];
            tc::tmem_ld32(tmem + lane_base + db * kSN + blk * 32, acc);
            const int32_t be = min(bt + 32, t1);
            int32_t pos = bt;
            while (pos < be) {  // runs of one cluster inside this 32-token block (warp-uniform)
              const int32_t re = min(jend, be);
              const int a = pos - bt, e = re - bt;
              float bm = -INFINITY;
              if (a == 0 && e == 32) {
#pragma unroll
                for (int q = 0; q < 32; ++q) bm = fmaxf(bm, acc[q]);
              } else {
#pragma unroll
                for (int q = 0; q < 32; ++q) bm = (q >= a && q < e) ? fmaxf(bm, acc[q]) : bm;
              }
              const float mn = fmaxf(m, bm * sc);
              float s0 = sum * tc::ex2(m - mn), s1 = 0.f;
              const float nm = -mn;
              if (a == 0 && e == 32) {
#pragma unroll
                for (int q = 0; q < 32; q += 2) {
                  s0 += tc::ex2(fmaf(acc[q], sc, nm));
                  s1 += tc::ex2(fmaf(acc[q + 1], sc, nm));
                }
              } else {
#pragma unroll
                for (int q = 0; q < 32; ++q)
                  if (q >= a && q < e) s0 += tc::ex2(fmaf(acc[q], sc, nm));
              }
              sum = s0 + s1;
              m = mn;
              pos = re;
              if (pos == jend) {  // cluster j complete
                if (row_ok) out[j] = (m + __log2f(sum)) * ln2;
                m = -INFINITY;
                sum = 0.f;
                ++j;
                advance();
              }
            }
          }
        }
        tc::tc_fence_before();
        tc::mbar_arrive(&bar_d_free[db]);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc::tc_fence_after();
    tc::tmem_dealloc<256>(tmem);
  }
}

}  // namespace

// Status word of the last scores launch: a bounded wait that gave up writes
// its code here (0 = ok).  Shared by all calls of this library instance.
__device__ int g_scores_err;

}  // namespace spr

using namespace spr;

extern "C" int spr_attention_mass_scores_status(int* out) {
  if (!out) return fail(SPR_ERR_ARG, "attention-mass scores status: null output");
  if (cudaMemcpyFromSymbol(out, g_scores_err, sizeof(int)) != cudaSuccess)
    return fail(SPR_ERR_LAUNCH, "attention-mass scores status: copy failed");
  return SPR_OK;
}

extern "C" int spr_attention_mass_scores(const float* q_centroids, const void* k_sorted, const int32_t* k_offsets,
                                         int64_t bh, int cq, int ck, int64_t n, int d, float* scores, void* stream) {
  if (d != kSD) return fail(SPR_ERR_SHAPE, "attention-mass scores require d=128, got %d", d);
  if (bh <= 0 || cq <= 0 || ck <= 0 || n <= 0 || bh > 65535 || n > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "attention-mass scores: bad shape bh=%lld cq=%d ck=%d n=%lld", (long long)bh, cq, ck,
                (long long)n);
  if (!aligned(q_centroids, 16) || !aligned(k_sorted, 16))
    return fail(SPR_ERR_ALIGN, "attention-mass scores: 16-byte alignment required");
  // Keys [bh][n][128] bf16: box 64 features (128 bytes) x 128 tokens.
  CUtensorMap kmap;
  int s = encode_map_3d(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k_sorted, kSD, n, bh, 64, kSN,
                        "attention-mass scores");
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream;
  cudaFuncSetAttribute(scores_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmem);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = score_items(bh, cq, ck).items;
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);
  int* err = nullptr;
  cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_scores_err);
  cudaMemsetAsync(err, 0, sizeof(int), st);
  scores_tc_kernel<<<grid, kSThreads, kSSmem, st>>>(kmap, q_centroids, k_offsets, cq, ck, n, items, scores, err);
  return check_launch("attention-mass scores (tcgen05)");
}
