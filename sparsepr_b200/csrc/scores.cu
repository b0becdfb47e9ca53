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

// Per-cluster and per-token terms of the SVG-EAR value-error score (VALUE
// mode of scores_tc_kernel).
// Per key cluster j (one warp): |vbar_j|^2, and for each token t of the
// cluster (sorted order) |v_t|^2 and v_t . vbar_j.
__global__ void value_terms_kernel(const __nv_bfloat16* __restrict__ vs, const float* __restrict__ vbar,
                                   const int32_t* __restrict__ koff, int ck, int64_t n, int64_t total,
                                   float* __restrict__ vc2, float* __restrict__ vn2, float* __restrict__ vu) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= total) return;
  const int64_t b = w / ck;
  const int j = (int)(w % ck);
  const float4 cb = reinterpret_cast<const float4*>(vbar + (b * ck + j) * kSD)[lane];
  float c2 = cb.x * cb.x + cb.y * cb.y + cb.z * cb.z + cb.w * cb.w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c2 += __shfl_xor_sync(0xffffffffu, c2, o);
  if (lane == 0) vc2[b * ck + j] = c2;
  const int32_t beg = koff[b * (ck + 1) + j], end = koff[b * (ck + 1) + j + 1];
  for (int32_t t = beg; t < end; ++t) {
    const uint2 u = reinterpret_cast<const uint2*>(vs + (b * n + t) * kSD)[lane];
    const __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    const float x0 = __low2float(h0), x1 = __high2float(h0), x2 = __low2float(h1), x3 = __high2float(h1);
    float nn = x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
    float dd = x0 * cb.x + x1 * cb.y + x2 * cb.z + x3 * cb.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nn += __shfl_xor_sync(0xffffffffu, nn, o);
      dd += __shfl_xor_sync(0xffffffffu, dd, o);
    }
    if (lane == 0) {
      vn2[b * n + t] = nn;
      vu[b * n + t] = dd;
    }
  }
}

// clog[b][c][j] = q_c . kbar_j / sqrt(D): grid (ceil(ck/32), bh); the block
// stages 32 centroid rows and each thread takes query centroids c.
__global__ void __launch_bounds__(256) centroid_logits_kernel(const float* __restrict__ qc,
                                                              const float* __restrict__ kbar, int cq, int ck,
                                                              float* __restrict__ clog) {
  __shared__ float4 s_k[32][kSD / 4];
  const int64_t b = blockIdx.y;
  const int j0 = blockIdx.x * 32;
  for (int i = threadIdx.x; i < 32 * (kSD / 4); i += blockDim.x) {
    const int jj = i / (kSD / 4), d4 = i % (kSD / 4);
    s_k[jj][d4] = j0 + jj < ck ? reinterpret_cast<const float4*>(kbar + (b * ck + j0 + jj) * kSD)[d4]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const float scale = rsqrtf((float)kSD);
  for (int c = threadIdx.x; c < cq; c += blockDim.x) {
    const float4* qr = reinterpret_cast<const float4*>(qc + (b * cq + c) * kSD);
    float acc[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) acc[jj] = 0.f;
    for (int d4 = 0; d4 < kSD / 4; ++d4) {
      const float4 qv = __ldg(qr + d4);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float4 kv = s_k[jj][d4];
        acc[jj] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, acc[jj]))));
      }
    }
    for (int jj = 0; jj < 32 && j0 + jj < ck; ++jj) clog[(b * cq + c) * ck + j0 + jj] = acc[jj] * scale;
  }
}

struct ValueTerms {
  const float* clog;  // [bh][cq][ck] centroid logits q_c . kbar_j / sqrt(D)
  const float* vc2;   // [bh][ck] |vbar_j|^2
  const float* vn2;   // [bh][n]  |v_t|^2 (sorted token order)
  const float* vu;    // [bh][n]  v_t . vbar_(cluster of t)
};

template <bool VALUE>
__global__ void __launch_bounds__(kSThreads, 1)
scores_tc_kernel(const __grid_constant__ CUtensorMap kmap, const float* __restrict__ qc,
                 const int32_t* __restrict__ koff, int cq, int ck, int64_t n, int64_t items,
                 float* __restrict__ scores, int* __restrict__ err, ValueTerms vt) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_a_full, bar_a_empty, bar_b_full[kSStages], bar_b_empty[kSStages], bar_d_full[2],
      bar_d_free[2], bar_mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ __align__(16) float s_vt[VALUE ? 2 : 1][2][kSN];  // token terms per tile (VALUE mode)
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
      if constexpr (!VALUE) {
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
      } else {
      float* out = scores + (b * cq + (row_ok ? c : 0)) * (int64_t)ck;
      const float* clog_row = vt.clog + (b * cq + (row_ok ? c : 0)) * (int64_t)ck;
      // Cluster walk: current cluster j spans tokens [jbeg, jend).  Base-2
      // running max m starts at the centroid logit c2; ea = sum 2^(2(l-m)) |v|^2,
      // eb = sum 2^(l-m) v.vbar (l = token logit in base 2).
      int j = c0;
      int32_t jbeg = t0, jend = t0;
      float c2 = 0.f, m = 0.f, ea = 0.f, eb = 0.f;
      auto advance = [&]() {
        while (j < c1) {
          jbeg = __ldg(koff + b * (ck + 1) + j);
          jend = __ldg(koff + b * (ck + 1) + j + 1);
          if (jend > jbeg) {
            c2 = __ldg(clog_row + j) * 1.4426950408889634f;
            m = c2;
            ea = 0.f;
            eb = 0.f;
            return;
          }
          if (row_ok) out[j] = -INFINITY;
          ++j;
        }
      };
      advance();
      for (int32_t tt = t0; tt < t1; tt += kSN, ++nt) {
        const int db = (int)(nt & 1);
        // Stage this tile's token terms (all four epilogue warps take part,
        // also after a wait gave up, so the named barrier is never short).
        {
          const int64_t t = tt + r;
          s_vt[nt & 1][0][r] = t < t1 ? __ldg(vt.vn2 + b * n + t) : 0.f;
          s_vt[nt & 1][1][r] = t < t1 ? __ldg(vt.vu + b * n + t) : 0.f;
          tc::named_bar(1, kSEpi);
        }
        ok = ok && __all_sync(0xffffffffu, tc::mbar_wait(&bar_d_full[db], (uint32_t)((nt >> 1) & 1), err, 44));
        tc::tc_fence_after();
        if (ok) {
#pragma unroll 1
          for (int blk = 0; blk < kSN / 32; ++blk) {
            const int32_t bt = tt + blk * 32;
            if (bt >= t1) break;
            float acc[32];
            tc::tmem_ld32(tmem + lane_base + db * kSN + blk * 32, acc);
            const float* wn = &s_vt[nt & 1][0][blk * 32];
            const float* wu = &s_vt[nt & 1][1][blk * 32];
            const int32_t be = min(bt + 32, t1);
            int32_t pos = bt;
            while (pos < be) {  // runs of one cluster inside this 32-token block (warp-uniform)
              const int32_t re = min(jend, be);
              const int a = pos - bt, e = re - bt;
              float bm = -INFINITY;
#pragma unroll
              for (int q = 0; q < 32; ++q) bm = (q >= a && q < e) ? fmaxf(bm, acc[q]) : bm;
              const float mn = fmaxf(m, bm * sc);
              const float rs = tc::ex2(m - mn);
              float A = ea * rs * rs, B = eb * rs;
              const float nm = -mn;
#pragma unroll
              for (int q = 0; q < 32; ++q) {
                if (q >= a && q < e) {
                  const float w = tc::ex2(fmaf(acc[q], sc, nm));
                  A = fmaf(w * w, wn[q], A);
                  B = fmaf(w, wu[q], B);
                }
              }
              ea = A;
              eb = B;
              m = mn;
              pos = re;
              if (pos == jend) {  // cluster j complete
                const float cnt = (float)(jend - jbeg);
                const float av = tc::ex2(c2 - m);
                const float err2 = fmaf(cnt * av * av, __ldg(vt.vc2 + b * ck + j), fmaf(-2.f * av, eb, ea));
                if (row_ok) out[j] = (__log2f(fmaxf(err2 / cnt, 1e-30f)) + 2.f * m) * ln2;
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

extern "C" int spr_attention_mass_scores_status_async(int32_t* dst, void* stream) {
  if (!dst) return fail(SPR_ERR_ARG, "attention-mass scores status: null destination");
  const cudaError_t e = cudaMemcpyFromSymbolAsync(dst, g_scores_err, sizeof(int), 0, cudaMemcpyDeviceToDevice,
                                                  (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "attention-mass scores status: %s", cudaGetErrorString(e));
  return SPR_OK;
}

namespace {

int check_score_shapes(const float* q_centroids, const void* k_sorted, int64_t bh, int cq, int ck, int64_t n, int d,
                       const char* what) {
  if (d != kSD) return fail(SPR_ERR_SHAPE, "%s require d=128, got %d", what, d);
  if (bh <= 0 || cq <= 0 || ck <= 0 || n <= 0 || bh > 65535 || n > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "%s: bad shape bh=%lld cq=%d ck=%d n=%lld", what, (long long)bh, cq, ck, (long long)n);
  if (!aligned(q_centroids, 16) || !aligned(k_sorted, 16))
    return fail(SPR_ERR_ALIGN, "%s: 16-byte alignment required", what);
  return SPR_OK;
}

template <bool VALUE>
int launch_scores(const float* q_centroids, const void* k_sorted, const int32_t* k_offsets, int64_t bh, int cq,
                  int ck, int64_t n, float* scores, ValueTerms vt, cudaStream_t st, const char* what) {
  // Keys [bh][n][128] bf16: box 64 features (128 bytes) x 128 tokens.
  CUtensorMap kmap;
  int s = encode_map_3d(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k_sorted, kSD, n, bh, 64, kSN, what);
  if (s) return s;
  cudaFuncSetAttribute(scores_tc_kernel<VALUE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmem);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = score_items(bh, cq, ck).items;
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);
  int* err = nullptr;
  cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_scores_err);
  cudaMemsetAsync(err, 0, sizeof(int), st);
  scores_tc_kernel<VALUE><<<grid, kSThreads, kSSmem, st>>>(kmap, q_centroids, k_offsets, cq, ck, n, items, scores,
                                                           err, vt);
  return check_launch(what);
}

struct ValueWs {
  float *clog, *vc2, *vn2, *vu;
};

ValueWs carve_value_ws(Carver& c, int64_t bh, int cq, int ck, int64_t n) {
  ValueWs w;
  w.clog = c.take<float>((size_t)bh * cq * ck);
  w.vc2 = c.take<float>((size_t)bh * ck);
  w.vn2 = c.take<float>((size_t)bh * n);
  w.vu = c.take<float>((size_t)bh * n);
  return w;
}

}  // namespace

extern "C" int spr_attention_mass_scores(const float* q_centroids, const void* k_sorted, const int32_t* k_offsets,
                                         int64_t bh, int cq, int ck, int64_t n, int d, float* scores, void* stream) {
  int s = check_score_shapes(q_centroids, k_sorted, bh, cq, ck, n, d, "attention-mass scores");
  if (s) return s;
  return launch_scores<false>(q_centroids, k_sorted, k_offsets, bh, cq, ck, n, scores, ValueTerms{},
                              (cudaStream_t)stream, "attention-mass scores (tcgen05)");
}

extern "C" size_t spr_svg_ear_value_scores_workspace_bytes(int64_t bh, int cq, int ck, int64_t n) {
  Carver c(nullptr, 0);
  carve_value_ws(c, bh, cq, ck, n);
  return c.off + 256;
}

extern "C" int spr_svg_ear_value_scores(const float* q_centroids, const void* k_sorted, const void* v_sorted,
                                        const float* k_centroids, const float* v_centroids,
                                        const int32_t* k_offsets, int64_t bh, int cq, int ck, int64_t n, int d,
                                        float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_score_shapes(q_centroids, k_sorted, bh, cq, ck, n, d, "SVG-EAR value scores");
  if (s) return s;
  if (!aligned(v_sorted, 16) || !aligned(k_centroids, 16) || !aligned(v_centroids, 16))
    return fail(SPR_ERR_ALIGN, "SVG-EAR value scores: 16-byte alignment required");
  Carver c(workspace, workspace_bytes);
  ValueWs w = carve_value_ws(c, bh, cq, ck, n);
  if (!workspace || !c.ok())
    return fail(SPR_ERR_WORKSPACE, "SVG-EAR value scores: workspace %zu < %zu", workspace_bytes, c.off);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t warps = bh * ck;
  value_terms_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(
      (const __nv_bfloat16*)v_sorted, v_centroids, k_offsets, ck, n, warps, w.vc2, w.vn2, w.vu);
  if ((s = check_launch("SVG-EAR value terms"))) return s;
  centroid_logits_kernel<<<dim3((unsigned)((ck + 31) / 32), (unsigned)bh), 256, 0, st>>>(q_centroids, k_centroids,
                                                                                        cq, ck, w.clog);
  if ((s = check_launch("SVG-EAR centroid logits"))) return s;
  return launch_scores<true>(q_centroids, k_sorted, k_offsets, bh, cq, ck, n, scores,
                             ValueTerms{w.clog, w.vc2, w.vn2, w.vu}, st, "SVG-EAR value scores (tcgen05)");
}
