// Block-sparse flash attention over kept (query-cluster, key-cluster) pairs on
// the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Work unit (one CTA): up to two 128-row query tiles A and B (256 consecutive
// rows) of one query cluster of the cluster-sorted Q.  Both tiles attend to
// the same keys: the concatenated token runs of the cluster's selected key
// clusters in the cluster-sorted K/V, consumed in 128-key tiles (only the last
// tile can be partial, so masking is a column bound).  Every K/V tile is
// loaded once and used by both query tiles.
//
// Warp roles (384 threads):
//   warps 0-3  softmax of tile A, warps 4-7 softmax of tile B: thread t of a
//              group owns query row t (= TMEM lane t).  Loads the S row from
//              TMEM, online softmax in base 2 with a lazily updated running
//              max, writes P (bf16) over the first 64 columns of its own S
//              region, rescales the O accumulator in TMEM when the max moves,
//              and finally normalises O and stores the row (through q_order:
//              the inverse permute is fused into the store).
//   warp 8     MMA issuer (one thread).  Order per key tile j:
//                PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)
//              so the tensor core works on one tile while the other tile's
//              softmax runs.  PV reads P from tensor memory.
//   warps 9-11 loaders: warps 9-10 gather K rows [64w, 64w+64) of each key
//              tile, warp 11 all V rows, each into a 2-stage ring with 16-byte
//              cp.async.  The selected clusters' runs (start, prefix length)
//              are staged in shared memory once per CTA; each loader lane
//              walks them with a forward cursor, and each warp instruction
//              moves two full 256-byte rows.
// TMEM: tile X in {A, B} owns columns [256X, 256X+128) for S(j) (P(j) over its
// first 64 columns, one 32-bit column per two keys) and [256X+128, 256X+256)
// for O.  tcgen05.commit tracks every earlier MMA of the issuing thread, so
// when S_X(j) is reported complete, PV_X(j-1) is complete too: the softmax may
// then rescale O_X and overwrite P_X without another barrier.  S_X(j+1) is
// issued after PV_X(j), which has read P_X by then (MMAs of one thread execute
// in issue order).
// The softmax arithmetic is the per-tile critical path: it uses packed fp32
// pair instructions (fma/add .f32x2), the three-input max, and takes one
// exponential in four off the MUFU unit (ex2_fma2).
// Operand tiles use the canonical 128-byte-swizzled K-major layout; V is the
// MN-major B operand of the PV product.
#include "tc_common.cuh"

namespace spr {

using namespace tc;

constexpr int kD = 128;
constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kPairRows = 2 * kTileM;   // query rows per CTA
constexpr int kSoftmaxThreads = 128;    // per query tile
constexpr int kThreadsTc = 384;
constexpr int kMaxRuns = 2048;  // key clusters per problem (ck) this kernel accepts
constexpr int kMaxRunsRepair = 1024;  // with the fused repair epilogue (its weights take the shared memory)
constexpr int kRepairRank = 16;
constexpr int kMaxProbes = 128;

// Kernel modes.
//   kModePlain : attention output (optionally stored through q_order).
//   kModeRepair: the same, then the reduced-rank residual repair applied in
//                the epilogue and probe rows overwritten by their dense rows
//                (kernels/triton/residual_repair.py:158-254 fused apply +
//                overwrite, CPU twin models/common/n8_v6.py:1384-1395).
//   kModeProbe : the probe pre-pass.  Tiles A and B hold the same probe rows
//                (gathered from the original-order Q); both see every key,
//                A unmasked (the exact dense rows, n8_v6.py:1234-1243) and B
//                masked to its row's selected key clusters (the rows' sparse
//                output, which the repair fit regresses from).
enum : int { kModePlain = 0, kModeRepair = 1, kModeProbe = 2 };

// Fused repair state (kModeRepair), per problem b:
//   image [b] (kRepairImageBytes): the tensor-core operands of the correction,
//     laid out as their shared-memory tiles (128-byte swizzle, K-major), each
//     fp32 matrix as a bf16 (hi, lo) pair, hi + lo = the value to ~2^-16:
//       L'hi, L'lo  [16 rows j][128 K d]  (L' = L / x_scale)        4 KB each
//       Bhi, Blo    [128 rows d][64 K j, j < 16 used, rest 0]       16 KB each
//   c0 [b][16] = -sum_d x_mean[d] L'[d][:], y_mean [b][128];
//   probe_tok [b][m] ascending token ids and probe_dense [b][m][128] their exact rows.
// out = bf16(v + alpha * (y_mean + (v L' + c0) B^T)), v = bf16(attention row).
constexpr int kImgL = 16 * kD * 2;        // one L' part
constexpr int kImgB = kD * 128;           // one B part (128 rows x 128 bytes)
constexpr int kRepairImageBytes = 2 * kImgL + 2 * kImgB;
struct AttnRepair {
  const uint8_t* image;
  const float* c0;
  const float* y_mean;
  const int32_t* probe_tok;
  const __nv_bfloat16* probe_dense;
  int m;
  float alpha;
};

// Probe pre-pass (kModeProbe), per problem b: rows [b][m] token ids into the
// original-order Q, row_cluster [b][m] their query clusters, routed [b][cq+1][ck+1]
// the cluster-pair map (header row/column first).  The keys are split into
// `splits` contiguous ranges (blockIdx.x); each CTA writes its unnormalised
// partial rows o_part [b][split][tile][m][128] and (running max, sum) ml_part
// [b][split][tile][m][2]; probe_merge_kernel combines them.
struct AttnProbe {
  const int32_t* rows;
  const int32_t* row_cluster;
  const uint8_t* routed;
  float* o_part;
  float* ml_part;
  int m;
  int splits;
};
constexpr int kTileBytes = kTileM * kD * 2;    // 32 KB per 128 x 128 bf16 tile
constexpr int kSmemTc = 1024 /*align slack*/ + 2 * kTileBytes /*Q_A, Q_B*/ + 4 * kTileBytes /*K,V x2*/;
constexpr uint32_t kIdescQK = idesc_bf16_f32(128, 128, 0);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, 1);
constexpr uint32_t kIdescD1 = idesc_bf16_f32(128, 16, 0);  // repair: v L' (N = 16, both K-major)

enum : int { kErrTimeoutLoad = 1, kErrTimeoutMma = 2, kErrTimeoutSoftmax = 3 };

// Packed fp32 pairs (sm_100 f32x2 instructions) and the three-input max.
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair of scores on the FMA pipe, for the share of the softmax
// exponentials taken off the MUFU unit.  Cody-Waite split x = n + f with
// n = round(x) from the low mantissa bits of x + 1.5*2^23 and |f| <= 1/2;
// 2^f from a cubic with constant term 1 fitted for minimum relative error on
// [-1/2, 1/2] (max 1.0e-4, below the 2^-9 rounding of P to bf16); 2^n added
// to the exponent field.  Inputs below -125 (including -inf) give 2^-125.
__device__ __forceinline__ void ex2_fma2(float x0, float x1, float& p0, float& p1) {
  const unsigned long long xc = pk2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const unsigned long long mg = pk2(12582912.f, 12582912.f);
  const unsigned long long t = add2(xc, mg);
  const unsigned long long f = add2(xc, fma2(t, pk2(-1.f, -1.f), mg));  // x - (t - magic)
  unsigned long long q = fma2(f, pk2(0.055008821f, 0.055008821f), pk2(0.24221078f, 0.24221078f));
  q = fma2(q, f, pk2(0.69328290f, 0.69328290f));
  q = fma2(q, f, pk2(1.f, 1.f));
  float q0, q1, t0, t1;
  up2(q, q0, q1);
  up2(t, t0, t1);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// err[0] = 0, tile_start[b][c] = first 256-row unit of query cluster c in
// problem b (exclusive prefix of ceil(size/256)); tile_start[b][cq] = total.
__global__ void tile_table_kernel(const int32_t* __restrict__ q_offsets, int cq, int32_t* __restrict__ tile_start,
                                  int* __restrict__ err) {
  const int64_t b = blockIdx.x;
  if (threadIdx.x != 0) return;
  if (b == 0) *err = 0;
  int32_t acc = 0;
  for (int c = 0; c < cq; ++c) {
    tile_start[b * (cq + 1) + c] = acc;
    const int32_t sz = q_offsets[b * (cq + 1) + c + 1] - q_offsets[b * (cq + 1) + c];
    acc += (sz + kPairRows - 1) / kPairRows;
  }
  tile_start[b * (cq + 1) + cq] = acc;
}

template <int MODE>
__global__ void __launch_bounds__(kThreadsTc, 1)
block_sparse_attn_tc_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const __nv_bfloat16* __restrict__ v, const int32_t* __restrict__ q_offsets,
                            const int32_t* __restrict__ k_offsets, const int32_t* __restrict__ sel_ids,
                            const int32_t* __restrict__ sel_counts, const int32_t* __restrict__ tile_start,
                            int64_t nq, int64_t nk, int cq, int ck, const int32_t* __restrict__ q_order,
                            __nv_bfloat16* __restrict__ out, float scale_log2, int* __restrict__ err,
                            const AttnRepair rep, const AttnProbe prb) {
  constexpr int kRuns = MODE == kModeRepair ? kMaxRunsRepair : (MODE == kModeProbe ? 1 : kMaxRuns);
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_k_full[2], bar_k_empty[2], bar_v_full[2], bar_v_empty[2], bar_s_full[2], bar_p_full[2],
      bar_o_done[2];
  __shared__ uint32_t s_tmem;
  __shared__ int32_t s_run_start[kRuns];
  __shared__ int32_t s_run_end[kRuns + 1];  // inclusive prefix of run lengths
  __shared__ int s_total;
  // Fused repair (kModeRepair only; one element otherwise).
  __shared__ float s_c0[MODE == kModeRepair ? kRepairRank : 1], s_ym[MODE == kModeRepair ? kD : 1];
  __shared__ int32_t s_ptok[MODE == kModeRepair ? kMaxProbes : 1];
  // Epilogue barriers of the repair MMAs (single phase): operand image landed,
  // rows v of tile x written, D1 = v L' done, coords of tile x written, D2 done.
  __shared__ uint64_t bar_img, bar_v_ready[2], bar_d1[2], bar_a2_ready[2], bar_d2[2];

  const int64_t b = blockIdx.y;
  int c = 0, row0 = 0, rows_a, rows_b;
  if constexpr (MODE == kModeProbe) {
    rows_a = rows_b = prb.m;  // one unit per problem: the probe rows in both tiles
  } else {
    const int unit = blockIdx.x;
    const int32_t* ts = tile_start + b * (cq + 1);
    if (unit >= ts[cq]) return;  // block-uniform, before any barrier or TMEM use
    int lo = 0, hi = cq - 1;     // query cluster owning the unit: last c with ts[c] <= unit
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (ts[mid] <= unit) lo = mid; else hi = mid - 1;
    }
    c = lo;
    const int32_t qbeg = q_offsets[b * (cq + 1) + c];
    const int32_t qend = q_offsets[b * (cq + 1) + c + 1];
    row0 = qbeg + (unit - ts[c]) * kPairRows;
    rows_a = min(kTileM, qend - row0);
    rows_b = max(0, min(kTileM, qend - row0 - kTileM));
  }
  const bool has_b = rows_b > 0;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // Q_A, Q_B
  uint8_t* sK = sQ + 2 * kTileBytes;    // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;    // 2 stages

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* qb = q + b * nq * kD;
  const __nv_bfloat16* kb = k + b * nk * kD;
  const __nv_bfloat16* vb = v + b * nk * kD;
  const int32_t* ids = MODE == kModeProbe ? nullptr : sel_ids + (b * cq + c) * (int64_t)ck;
  const int nsel = MODE == kModeProbe ? 0 : sel_counts[b * cq + c];
  const int32_t* ko = k_offsets + b * (ck + 1);

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_k_full[i], 64);  // two K loader warps
      mbar_init(&bar_v_full[i], 32);  // one V loader warp
      mbar_init(&bar_k_empty[i], 1);
      mbar_init(&bar_v_empty[i], 1);
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_p_full[i], kSoftmaxThreads);
      mbar_init(&bar_o_done[i], 1);
    }
    mbar_fence_init();
  }
  if (warp == 8) tmem_alloc<512>(&s_tmem);
  if constexpr (MODE == kModeRepair) {  // repair vectors and probe tokens of this problem
    if (tid == 0) {
      mbar_init(&bar_img, 1);
      for (int i = 0; i < 2; ++i) {
        mbar_init(&bar_v_ready[i], kSoftmaxThreads);
        mbar_init(&bar_d1[i], 1);
        mbar_init(&bar_a2_ready[i], kSoftmaxThreads);
        mbar_init(&bar_d2[i], 1);
      }
      mbar_fence_init();
    }
    if (tid < kRepairRank) s_c0[tid] = rep.c0[b * kRepairRank + tid];
    if (tid < kD) s_ym[tid] = rep.y_mean[b * kD + tid];
    if (tid < rep.m) s_ptok[tid] = rep.probe_tok[b * rep.m + tid];
  }
  if (MODE == kModeProbe && warp == 9 && lane == 0) {  // this split's key range: one run over the sorted K/V
    const int64_t tiles = (nk + kTileN - 1) / kTileN;
    const int64_t per = (tiles + prb.splits - 1) / prb.splits;
    const int64_t k0 = min((int64_t)blockIdx.x * per * kTileN, nk), k1 = min(k0 + per * kTileN, nk);
    s_run_start[0] = (int32_t)k0;
    s_run_end[0] = (int32_t)(k1 - k0);
    s_total = (int)(k1 - k0);
  }
  if (MODE != kModeProbe && warp == 9) {  // run table of the selected key clusters: start row and prefix length
    int carry = 0;
    for (int base = 0; base < nsel; base += 32) {
      const int i = base + lane;
      int start = 0, len = 0;
      if (i < nsel) {
        const int kc = ids[i];
        start = ko[kc];
        len = ko[kc + 1] - start;
      }
      int incl = len;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (i < nsel) {
        s_run_start[i] = start;
        s_run_end[i] = carry + incl;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_total = carry;
  }
  // Q tiles (all threads), zero rows past the cluster end.  Probe mode: both
  // tiles hold the probe rows, gathered from the original-order Q.
  for (int i = tid; i < 2 * kTileM * 16; i += kThreadsTc) {
    const int t = i >> 11, r = (i >> 4) & 127, ch = i & 15;
    const bool ok = r < (t ? rows_b : rows_a);
    int64_t src_row;
    if constexpr (MODE == kModeProbe)
      src_row = ok ? (int64_t)prb.rows[b * prb.m + r] : 0;
    else
      src_row = row0 + t * kTileM + (ok ? r : 0);
    cp_async16(smem_addr(sQ + t * kTileBytes) + sw128_off(r, ch, kTileM), qb + src_row * kD + ch * 8, ok);
  }
  cp_async_commit();
  cp_async_wait_all();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int total = s_total;
  const int ntiles = (total + kTileN - 1) / kTileN;

  if (warp >= 9) {
    // ------------------------------------------------------------ loaders
    const bool is_v = warp == 11;
    const int nsub = is_v ? 4 : 2;                // 32-row groups handled by this warp
    const int band = is_v ? 0 : (warp - 9) * 64;  // first row of this warp's band
    const __nv_bfloat16* srcb = is_v ? vb : kb;
    uint8_t* ring = is_v ? sV : sK;
    uint64_t* full = is_v ? bar_v_full : bar_k_full;
    uint64_t* empty = is_v ? bar_v_empty : bar_k_empty;
    const int half = lane >> 4, ch = lane & 15;
    // Per-lane run cursors: slot g = j*128 + band + 32*sub + lane grows by 128
    // per tile, so each cursor only walks forward over the runs it passes.
    int cur[4] = {0, 0, 0, 0};
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      int src[4];
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        src[sub] = -1;
        const int g = j * kTileN + band + sub * 32 + lane;
        if (sub < nsub && g < total) {
          while (s_run_end[cur[sub]] <= g) ++cur[sub];
          const int prev = cur[sub] > 0 ? s_run_end[cur[sub] - 1] : 0;
          src[sub] = s_run_start[cur[sub]] + (g - prev);
        }
      }
      if (j >= 2 && !mbar_wait(&empty[st], ((j >> 1) - 1) & 1, err, kErrTimeoutLoad)) break;
      // Swizzled destination of (row r, chunk ch): rows of one warp step differ
      // only in (r & 7), fixed per unrolled iteration.
      const uint32_t dst = smem_addr(ring + st * kTileBytes) + (uint32_t)(ch >> 3) * (kTileN * 128) +
                           (uint32_t)band * 128;
      const __nv_bfloat16* colp = srcb + ch * 8;
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        if (sub >= nsub) break;  // warp-uniform
#pragma unroll
        for (int pr = 0; pr < 16; ++pr) {  // two rows per instruction: lanes 0-15 row 2pr, 16-31 row 2pr+1
          const int rl = 2 * pr + half;
          const int rsrc = __shfl_sync(0xffffffffu, src[sub], rl);
          const int rr = sub * 32 + rl;  // row within this warp's band (band start is 8-aligned)
          const uint32_t o = (uint32_t)rr * 128 + ((uint32_t)((ch & 7) ^ (rr & 7)) << 4);
          cp_async16(dst + o, colp + (uint32_t)max(rsrc, 0) * (uint32_t)kD, rsrc >= 0);
        }
      }
      cp_async_arrive(&full[st]);  // completes when this lane's copies have landed
    }
    cp_async_wait_all();
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t aq = smem_addr(sQ);
      auto issue_s = [&](int x, int j) {  // S_x(j) = Q_x K_j^T (K_j resident)
        const uint32_t bk = smem_addr(sK + (j & 1) * kTileBytes);
        const uint32_t ax = aq + x * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {  // K-major: 32 B per 16-element step, second half +16 KB
          const uint32_t koff = (kk >> 2) * (kTileM * 128) + (kk & 3) * 32;
          mma_f16(tmem + 256 * x, sw128_desc(ax + koff, 16, 1024), sw128_desc(bk + koff, 16, 1024), kIdescQK,
                  kk > 0);
        }
        mma_commit(&bar_s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {  // O_x += P_x(j) V_j, P_x from tensor memory
        const uint32_t bv = smem_addr(sV + (j & 1) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {  // 16 keys per step = 8 TMEM columns of P
          const uint32_t voff = kk * 2048;         // V is MN-major: 16 rows = 2 x 1024 B
          mma_f16_ts(tmem + 256 * x + 128, tmem + 256 * x + kk * 8, sw128_desc(bv + voff, kTileN * 128, 1024),
                     kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&bar_k_full[0], 0, err, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (has_b) issue_s(1, 0);
        mma_commit(&bar_k_empty[0]);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const bool next = j + 1 < ntiles;
        if (!(ok = mbar_wait(&bar_v_full[j & 1], (j >> 1) & 1, err, kErrTimeoutMma))) break;
        if (next && !(ok = mbar_wait(&bar_k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, err, kErrTimeoutMma))) break;
        if (!(ok = mbar_wait(&bar_p_full[0], j & 1, err, kErrTimeoutMma))) break;
        tc_fence_after();
        issue_pv(0, j);
        if (next) issue_s(0, j + 1);
        if (has_b) {
          if (!(ok = mbar_wait(&bar_p_full[1], j & 1, err, kErrTimeoutMma))) break;
          tc_fence_after();
          issue_pv(1, j);
          if (next) issue_s(1, j + 1);
        }
        mma_commit(&bar_v_empty[j & 1]);
        if (next) mma_commit(&bar_k_empty[(j + 1) & 1]);
      }
      mma_commit(&bar_o_done[0]);
      mma_commit(&bar_o_done[1]);
    }
    if constexpr (MODE == kModeRepair) {
      // Repair MMAs of the epilogue, per query tile x: D1 = v L' (two bf16 parts
      // of L', N = 16) into the first columns of x's O region, then
      // D2 = coords B^T (hi.hi + hi.lo + lo.hi, one K = 16 step each) into x's
      // S region.  The operand image goes to the K/V rings, free once every
      // MMA above has completed.
      if (lane == 0) {
        bool eok = true;
        if (ntiles > 0)
          eok = mbar_wait(&bar_o_done[0], 0, err, kErrTimeoutMma) && mbar_wait(&bar_o_done[1], 0, err, kErrTimeoutMma);
        const uint32_t img = smem_addr(sK);
        const uint32_t l_hi = img, l_lo = img + kImgL, b_hi = img + 2 * kImgL, b_lo = b_hi + kImgB;
        const uint32_t a2 = img + kRepairImageBytes;  // [tile][hi, lo] coords tiles, 128 rows x 128 B each
        bool img_issued = false;
        if (eok) {
          tc_fence_after();
          mbar_expect_tx(&bar_img, (uint32_t)kRepairImageBytes);
          bulk_load(img, rep.image + b * (int64_t)kRepairImageBytes, (uint32_t)kRepairImageBytes, &bar_img);
          img_issued = true;
          eok = mbar_wait(&bar_img, 0, err, kErrTimeoutMma);
        }
        const int tiles = has_b ? 2 : 1;
        for (int xt = 0; eok && xt < tiles; ++xt) {
          if (!(eok = mbar_wait(&bar_v_ready[xt], 0, err, kErrTimeoutMma))) break;
          tc_fence_after();
          const uint32_t va = smem_addr(sQ + xt * kTileBytes);
#pragma unroll
          for (int part = 0; part < 2; ++part) {
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t koff_a = (kk >> 2) * (kTileM * 128) + (kk & 3) * 32;
              const uint32_t koff_b = (kk >> 2) * (16 * 128) + (kk & 3) * 32;
              mma_f16(tmem + 256 * xt + 128, sw128_desc(va + koff_a, 16, 1024),
                      sw128_desc((part ? l_lo : l_hi) + koff_b, 16, 1024), kIdescD1, (part > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&bar_d1[xt]);
        }
        for (int xt = 0; eok && xt < tiles; ++xt) {
          if (!(eok = mbar_wait(&bar_a2_ready[xt], 0, err, kErrTimeoutMma))) break;
          tc_fence_after();
          const uint32_t a_hi = a2 + xt * 2 * kImgB, a_lo = a_hi + kImgB;
          mma_f16(tmem + 256 * xt, sw128_desc(a_hi, 16, 1024), sw128_desc(b_hi, 16, 1024), kIdescQK, 0u);
          mma_f16(tmem + 256 * xt, sw128_desc(a_hi, 16, 1024), sw128_desc(b_lo, 16, 1024), kIdescQK, 1u);
          mma_f16(tmem + 256 * xt, sw128_desc(a_lo, 16, 1024), sw128_desc(b_hi, 16, 1024), kIdescQK, 1u);
          mma_commit(&bar_d2[xt]);
        }
        // Every MMA issued here has finished before TMEM is freed; a copy still
        // in flight (a wait gave up) lands before the CTA exits.
        mma_commit(&bar_o_done[0]);
        if (img_issued) mbar_drain(&bar_img, 0);
        mbar_drain(&bar_o_done[0], ntiles > 0 ? 1 : 0);
      }
    }
  } else if (warp < 4 || has_b) {
    // ------------------------------------------------------------ softmax (thread = row)
    const int x = warp >> 2;  // query tile
    const int rows = x ? rows_b : rows_a;
    const int row = tid & 127;  // TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + 256 * x, tO = tS + 128;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Probe mode, tile B: this row's cluster-pair map row and a forward cursor
    // over the key clusters of the sorted keys.
    const bool masked = MODE == kModeProbe && x == 1;
    const uint8_t* maprow = nullptr;
    int kc_cur = 0;
    const int key0 = MODE == kModeProbe ? s_run_start[0] : 0;  // first sorted key of this split
    if (MODE == kModeProbe && masked && row < rows) {
      const int crow = prb.row_cluster[b * prb.m + row];
      maprow = prb.routed + ((b * (cq + 1)) + crow + 1) * (int64_t)(ck + 1) + 1;
    }
    for (int j = 0; j < ntiles && ok; ++j) {
      const uint32_t tSj = tS;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_s_full[x], j & 1, err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      float s[kTileN];
      tmem_ld32_async(tSj, s);  // four loads in flight, one wait
      tmem_ld32_async(tSj + 32, s + 32);
      tmem_ld32_async(tSj + 64, s + 64);
      tmem_ld32_async(tSj + 96, s + 96);
      tmem_wait_ld();
      reg_fence32(s);
      reg_fence32(s + 32);
      reg_fence32(s + 64);
      reg_fence32(s + 96);
      const int valid = total - j * kTileN;
      if (valid < kTileN) {  // only the last tile of a cluster is partial (warp-uniform)
#pragma unroll
        for (int i = 0; i < kTileN; ++i) s[i] = i < valid ? s[i] : -INFINITY;
      }
      if (MODE == kModeProbe && masked) {
        // Keys of this tile that lie in a key cluster this row's query
        // cluster keeps; the cluster segments are the same for every row.
        uint32_t keep[4] = {0u, 0u, 0u, 0u};
        const int t0 = key0 + j * kTileN, t1 = min(t0 + kTileN, key0 + total);
        if (j == 0) {  // first tile of this split: the key cluster holding t0 by binary search
          int lo2 = 0, hi2 = ck - 1;  // last kc with ko[kc] <= t0
          while (lo2 < hi2) {
            const int mid = (lo2 + hi2 + 1) >> 1;
            if (ko[mid] <= t0) lo2 = mid; else hi2 = mid - 1;
          }
          kc_cur = lo2;
        }
        while (ko[kc_cur + 1] <= t0) ++kc_cur;
        for (int pos = t0, kc = kc_cur; pos < t1; ++kc) {
          const int seg_end = min((int)ko[kc + 1], t1);
          if (seg_end > pos && maprow && maprow[kc]) {
            const int lo_i = pos - t0, hi_i = seg_end - t0;  // bits [lo_i, hi_i) of the tile
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const int a0 = max(lo_i - 32 * w, 0), a1 = min(hi_i - 32 * w, 32);
              if (a1 > a0) keep[w] |= (a1 - a0 == 32 ? 0xffffffffu : ((1u << (a1 - a0)) - 1u)) << a0;
            }
          }
          pos = max(pos, seg_end);
        }
#pragma unroll
        for (int i = 0; i < kTileN; ++i) s[i] = ((keep[i >> 5] >> (i & 31)) & 1u) ? s[i] : -INFINITY;
      }
      float m8[8];  // eight independent max chains, two scores per instruction
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) m8[cc] = fmaxf(s[2 * cc], s[2 * cc + 1]);
#pragma unroll
      for (int i = 16; i < kTileN; i += 16) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) m8[cc] = max3(m8[cc], s[i + 2 * cc], s[i + 2 * cc + 1]);
      }
      const float mx = max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7])) * scale_log2;
      // Lazy max: keep the running max unless it grew by more than 8 (base 2).
      float alpha = 1.f;
      if (mx > m_run + 8.f || m_run == -INFINITY) {
        alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - mx);
        m_run = mx;
      }
      // A row whose keys so far are all masked (probe mode) keeps m = -inf and
      // exponentiates against 0 instead: every p is 0 and no NaN appears.
      const float m_use = MODE == kModeProbe && m_run == -INFINITY ? 0.f : m_run;
      const unsigned long long sc2 = pk2(scale_log2, scale_log2), nm2 = pk2(-m_use, -m_use);
      unsigned long long sum2[4] = {0ull, 0ull, 0ull, 0ull};  // packed partial sums (+0.0f pairs)
      // P(j) over the first 64 columns of S(j) (already loaded above), in two
      // 64-key halves stored as soon as each is packed.
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pk[kTileN / 4];
#pragma unroll
        for (int i = 64 * hf; i < 64 * hf + 64; i += 2) {
          float x0, x1, p0, p1;
          up2(fma2(pk2(s[i], s[i + 1]), sc2, nm2), x0, x1);
          if ((i & 7) == 0) {  // one pair in four on the FMA pipe, the rest on MUFU
            ex2_fma2(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          sum2[(i >> 1) & 3] = add2(sum2[(i >> 1) & 3], pk2(p0, p1));
          __nv_bfloat162 hh = __floats2bfloat162_rn(p0, p1);
          pk[(i - 64 * hf) >> 1] = *reinterpret_cast<uint32_t*>(&hh);
        }
        tmem_st32(tSj + 32 * hf, reinterpret_cast<const float*>(pk));
      }
      float a0, a1, b0, b1;
      up2(add2(sum2[0], sum2[1]), a0, a1);
      up2(add2(sum2[2], sum2[3]), b0, b1);
      l_run = l_run * alpha + ((a0 + a1) + (b0 + b1));
      // PV_x(j-1) is complete (S_x(j) completed after it): O_x may be rescaled
      // (PV_x(j) waits for the arrive below).
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {  // warp-uniform: TMEM ld/st are warp-collective
        float o[32];
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          tmem_ld32(tO + cb * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tO + cb * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[x]);
    }
    // Epilogue: O / l, bf16, stored through the inverse permutation.
    if (ok && ntiles > 0) ok = mbar_wait(&bar_o_done[x], 0, err, kErrTimeoutSoftmax);
    const bool have = __all_sync(0xffffffffu, ok && ntiles > 0);
    tc_fence_after();
    const float inv = (have && l_run > 0.f) ? 1.f / l_run : 0.f;
    if constexpr (MODE == kModeProbe) {
      // Unnormalised partial rows of this key split (tile A: all keys, tile B:
      // the kept ones).  A row that saw no kept key reports l = 0.
      const bool any = have && m_run != -INFINITY;
      const int64_t pr = ((b * prb.splits + blockIdx.x) * 2 + x) * (int64_t)prb.m + (row < rows ? row : 0);
      float4* orow = reinterpret_cast<float4*>(prb.o_part + pr * kD);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float o[32];
        if (have) {
          tmem_ld32(tO + cb * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (row < rows) {
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            orow[cb * 8 + q4] = any ? make_float4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3])
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (row < rows) {
        prb.ml_part[2 * pr] = any ? m_run : -INFINITY;
        prb.ml_part[2 * pr + 1] = any ? l_run : 0.f;
      }
    } else if constexpr (MODE == kModeRepair) {
      // v = bf16(O / l) into x's Q tile (K-major, the MMA layout); the MMA
      // warp forms D1 = v L'; coords = D1 + c0 go back as bf16 (hi, lo) rows;
      // the MMA warp forms D2 = coords B^T; out = bf16(v + alpha (y_mean + D2)),
      // or the exact dense row for a probe token.
      const int64_t s_row = row0 + x * kTileM + row;
      const int64_t dst = (row < rows) ? (q_order ? (int64_t)q_order[b * nq + s_row] : s_row) : 0;
      uint8_t* vt = sQ + x * kTileBytes;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float o[32];
        if (have) {
          tmem_ld32(tO + cb * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 hh = __floats2bfloat162_rn(o[q4 * 8 + 2 * e] * inv, o[q4 * 8 + 2 * e + 1] * inv);
            w[e] = *reinterpret_cast<uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(vt + sw128_off(row, cb * 4 + q4, kTileM)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar_v_ready[x]);
      bool eok = __all_sync(0xffffffffu, mbar_wait(&bar_d1[x], 0, err, kErrTimeoutSoftmax));
      tc_fence_after();
      {
        float d1v[32];
        if (eok) {
          tmem_ld32(tO, d1v);  // columns 0..15 hold D1
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) d1v[i] = 0.f;
        }
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int jp = 0; jp < kRepairRank / 2; ++jp) {
          const float c0v = d1v[2 * jp] + s_c0[2 * jp], c1v = d1v[2 * jp + 1] + s_c0[2 * jp + 1];
          const __nv_bfloat162 hi = __floats2bfloat162_rn(c0v, c1v);
          const __nv_bfloat162 lo = __floats2bfloat162_rn(c0v - __low2float(hi), c1v - __high2float(hi));
          hw[jp] = *reinterpret_cast<const uint32_t*>(&hi);
          lw[jp] = *reinterpret_cast<const uint32_t*>(&lo);
        }
        uint8_t* a2 = sK + kRepairImageBytes + x * 2 * kImgB;  // coords tiles of this query tile
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          *reinterpret_cast<uint4*>(a2 + sw128_off(row, ch, kTileM)) =
              make_uint4(hw[4 * ch], hw[4 * ch + 1], hw[4 * ch + 2], hw[4 * ch + 3]);
          *reinterpret_cast<uint4*>(a2 + kImgB + sw128_off(row, ch, kTileM)) =
              make_uint4(lw[4 * ch], lw[4 * ch + 1], lw[4 * ch + 2], lw[4 * ch + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar_a2_ready[x]);
      eok = eok && __all_sync(0xffffffffu, mbar_wait(&bar_d2[x], 0, err, kErrTimeoutSoftmax));
      tc_fence_after();
      // Probe token?  (s_ptok ascending; -1 when not found.)
      int probe = -1;
      {
        int plo = 0, phi = rep.m - 1;
        while (plo <= phi) {
          const int mid = (plo + phi) >> 1;
          const int32_t tv = s_ptok[mid];
          if (tv == (int32_t)dst) { probe = mid; break; }
          if (tv < (int32_t)dst) plo = mid + 1; else phi = mid - 1;
        }
      }
      uint4* orow = reinterpret_cast<uint4*>(out + (b * nq + dst) * kD);
      const uint4* prow = reinterpret_cast<const uint4*>(rep.probe_dense + (b * rep.m + max(probe, 0)) * (int64_t)kD);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float d2v[32];
        if (eok) {
          tmem_ld32(tS + cb * 32, d2v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) d2v[i] = 0.f;
        }
        if (row < rows) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w4;
            if (probe >= 0) {
              w4 = prow[cb * 4 + q4];
            } else {
              const uint4 vv = *reinterpret_cast<const uint4*>(vt + sw128_off(row, cb * 4 + q4, kTileM));
              const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(&vw[e]);
                const int dcol = cb * 32 + q4 * 8 + 2 * e;
                const float r0 = fmaf(rep.alpha, s_ym[dcol] + d2v[q4 * 8 + 2 * e], __low2float(v2));
                const float r1 = fmaf(rep.alpha, s_ym[dcol + 1] + d2v[q4 * 8 + 2 * e + 1], __high2float(v2));
                __nv_bfloat162 hh = __floats2bfloat162_rn(r0, r1);
                w[e] = *reinterpret_cast<uint32_t*>(&hh);
              }
              w4 = make_uint4(w[0], w[1], w[2], w[3]);
            }
            orow[cb * 4 + q4] = w4;
          }
        }
      }
    } else {
      const int64_t s_row = row0 + x * kTileM + row;
      const int64_t dst = (row < rows) ? (q_order ? (int64_t)q_order[b * nq + s_row] : s_row) : 0;
      uint4* orow = reinterpret_cast<uint4*>(out + (b * nq + dst) * kD);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float o[32];
        if (have) {
          tmem_ld32(tO + cb * 32, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (row < rows) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 hh = __floats2bfloat162_rn(o[q4 * 8 + 2 * e] * inv, o[q4 * 8 + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<uint32_t*>(&hh);
            }
            orow[cb * 4 + q4] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

}  // namespace spr

namespace spr {

// Per problem b: L' = L / xs (correctly rounded division), c0[j] = -sum_d xm[d] L'[d][j]
// in d order, and the repair operand image of the attention epilogue (bf16 hi/lo
// parts of L'^T [16 x 128] and of B [128 x 16] in their 128-byte-swizzled
// K-major shared-memory layouts, B's K padded with zeros to 64).
__global__ void repair_fold_kernel(const float* __restrict__ xm, const float* __restrict__ xs,
                                   const float* __restrict__ left, const float* __restrict__ basis,
                                   uint8_t* __restrict__ image, float* __restrict__ c0) {
  const int64_t b = blockIdx.x;
  __shared__ float sh[kD * kRepairRank];
  uint8_t* img = image + b * (int64_t)kRepairImageBytes;
  for (int i = threadIdx.x; i < kD * kRepairRank; i += blockDim.x) {
    const int d = i / kRepairRank, j = i % kRepairRank;
    const float lv = __fdiv_rn(left[b * kD * kRepairRank + i], xs[b * kD + d]);
    sh[i] = lv;
    // L'^T: row j, K index d.
    const __nv_bfloat16 lh = __float2bfloat16_rn(lv);
    const __nv_bfloat16 ll = __float2bfloat16_rn(lv - __bfloat162float(lh));
    const uint32_t lo = sw128_off(j, d >> 3, 16) + (d & 7) * 2;
    *reinterpret_cast<__nv_bfloat16*>(img + lo) = lh;
    *reinterpret_cast<__nv_bfloat16*>(img + kImgL + lo) = ll;
  }
  for (int i = threadIdx.x; i < kD * 64; i += blockDim.x) {
    // B: row d, K index j (j >= 16 is zero padding).
    const int d = i / 64, j = i % 64;
    const float bv = j < kRepairRank ? basis[b * kD * kRepairRank + d * kRepairRank + j] : 0.f;
    const __nv_bfloat16 bh = __float2bfloat16_rn(bv);
    const __nv_bfloat16 bl = __float2bfloat16_rn(bv - __bfloat162float(bh));
    const uint32_t bo = sw128_off(d, j >> 3, kD) + (j & 7) * 2;
    *reinterpret_cast<__nv_bfloat16*>(img + 2 * kImgL + bo) = bh;
    *reinterpret_cast<__nv_bfloat16*>(img + 2 * kImgL + kImgB + bo) = bl;
  }
  __syncthreads();
  if (threadIdx.x < kRepairRank) {
    float c = 0.f;
    for (int d = 0; d < kD; ++d) c = fmaf(-xm[b * kD + d], sh[d * kRepairRank + threadIdx.x], c);
    c0[b * kRepairRank + threadIdx.x] = c;
  }
}

// Combine the key splits of the probe pre-pass, per (b, tile, row) and column:
// M = max_s m_s, out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s in split
// order (0 when no split saw a kept key), rounded to bf16.  Tile 0 -> out_dense,
// tile 1 -> out_base.
__global__ void probe_merge_kernel(const float* __restrict__ o_part, const float* __restrict__ ml_part, int splits,
                                   int m, __nv_bfloat16* __restrict__ out_dense, __nv_bfloat16* __restrict__ out_base) {
  const int r = blockIdx.x, x = blockIdx.y, col = threadIdx.x;
  const int64_t b = blockIdx.z;
  float mx = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) mx = fmaxf(mx, ml_part[2 * (((b * splits + sp) * 2 + x) * (int64_t)m + r)]);
  float l = 0.f, acc = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const int64_t pr = ((b * splits + sp) * 2 + x) * (int64_t)m + r;
    const float ms = ml_part[2 * pr];
    if (ms == -INFINITY) continue;
    const float w = exp2f(ms - mx);
    l = fmaf(w, ml_part[2 * pr + 1], l);
    acc = fmaf(w, o_part[pr * kD + col], acc);
  }
  __nv_bfloat16* dst = x ? out_base : out_dense;
  dst[(b * m + r) * kD + col] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
}

template <int MODE>
static int launch_attn(dim3 grid, const void* q, const void* k, const void* v, const int32_t* q_offsets,
                       const int32_t* k_offsets, const int32_t* sel_ids, const int32_t* sel_counts,
                       const int32_t* tile_start, int64_t nq, int64_t nk, int d, int cq, int ck,
                       const int32_t* q_order, void* out, int* err, const AttnRepair& rep, const AttnProbe& prb,
                       cudaStream_t st) {
  const cudaError_t e =
      cudaFuncSetAttribute(block_sparse_attn_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
  if (e != cudaSuccess)
    return fail(SPR_ERR_LAUNCH, "block-sparse attention: shared-memory opt-in (%d B): %s", kSmemTc,
                cudaGetErrorString(e));
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)d);
  block_sparse_attn_tc_kernel<MODE><<<grid, kThreadsTc, kSmemTc, st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, q_offsets, k_offsets, sel_ids,
      sel_counts, tile_start, nq, nk, cq, ck, q_order, (__nv_bfloat16*)out, scale_log2, err, rep, prb);
  return check_launch(MODE == kModeProbe ? "probe rows attention" : "block-sparse attention");
}
}  // namespace spr

using namespace spr;

static size_t repair_fold_floats(int64_t bh) { return (size_t)bh * (kRepairImageBytes / 4 + kRepairRank); }

extern "C" size_t spr_block_sparse_attn_workspace_bytes(int64_t bh, int64_t nq, int cq) {
  (void)nq;
  return 256 + align_up((size_t)bh * (cq + 1) * sizeof(int32_t), 256) + 256 +
         align_up(repair_fold_floats(bh) * sizeof(float), 256) + 256;
}

extern "C" int spr_block_sparse_attn(const void* q_perm, const void* k_perm, const void* v_perm,
                                     const int32_t* q_offsets, const int32_t* k_offsets, const int32_t* sel_ids,
                                     const int32_t* sel_counts, int64_t bh, int64_t nq, int64_t nk, int d, int cq,
                                     int ck, const int32_t* q_order, const SprRepairState* repair, void* out,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (d != kD) return fail(SPR_ERR_SHAPE, "block-sparse attention requires d=128, got %d", d);
  if (ck > kMaxRuns) return fail(SPR_ERR_SHAPE, "block-sparse attention: ck=%d exceeds %d", ck, kMaxRuns);
  if (bh <= 0 || nq <= 0 || nk <= 0 || cq <= 0 || ck <= 0 || bh > 65535 || nq > INT32_MAX || nk > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "block-sparse attention: bad shape");
  if (!aligned(q_perm, 16) || !aligned(k_perm, 16) || !aligned(v_perm, 16) || !aligned(out, 16))
    return fail(SPR_ERR_ALIGN, "block-sparse attention: 16-byte alignment required");
  if (repair) {
    if (repair->rank != kRepairRank)
      return fail(SPR_ERR_SHAPE, "fused repair: rank %d unsupported (16)", repair->rank);
    if (ck > kMaxRunsRepair)
      return fail(SPR_ERR_SHAPE, "fused repair: ck=%d exceeds %d", ck, kMaxRunsRepair);
    if (repair->m < 0 || repair->m > kMaxProbes || (repair->m > 0 && (!repair->probe_rows || !repair->probe_dense)))
      return fail(SPR_ERR_SHAPE, "fused repair: m=%d probe rows (0..%d, rows and dense rows given)", repair->m,
                  kMaxProbes);
    if (!repair->x_mean || !repair->x_scale || !repair->y_mean || !repair->left || !repair->basis)
      return fail(SPR_ERR_ARG, "fused repair: null state tensor");
    if (repair->m > 0 && !aligned(repair->probe_dense, 16))
      return fail(SPR_ERR_ALIGN, "fused repair: dense probe rows must be 16-byte aligned");
  }
  Carver cv(workspace, workspace_bytes);
  int* err = cv.take<int>(64);
  int32_t* tile_start = cv.take<int32_t>((size_t)bh * (cq + 1));
  float* fold = cv.take<float>(repair_fold_floats(bh));
  if (!workspace || !cv.ok())
    return fail(SPR_ERR_WORKSPACE, "block-sparse attention: workspace %zu < %zu", workspace_bytes, cv.off);
  cudaStream_t st = (cudaStream_t)stream;
  tile_table_kernel<<<(unsigned)bh, 32, 0, st>>>(q_offsets, cq, tile_start, err);
  int s = check_launch("attention tile table");
  if (s) return s;
  // Upper bound on 256-row units per problem: every cluster may add one partial unit.
  const int64_t max_tiles = (nq + kPairRows - 1) / kPairRows + cq;
  const dim3 grid((unsigned)max_tiles, (unsigned)bh);
  AttnProbe prb{};
  AttnRepair rep{};
  if (!repair)
    return launch_attn<kModePlain>(grid, q_perm, k_perm, v_perm, q_offsets, k_offsets, sel_ids, sel_counts,
                                   tile_start, nq, nk, d, cq, ck, q_order, out, err, rep, prb, st);
  uint8_t* image = reinterpret_cast<uint8_t*>(fold);
  float* c0 = fold + (size_t)bh * (kRepairImageBytes / 4);
  repair_fold_kernel<<<(unsigned)bh, 256, 0, st>>>(repair->x_mean, repair->x_scale, repair->left, repair->basis,
                                                   image, c0);
  if ((s = check_launch("fused repair: fold"))) return s;
  rep.image = image;
  rep.c0 = c0;
  rep.y_mean = repair->y_mean;
  rep.probe_tok = repair->probe_rows;
  rep.probe_dense = (const __nv_bfloat16*)repair->probe_dense;
  rep.m = repair->m;
  rep.alpha = repair->alpha;
  return launch_attn<kModeRepair>(grid, q_perm, k_perm, v_perm, q_offsets, k_offsets, sel_ids, sel_counts,
                                  tile_start, nq, nk, d, cq, ck, q_order, out, err, rep, prb, st);
}

// Key splits of the probe pre-pass: about two CTAs per SM over all problems,
// at most 16 per problem and at least 4 key tiles per split.
static int probe_splits(int64_t bh, int64_t nk) {
  const int64_t tiles = (nk + kTileN - 1) / kTileN;
  int64_t sp = std::max<int64_t>(1, (2 * 148) / bh);
  sp = std::min<int64_t>(sp, 16);
  sp = std::min<int64_t>(sp, std::max<int64_t>(1, tiles / 4));
  return (int)sp;
}

extern "C" size_t spr_probe_rows_attn_workspace_bytes(int64_t bh, int64_t nk, int m) {
  const size_t part = (size_t)bh * probe_splits(bh, nk) * 2 * (size_t)m;
  return 256 + align_up(part * kD * sizeof(float), 256) + align_up(part * 2 * sizeof(float), 256) + 256;
}

extern "C" int spr_probe_rows_attn(const void* q, const void* k_perm, const void* v_perm, const int32_t* k_offsets,
                                   const uint8_t* routed, const int32_t* rows, const int32_t* row_cluster,
                                   int64_t bh, int64_t n, int64_t nk, int d, int cq, int ck, int m, void* out_dense,
                                   void* out_base, void* workspace, size_t workspace_bytes, void* stream) {
  if (d != kD) return fail(SPR_ERR_SHAPE, "probe rows attention requires d=128, got %d", d);
  if (bh <= 0 || n <= 0 || nk <= 0 || cq <= 0 || ck <= 0 || bh > 65535 || n > INT32_MAX || nk > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "probe rows attention: bad shape");
  if (m <= 0 || m > kTileM) return fail(SPR_ERR_SHAPE, "probe rows attention: m=%d must be in [1,%d]", m, kTileM);
  if (!aligned(q, 16) || !aligned(k_perm, 16) || !aligned(v_perm, 16) || !aligned(out_dense, 16) ||
      !aligned(out_base, 16))
    return fail(SPR_ERR_ALIGN, "probe rows attention: 16-byte alignment required");
  const int splits = probe_splits(bh, nk);
  const size_t part = (size_t)bh * splits * 2 * (size_t)m;
  Carver cv(workspace, workspace_bytes);
  int* err = cv.take<int>(64);
  float* o_part = cv.take<float>(part * kD);
  float* ml_part = cv.take<float>(part * 2);
  if (!workspace || !cv.ok())
    return fail(SPR_ERR_WORKSPACE, "probe rows attention: workspace %zu < %zu", workspace_bytes, cv.off);
  cudaStream_t st = (cudaStream_t)stream;
  cudaMemsetAsync(err, 0, sizeof(int), st);
  AttnProbe prb{rows, row_cluster, routed, o_part, ml_part, m, splits};
  AttnRepair rep{};
  int s = launch_attn<kModeProbe>(dim3((unsigned)splits, (unsigned)bh), q, k_perm, v_perm, nullptr, k_offsets,
                                  nullptr, nullptr, nullptr, n, nk, d, cq, ck, nullptr, nullptr, err, rep, prb, st);
  if (s) return s;
  probe_merge_kernel<<<dim3((unsigned)m, 2, (unsigned)bh), kD, 0, st>>>(o_part, ml_part, splits, m,
                                                                       (__nv_bfloat16*)out_dense,
                                                                       (__nv_bfloat16*)out_base);
  return check_launch("probe rows attention: merge");
}

// ---------------------------------------------------------------------------
// No-allocation variant.  Some callers cannot allocate device memory at all:
// a host framework that hands every byte of HBM to its own pool and forbids
// other allocations, or a latency-critical loop that may not call cudaMalloc
// (it can synchronise the whole device) and has no buffer to lend as a
// workspace.  For them the attention call below keeps its scratch (the status
// word and the per-problem tile table) in a fixed array in device memory that
// the library owns.
//
// The array is `static __device__`: every GPU that loads this library holds
// its 256 KiB + 256 B until the process exits.  In host code its name is only
// a host-side stand-in for the symbol, not a device address, so on every call
// the host asks the runtime for the real address on the current device
// (cudaGetSymbolAddress) and passes that pointer to the kernels.  The status
// word of the last call (0 = ok, else the bounded wait that gave up) is read
// back with spr_block_sparse_attn_noalloc_status.
// ---------------------------------------------------------------------------
namespace spr {
constexpr int kNoAllocStatusInts = 64;       // status word + padding (keeps the table 256-byte aligned)
constexpr int kNoAllocTableInts = 65536;     // maximum bh * (cq + 1)
static __device__ __align__(256) int32_t g_attn_noalloc_scratch[kNoAllocStatusInts + kNoAllocTableInts];

// Device address of the scratch array on the current device, looked up on
// every call (cheap next to the launches) so that a context created again
// after cudaDeviceReset never sees a stale address.
static int noalloc_scratch(int32_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return fail(SPR_ERR_LAUNCH, "no-alloc attention: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = static_cast<int32_t*>(p);
  return SPR_OK;
}

}  // namespace spr

extern "C" int spr_block_sparse_attn_noalloc(const void* q_perm, const void* k_perm, const void* v_perm,
                                             const int32_t* q_offsets, const int32_t* k_offsets,
                                             const int32_t* sel_ids, const int32_t* sel_counts, int64_t bh,
                                             int64_t nq, int64_t nk, int d, int cq, int ck, const int32_t* q_order,
                                             void* out, void* stream) {
  if (d != kD) return fail(SPR_ERR_SHAPE, "block-sparse attention requires d=128, got %d", d);
  if (ck > kMaxRuns) return fail(SPR_ERR_SHAPE, "block-sparse attention: ck=%d exceeds %d", ck, kMaxRuns);
  if (bh <= 0 || nq <= 0 || nk <= 0 || cq <= 0 || ck <= 0 || bh > 65535 || nq > INT32_MAX || nk > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "block-sparse attention: bad shape");
  if (bh * (int64_t)(cq + 1) > kNoAllocTableInts)
    return fail(SPR_ERR_SHAPE,
                "no-alloc attention: bh*(cq+1)=%lld exceeds the fixed scratch of %d entries; "
                "use spr_block_sparse_attn with a caller workspace",
                (long long)(bh * (int64_t)(cq + 1)), kNoAllocTableInts);
  if (!aligned(q_perm, 16) || !aligned(k_perm, 16) || !aligned(v_perm, 16) || !aligned(out, 16))
    return fail(SPR_ERR_ALIGN, "block-sparse attention: 16-byte alignment required");
  int32_t* scratch = nullptr;
  int s = noalloc_scratch(&scratch);
  if (s) return s;
  int* err = scratch;                               // zeroed by tile_table_kernel on every call
  int32_t* tile_start = scratch + kNoAllocStatusInts;  // fully rewritten on every call
  cudaStream_t st = (cudaStream_t)stream;
  tile_table_kernel<<<(unsigned)bh, 32, 0, st>>>(q_offsets, cq, tile_start, err);
  if ((s = check_launch("attention tile table"))) return s;
  const int64_t max_tiles = (nq + kPairRows - 1) / kPairRows + cq;
  AttnProbe prb{};
  AttnRepair rep{};
  return launch_attn<kModePlain>(dim3((unsigned)max_tiles, (unsigned)bh), q_perm, k_perm, v_perm, q_offsets,
                                 k_offsets, sel_ids, sel_counts, tile_start, nq, nk, d, cq, ck, q_order, out, err,
                                 rep, prb, st);
}

extern "C" int spr_block_sparse_attn_noalloc_status(int* out) {
  if (!out) return fail(SPR_ERR_ARG, "no-alloc attention status: null output");
  const cudaError_t e = cudaMemcpyFromSymbol(out, g_attn_noalloc_scratch, sizeof(int32_t));
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "no-alloc attention status: %s", cudaGetErrorString(e));
  return SPR_OK;
}
