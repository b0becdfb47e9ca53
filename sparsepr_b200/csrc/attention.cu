// Block-sparse flash attention over kept (query-cluster, key-cluster) pairs on
// the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Work unit (one CTA): a 128-row tile of one query cluster of the
// cluster-sorted Q.  Its keys are the concatenated token runs of the selected
// key clusters of the cluster-sorted K/V, consumed in 128-key tiles; only the
// last tile of a cluster can be partial, so masking is a column bound.
//
// Warp roles (256 threads):
//   warps 0-3  softmax: thread t owns query row t (= TMEM lane t).  Loads the
//              S row from TMEM, online softmax in base 2 with a lazily
//              updated running max, writes P (bf16) to tensor memory, rescales
//              the O accumulator in TMEM when the max moves, and finally
//              normalises O and stores the row (through q_order: the inverse
//              permute is fused into the store).
//   warp 4     MMA issuer (one thread): S(j) = Q K_j^T into one of two TMEM S
//              buffers, O += P(j) V_j into the TMEM O accumulator with P read
//              from tensor memory (no shared-memory round trip for P).
//   warps 5-8  loaders: warps 5-6 gather K rows, warps 7-8 V rows, each into
//              its own 2-stage ring with 16-byte cp.async.  K stage j is freed
//              as soon as S(j) is done and V stage j when PV(j) is done, so
//              the gather latency of tile j+2 hides behind the MMAs of tiles
//              j and j+1.  The selected clusters' runs (start, prefix length)
//              are staged in shared memory once per CTA; each loader lane
//              resolves one key slot by binary search, and each warp
//              instruction moves two full 256-byte rows.
// TMEM: columns [0,128) and [128,256) are the two S buffers, [256,384) is O,
// [384,448) is P (bf16 pairs, one 32-bit column per two keys).
// Operand tiles use the canonical 128-byte-swizzled K-major layout; V is the
// MN-major B operand of the PV product.
#include "tc_common.cuh"

namespace spr {

using namespace tc;

constexpr int kD = 128;
constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kSoftmaxThreads = 128;
constexpr int kLoaderThreads = 128;
constexpr int kThreadsTc = 288;
constexpr int kMaxRuns = 2048;  // key clusters per problem (ck) this kernel accepts
constexpr int kTileBytes = kTileM * kD * 2;    // 32 KB per 128 x 128 bf16 tile
constexpr int kSmemTc = 1024 /*align slack*/ + kTileBytes /*Q*/ + 4 * kTileBytes /*K,V x2*/;
constexpr uint32_t kIdescQK = idesc_bf16_f32(128, 128, 0);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, 1);

enum : int { kErrTimeoutLoad = 1, kErrTimeoutMma = 2, kErrTimeoutSoftmax = 3 };

// err[0] = 0, tile_start[b][c] = first 128-row tile of query cluster c in
// problem b (exclusive prefix of ceil(size/128)); tile_start[b][cq] = total.
__global__ void tile_table_kernel(const int32_t* __restrict__ q_offsets, int cq, int32_t* __restrict__ tile_start,
                                  int* __restrict__ err) {
  const int64_t b = blockIdx.x;
  if (threadIdx.x != 0) return;
  if (b == 0) *err = 0;
  int32_t acc = 0;
  for (int c = 0; c < cq; ++c) {
    tile_start[b * (cq + 1) + c] = acc;
    const int32_t sz = q_offsets[b * (cq + 1) + c + 1] - q_offsets[b * (cq + 1) + c];
    acc += (sz + kTileM - 1) / kTileM;
  }
  tile_start[b * (cq + 1) + cq] = acc;
}

__global__ void __launch_bounds__(kThreadsTc, 1)
block_sparse_attn_tc_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const __nv_bfloat16* __restrict__ v, const int32_t* __restrict__ q_offsets,
                            const int32_t* __restrict__ k_offsets, const int32_t* __restrict__ sel_ids,
                            const int32_t* __restrict__ sel_counts, const int32_t* __restrict__ tile_start,
                            int64_t nq, int64_t nk, int cq, int ck, const int32_t* __restrict__ q_order,
                            __nv_bfloat16* __restrict__ out, float scale_log2, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_k_full[2], bar_k_empty[2], bar_v_full[2], bar_v_empty[2], bar_s_full[2], bar_p_full,
      bar_o_done;
  __shared__ uint32_t s_tmem;
  __shared__ int32_t s_run_start[kMaxRuns];
  __shared__ int32_t s_run_end[kMaxRuns + 1];  // inclusive prefix of run lengths
  __shared__ int s_total;

  const int64_t b = blockIdx.y;
  const int tile = blockIdx.x;
  const int32_t* ts = tile_start + b * (cq + 1);
  if (tile >= ts[cq]) return;  // block-uniform, before any barrier or TMEM use
  int lo = 0, hi = cq - 1;     // query cluster owning the tile: last c with ts[c] <= tile
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ts[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int c = lo;
  const int32_t qbeg = q_offsets[b * (cq + 1) + c];
  const int32_t qend = q_offsets[b * (cq + 1) + c + 1];
  const int32_t row0 = qbeg + (tile - ts[c]) * kTileM;
  const int rows = min(kTileM, qend - row0);

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;        // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;    // 2 stages

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* qb = q + b * nq * kD;
  const __nv_bfloat16* kb = k + b * nk * kD;
  const __nv_bfloat16* vb = v + b * nk * kD;
  const int32_t* ids = sel_ids + (b * cq + c) * (int64_t)ck;
  const int nsel = sel_counts[b * cq + c];
  const int32_t* ko = k_offsets + b * (ck + 1);

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_k_full[i], kLoaderThreads / 2);
      mbar_init(&bar_v_full[i], kLoaderThreads / 2);
      mbar_init(&bar_k_empty[i], 1);
      mbar_init(&bar_v_empty[i], 1);
      mbar_init(&bar_s_full[i], 1);
    }
    mbar_init(&bar_p_full, kSoftmaxThreads);
    mbar_init(&bar_o_done, 1);
    mbar_fence_init();
  }
  if (warp == 4) tmem_alloc<512>(&s_tmem);
  if (warp == 5) {  // run table of the selected key clusters: start row and prefix length
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
  // Q tile (all threads), zero rows past the cluster end.
  for (int i = tid; i < kTileM * 16; i += kThreadsTc) {
    const int r = i >> 4, ch = i & 15;
    const bool ok = r < rows;
    cp_async16(smem_addr(sQ) + sw128_off(r, ch, kTileM), qb + (int64_t)(row0 + (ok ? r : 0)) * kD + ch * 8, ok);
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

  if (warp >= 5) {
    // ------------------------------------------------------------ loaders
    const bool is_v = warp >= 7;                 // warps 5-6: K, warps 7-8: V
    const int gw = (warp - 5) & 1;               // rows [64*gw, 64*gw+64) of each key tile
    const __nv_bfloat16* srcb = is_v ? vb : kb;
    uint8_t* ring = is_v ? sV : sK;
    uint64_t* full = is_v ? bar_v_full : bar_k_full;
    uint64_t* empty = is_v ? bar_v_empty : bar_k_empty;
    const int half = lane >> 4, ch = lane & 15;
    // Per-lane run cursors: slot g = j*128 + 64*gw + 32*sub + lane grows by 128
    // per tile, so each cursor only walks forward over the runs it passes.
    int cur[2] = {0, 0};
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      int src[2];
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        const int g = j * kTileN + gw * 64 + sub * 32 + lane;
        src[sub] = -1;
        if (g < total) {
          while (s_run_end[cur[sub]] <= g) ++cur[sub];
          const int prev = cur[sub] > 0 ? s_run_end[cur[sub] - 1] : 0;
          src[sub] = s_run_start[cur[sub]] + (g - prev);
        }
      }
      if (j >= 2) mbar_wait(&empty[st], ((j >> 1) - 1) & 1, err, kErrTimeoutLoad);
      // Swizzled destination of (row r, chunk ch): rows of one warp step differ
      // only in (r & 7), fixed per unrolled iteration.
      const uint32_t dst = smem_addr(ring + st * kTileBytes) + (uint32_t)(ch >> 3) * (kTileN * 128) +
                           (uint32_t)(gw * 64) * 128;
      const __nv_bfloat16* colp = srcb + ch * 8;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
#pragma unroll
        for (int pr = 0; pr < 16; ++pr) {  // two rows per instruction: lanes 0-15 row 2pr, 16-31 row 2pr+1
          const int rl = 2 * pr + half;
          const int rsrc = __shfl_sync(0xffffffffu, src[sub], rl);
          const int rr = sub * 32 + rl;  // row within this warp's 64-row band (band start is 8-aligned)
          const uint32_t o = (uint32_t)rr * 128 + ((uint32_t)((ch & 7) ^ (rr & 7)) << 4);
          cp_async16(dst + o, colp + (uint32_t)max(rsrc, 0) * (uint32_t)kD, rsrc >= 0);
        }
      }
      cp_async_arrive(&full[st]);  // completes when this lane's copies have landed
    }
    cp_async_wait_all();
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t tS[2] = {tmem, tmem + 128};
      const uint32_t tO = tmem + 256, tP = tmem + 384;
      const uint32_t aq = smem_addr(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&bar_k_full[st], (j >> 1) & 1, err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t bk = smem_addr(sK + st * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {  // K-major: 32 B per 16-element step, second half +16 KB
          const uint32_t koff = (kk >> 2) * (kTileM * 128) + (kk & 3) * 32;
          mma_f16(tS[st], sw128_desc(aq + koff, 16, 1024), sw128_desc(bk + koff, 16, 1024), kIdescQK, kk > 0);
        }
        mma_commit(&bar_s_full[st]);
        mma_commit(&bar_k_empty[st]);
        return true;
      };
      bool ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j & 1;
        if (!(ok = mbar_wait(&bar_p_full, j & 1, err, kErrTimeoutMma))) break;
        if (!(ok = mbar_wait(&bar_v_full[st], (j >> 1) & 1, err, kErrTimeoutMma))) break;
        tc_fence_after();
        const uint32_t bv = smem_addr(sV + st * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {  // 16 keys per step
          const uint32_t voff = kk * 2048;  // V is MN-major: 16 rows = 2 x 1024 B
          mma_f16_ts(tO, tP + kk * 8, sw128_desc(bv + voff, kTileN * 128, 1024), kIdescPV,  // 16 keys = 8 columns
                     (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bar_o_done);
        mma_commit(&bar_v_empty[st]);
        if (j + 2 < ntiles) ok = issue_s(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (thread = row)
    const int row = tid;  // TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_s_full[st], (j >> 1) & 1, err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc_fence_after();
      float s[kTileN];
      tmem_ld64(tmem + lane_base + st * 128, s);
      tmem_ld64(tmem + lane_base + st * 128 + 64, s + 64);
      const int valid = total - j * kTileN;
      if (valid < kTileN) {  // only the last tile of a cluster is partial (warp-uniform)
#pragma unroll
        for (int x = 0; x < kTileN; ++x) s[x] = x < valid ? s[x] : -INFINITY;
      }
      float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int x = 4; x < kTileN; x += 4) {
        m4[0] = fmaxf(m4[0], s[x]);
        m4[1] = fmaxf(m4[1], s[x + 1]);
        m4[2] = fmaxf(m4[2], s[x + 2]);
        m4[3] = fmaxf(m4[3], s[x + 3]);
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale_log2;
      // Lazy max: keep the running max unless it grew by more than 8 (base 2).
      float alpha = 1.f;
      if (mx > m_run + 8.f || m_run == -INFINITY) {
        alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - mx);
        m_run = mx;
      }
      const float neg_m = -m_run;
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[kTileN / 2];
#pragma unroll
      for (int x = 0; x < kTileN; x += 2) {
        const float p0 = ex2(fmaf(s[x], scale_log2, neg_m));
        const float p1 = ex2(fmaf(s[x + 1], scale_log2, neg_m));
        sum4[(x >> 1) & 3] += p0 + p1;
        __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
        pk[x >> 1] = *reinterpret_cast<uint32_t*>(&h);
      }
      const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      l_run = l_run * alpha + sum;
      if (j > 0) {
        // PV(j-1) must be complete before O is rescaled and P is overwritten.
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_o_done, (j - 1) & 1, err, kErrTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {  // warp-uniform: TMEM ld/st are warp-collective
          float o[32];
#pragma unroll
          for (int cb = 0; cb < 4; ++cb) {
            tmem_ld32(tmem + lane_base + 256 + cb * 32, o);
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] *= alpha;
            tmem_st32(tmem + lane_base + 256 + cb * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P(j) replaces P(j-1), which PV(j-1) (complete, waited above) has read.
      tmem_st32(tmem + lane_base + 384, reinterpret_cast<const float*>(pk));
      tmem_st32(tmem + lane_base + 384 + 32, reinterpret_cast<const float*>(pk + 32));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full);
    }
    // Epilogue: O / l, bf16, stored through the inverse permutation.
    if (ok && ntiles > 0) ok = mbar_wait(&bar_o_done, (ntiles - 1) & 1, err, kErrTimeoutSoftmax);
    const bool have = __all_sync(0xffffffffu, ok && ntiles > 0);
    tc_fence_after();
    const float inv = (have && l_run > 0.f) ? 1.f / l_run : 0.f;
    const int64_t s_row = row0 + row;
    const int64_t dst = (row < rows) ? (q_order ? (int64_t)q_order[b * nq + s_row] : s_row) : 0;
    uint4* orow = reinterpret_cast<uint4*>(out + (b * nq + dst) * kD);
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      float o[32];
      if (have) {
        tmem_ld32(tmem + lane_base + 256 + cb * 32, o);
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x) o[x] = 0.f;
      }
      if (row < rows) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 h = __floats2bfloat162_rn(o[q4 * 8 + 2 * e] * inv, o[q4 * 8 + 2 * e + 1] * inv);
            w[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          orow[cb * 4 + q4] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

}  // namespace spr

using namespace spr;

extern "C" size_t spr_block_sparse_attn_workspace_bytes(int64_t bh, int64_t nq, int cq) {
  (void)nq;
  return 256 + align_up((size_t)bh * (cq + 1) * sizeof(int32_t), 256) + 256;
}

extern "C" int spr_block_sparse_attn(const void* q_perm, const void* k_perm, const void* v_perm,
                                     const int32_t* q_offsets, const int32_t* k_offsets, const int32_t* sel_ids,
                                     const int32_t* sel_counts, int64_t bh, int64_t nq, int64_t nk, int d, int cq,
                                     int ck, const int32_t* q_order, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (d != kD) return fail(SPR_ERR_SHAPE, "block-sparse attention requires d=128, got %d", d);
  if (ck > kMaxRuns) return fail(SPR_ERR_SHAPE, "block-sparse attention: ck=%d exceeds %d", ck, kMaxRuns);
  if (bh <= 0 || nq <= 0 || nk <= 0 || cq <= 0 || ck <= 0 || bh > 65535 || nq > INT32_MAX || nk > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "block-sparse attention: bad shape");
  if (!aligned(q_perm, 16) || !aligned(k_perm, 16) || !aligned(v_perm, 16) || !aligned(out, 16))
    return fail(SPR_ERR_ALIGN, "block-sparse attention: 16-byte alignment required");
  Carver cv(workspace, workspace_bytes);
  int* err = cv.take<int>(64);
  int32_t* tile_start = cv.take<int32_t>((size_t)bh * (cq + 1));
  if (!workspace || !cv.ok())
    return fail(SPR_ERR_WORKSPACE, "block-sparse attention: workspace %zu < %zu", workspace_bytes, cv.off);
  cudaStream_t st = (cudaStream_t)stream;
  tile_table_kernel<<<(unsigned)bh, 32, 0, st>>>(q_offsets, cq, tile_start, err);
  int s = check_launch("attention tile table");
  if (s) return s;
  cudaFuncSetAttribute(block_sparse_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
  // Upper bound on tiles per problem: every cluster may add one partial tile.
  const int64_t max_tiles = (nq + kTileM - 1) / kTileM + cq;
  dim3 grid((unsigned)max_tiles, (unsigned)bh);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)d);
  block_sparse_attn_tc_kernel<<<grid, kThreadsTc, kSmemTc, st>>>(
      (const __nv_bfloat16*)q_perm, (const __nv_bfloat16*)k_perm, (const __nv_bfloat16*)v_perm, q_offsets, k_offsets,
      sel_ids, sel_counts, tile_start, nq, nk, cq, ck, q_order, (__nv_bfloat16*)out, scale_log2, err);
  return check_launch("block-sparse attention");
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
// a host-side stand-in for the symbol, not a device address, so the host asks
// the runtime for the real address once per device (cudaGetSymbolAddress with
// that device current) and passes that pointer to the kernels.
// ---------------------------------------------------------------------------
#include <mutex>

namespace spr {
constexpr int kNoAllocStatusInts = 64;       // status word + padding (keeps the table 256-byte aligned)
constexpr int kNoAllocTableInts = 65536;     // maximum bh * (cq + 1)
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) int32_t g_attn_noalloc_scratch[kNoAllocStatusInts + kNoAllocTableInts];
static std::mutex g_noalloc_mu;
static int32_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (set up on first use).
static int noalloc_scratch(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "no-alloc attention: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(SPR_ERR_ARG, "no-alloc attention: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(SPR_ERR_LAUNCH, "no-alloc attention: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
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
  cudaFuncSetAttribute(block_sparse_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
  const int64_t max_tiles = (nq + kTileM - 1) / kTileM + cq;
  dim3 grid((unsigned)max_tiles, (unsigned)bh);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)d);
  block_sparse_attn_tc_kernel<<<grid, kThreadsTc, kSmemTc, st>>>(
      (const __nv_bfloat16*)q_perm, (const __nv_bfloat16*)k_perm, (const __nv_bfloat16*)v_perm, q_offsets, k_offsets,
      sel_ids, sel_counts, tile_start, nq, nk, cq, ck, q_order, (__nv_bfloat16*)out, scale_log2, err);
  return check_launch("block-sparse attention (no-alloc)");
}
