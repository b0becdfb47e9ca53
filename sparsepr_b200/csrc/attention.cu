// Block-sparse flash attention over kept (query-cluster, key-cluster) pairs.
//
// Work unit: one 64-row tile of one query cluster (rows of the cluster-sorted
// Q).  Its keys are the concatenated token runs of the selected key clusters
// of the cluster-sorted K/V; 64-key tiles are gathered row by row with
// 16-byte cp.async (no index list is materialised), double buffered.
// bf16 tensor-core MMA with fp32 accumulation and an online softmax; the
// output row is stored through the inverse permutation when q_order is given.
#include "common.cuh"

namespace spr {

constexpr int kD = 128;       // head dim
constexpr int kBM = 64;       // query rows per CTA (16 per warp)
constexpr int kBN = 64;       // keys per tile
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunks = kD * 2 / 16;  // 16-byte chunks per row (16)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Swizzled byte offset of (row, 16-byte chunk) in a [rows][128] bf16 tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * (kD * 2) + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// tile_start[b][c] = first 64-row tile of query cluster c in problem b
// (exclusive prefix of ceil(size/64)); tile_start[b][cq] = tiles of b.
__global__ void tile_table_kernel(const int32_t* __restrict__ q_offsets, int cq, int32_t* __restrict__ tile_start) {
  const int64_t b = blockIdx.x;
  if (threadIdx.x != 0) return;
  int32_t acc = 0;
  for (int c = 0; c < cq; ++c) {
    tile_start[b * (cq + 1) + c] = acc;
    const int32_t sz = q_offsets[b * (cq + 1) + c + 1] - q_offsets[b * (cq + 1) + c];
    acc += (sz + kBM - 1) / kBM;
  }
  tile_start[b * (cq + 1) + cq] = acc;
}

__global__ void __launch_bounds__(kThreads, 2)
block_sparse_attn_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                         const __nv_bfloat16* __restrict__ v, const int32_t* __restrict__ q_offsets,
                         const int32_t* __restrict__ k_offsets, const int32_t* __restrict__ sel_ids,
                         const int32_t* __restrict__ sel_counts, const int32_t* __restrict__ tile_start,
                         int64_t nq, int64_t nk, int cq, int ck, const int32_t* __restrict__ q_order,
                         __nv_bfloat16* __restrict__ out, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                          // 64 x 128
  uint8_t* sK = smem + kBM * kD * 2;           // 2 x 64 x 128
  uint8_t* sV = sK + 2 * kBN * kD * 2;         // 2 x 64 x 128
  __shared__ int32_t s_src[2][kBN];
  __shared__ int s_ntiles;

  const int64_t b = blockIdx.y;
  const int tile = blockIdx.x;
  const int32_t* ts = tile_start + b * (cq + 1);
  if (tile >= ts[cq]) return;
  // Query cluster owning this tile: the last c with ts[c] <= tile.
  int lo = 0, hi = cq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ts[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int c = lo;
  const int32_t qbeg = q_offsets[b * (cq + 1) + c];
  const int32_t qend = q_offsets[b * (cq + 1) + c + 1];
  const int32_t row0 = qbeg + (tile - ts[c]) * kBM;
  const int rows = min(kBM, qend - row0);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* qb = q + b * nq * kD;
  const __nv_bfloat16* kb = k + b * nk * kD;
  const __nv_bfloat16* vb = v + b * nk * kD;
  const int32_t* ids = sel_ids + (b * cq + c) * (int64_t)ck;
  const int nsel = sel_counts[b * cq + c];
  const int32_t* ko = k_offsets + b * (ck + 1);

  // Q tile.
  for (int i = tid; i < kBM * kChunks; i += kThreads) {
    const int r = i / kChunks, ch = i % kChunks;
    const bool ok = r < rows;
    cp_async16(smem_u32(sQ + swz(r, ch)), qb + (int64_t)(row0 + (ok ? r : 0)) * kD + ch * 8, ok);
  }
  cp_async_commit();

  // Thread 0 walks the selected runs and publishes each key tile's slot map.
  int cur_pos = 0, cur_off = 0;
  auto build_tile = [&](int buf) {
    int filled = 0;
    while (filled < kBN && cur_pos < nsel) {
      const int kc = ids[cur_pos];
      const int32_t rb = ko[kc], re = ko[kc + 1];
      const int32_t avail = (re - rb) - cur_off;
      if (avail <= 0) { cur_pos++; cur_off = 0; continue; }
      const int take = min(avail, kBN - filled);
      for (int j = 0; j < take; ++j) s_src[buf][filled + j] = rb + cur_off + j;
      filled += take;
      cur_off += take;
    }
    for (int j = filled; j < kBN; ++j) s_src[buf][j] = -1;
  };
  auto issue_kv = [&](int buf) {
    for (int i = tid; i < kBN * kChunks; i += kThreads) {
      const int r = i / kChunks, ch = i % kChunks;
      const int32_t src = s_src[buf][r];
      const bool ok = src >= 0;
      const int64_t off = (int64_t)(ok ? src : 0) * kD + ch * 8;
      cp_async16(smem_u32(sK + buf * kBN * kD * 2 + swz(r, ch)), kb + off, ok);
      cp_async16(smem_u32(sV + buf * kBN * kD * 2 + swz(r, ch)), vb + off, ok);
    }
    cp_async_commit();
  };

  if (tid == 0) {
    int64_t tot = 0;
    for (int i = 0; i < nsel; ++i) tot += ko[ids[i] + 1] - ko[ids[i]];
    s_ntiles = (int)((tot + kBN - 1) / kBN);
    build_tile(0);
  }
  __syncthreads();
  const int ntiles = s_ntiles;
  if (ntiles > 0) issue_kv(0);

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qa[8][4];  // Q fragments for this warp's 16 rows, 8 k-steps of 16
  const int t4 = lane & 3;

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      if (tid == 0) build_tile(buf ^ 1);
      __syncthreads();
      issue_kv(buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sQ + swz(r, ch)), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    const uint8_t* tK = sK + buf * kBN * kD * 2;
    const uint8_t* tV = sV + buf * kBN * kD * 2;
    // S = Q K^T for 16 rows x 64 keys.
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n tiles
        const int r = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(tK + swz(r, ch)), b0, b1, b2, b3);
        mma_bf16(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma_bf16(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
      }
    }
    // Mask invalid key slots, online softmax (base 2).
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * 8 + 2 * t4 + (e & 1);
        float val = s[j][e] * scale_log2;
        if (s_src[buf][key] < 0) val = -INFINITY;
        s[j][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mn = fmaxf(m_r[h], mx[h]);
      alpha[h] = (m_r[h] == -INFINITY) ? 0.f : exp2f(m_r[h] - mn);
      m_r[h] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mref = m_r[e >> 1];
        const float p = (mref == -INFINITY) ? 0.f : exp2f(s[j][e] - mref);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) l_r[h] = l_r[h] * alpha[h] + rs[h];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha[0]; o[j][1] *= alpha[0];
      o[j][2] *= alpha[1]; o[j][3] *= alpha[1];
    }
    // O += P V.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      const uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // pairs of 8-wide d tiles
        const int r = kk * 16 + (((lane >> 3) & 1) << 3) + (lane & 7);
        const int ch = np * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(tV + swz(r, ch)), b0, b1, b2, b3);
        mma_bf16(o[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is refilled in the next iteration
  }

  cp_async_wait<0>();  // the Q group is still pending when the cluster has no keys
  float inv[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float l = l_r[h];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[h] = l > 0.f ? 1.f / l : 0.f;
  }
  const int g = lane >> 2;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = warp * 16 + g + h * 8;
    if (r >= rows) continue;
    const int64_t s_row = row0 + r;
    const int64_t dst = q_order ? (int64_t)q_order[b * nq + s_row] : s_row;
    __nv_bfloat16* orow = out + (b * nq + dst) * kD;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int col = j * 8 + 2 * t4;
      *reinterpret_cast<__nv_bfloat162*>(orow + col) =
          __floats2bfloat162_rn(o[j][2 * h] * inv[h], o[j][2 * h + 1] * inv[h]);
    }
  }
}

}  // namespace spr

using namespace spr;

extern "C" size_t spr_block_sparse_attn_workspace_bytes(int64_t bh, int64_t nq, int cq) {
  (void)nq;
  return align_up((size_t)bh * (cq + 1) * sizeof(int32_t), 256) + 256;
}

extern "C" int spr_block_sparse_attn(const void* q_perm, const void* k_perm, const void* v_perm,
                                     const int32_t* q_offsets, const int32_t* k_offsets, const int32_t* sel_ids,
                                     const int32_t* sel_counts, int64_t bh, int64_t nq, int64_t nk, int d, int cq,
                                     int ck, const int32_t* q_order, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (d != kD) return fail(SPR_ERR_SHAPE, "block-sparse attention requires d=128, got %d", d);
  if (bh <= 0 || nq <= 0 || nk <= 0 || cq <= 0 || ck <= 0 || bh > 65535 || nq > INT32_MAX || nk > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "block-sparse attention: bad shape");
  if (!aligned(q_perm, 16) || !aligned(k_perm, 16) || !aligned(v_perm, 16) || !aligned(out, 16))
    return fail(SPR_ERR_ALIGN, "block-sparse attention: 16-byte alignment required");
  Carver cv(workspace, workspace_bytes);
  int32_t* tile_start = cv.take<int32_t>((size_t)bh * (cq + 1));
  if (!workspace || !cv.ok())
    return fail(SPR_ERR_WORKSPACE, "block-sparse attention: workspace %zu < %zu", workspace_bytes, cv.off);
  cudaStream_t st = (cudaStream_t)stream;
  tile_table_kernel<<<(unsigned)bh, 32, 0, st>>>(q_offsets, cq, tile_start);
  int s = check_launch("attention tile table");
  if (s) return s;
  const int smem = (kBM + 4 * kBN) * kD * 2;
  cudaFuncSetAttribute(block_sparse_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  // Upper bound on tiles per problem: every cluster may add one partial tile.
  const int64_t max_tiles = (nq + kBM - 1) / kBM + cq;
  dim3 grid((unsigned)max_tiles, (unsigned)bh);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)d);
  block_sparse_attn_kernel<<<grid, kThreads, smem, st>>>(
      (const __nv_bfloat16*)q_perm, (const __nv_bfloat16*)k_perm, (const __nv_bfloat16*)v_perm, q_offsets, k_offsets,
      sel_ids, sel_counts, tile_start, nq, nk, cq, ck, q_order, (__nv_bfloat16*)out, scale_log2);
  return check_launch("block-sparse attention");
}
