// Batched Lloyd k-means: distance/argmin assignment, stable counting sort of
// the labels, segmented (atomic-free) centroid means and an on-device
// convergence flag, so a full k-means run needs no host synchronisation.
#include "common.cuh"
#include "kmeans_assign.cuh"

namespace spr {

constexpr int kSortChunk = 2048;  // tokens per histogram / scatter chunk

// ---------------------------------------------------------------------------
// Stable counting sort of labels.
// ---------------------------------------------------------------------------

// counts[b][chunk][c] = #tokens of cluster c in chunk `chunk` of problem b
// (cluster-contiguous, so the histogram store, the scan and the scatter's
// start loads are coalesced).
__global__ void label_hist_kernel(const int32_t* __restrict__ labels, int64_t n, int k, int nchunks,
                                  int32_t* __restrict__ counts, const int* __restrict__ done) {
  if (done && *done) return;
  extern __shared__ int32_t sh_cnt[];
  const int chunk = blockIdx.x;
  const int64_t b = blockIdx.y;
  for (int c = threadIdx.x; c < k; c += blockDim.x) sh_cnt[c] = 0;
  __syncthreads();
  const int64_t t0 = (int64_t)chunk * kSortChunk;
  const int64_t t1 = min(n, t0 + kSortChunk);
  const int32_t* lab = labels + b * n;
  for (int64_t t = t0 + threadIdx.x; t < t1; t += blockDim.x) atomicAdd(&sh_cnt[lab[t]], 1);
  __syncthreads();
  int32_t* out = counts + (int64_t)b * k * nchunks;
  for (int c = threadIdx.x; c < k; c += blockDim.x) out[(int64_t)chunk * k + c] = sh_cnt[c];
}

// Per problem: sizes, exclusive offsets and per-(cluster, chunk) start positions
// (written back into `counts`).
__global__ void label_scan_kernel(int32_t* __restrict__ counts, int k, int nchunks,
                                  int32_t* __restrict__ sizes, int32_t* __restrict__ offsets,
                                  const int* __restrict__ done) {
  if (done && *done) return;
  __shared__ int32_t sh_part[1024];
  const int64_t b = blockIdx.x;
  int32_t* cnt = counts + b * (int64_t)k * nchunks;
  // Each thread owns a contiguous range of clusters.
  const int per = (k + blockDim.x - 1) / blockDim.x;
  const int c0 = threadIdx.x * per;
  const int c1 = min(k, c0 + per);
  // Chunk counts are read eight at a time into registers before any store,
  // so the loads of a group overlap (a load after a store to the same array
  // would otherwise wait for it).
  constexpr int CB = 8;
  int32_t local = 0;
  for (int c = c0; c < c1; ++c) {
    int32_t s = 0;
    for (int ch0 = 0; ch0 < nchunks; ch0 += CB) {
      int32_t v[CB];
#pragma unroll
      for (int u = 0; u < CB; ++u) v[u] = ch0 + u < nchunks ? cnt[(int64_t)(ch0 + u) * k + c] : 0;
#pragma unroll
      for (int u = 0; u < CB; ++u) {
        if (ch0 + u < nchunks) cnt[(int64_t)(ch0 + u) * k + c] = s;  // exclusive within the cluster
        s += v[u];
      }
    }
    sizes[b * k + c] = s;
    local += s;
  }
  sh_part[threadIdx.x] = local;
  __syncthreads();
  // Inclusive scan of the per-thread totals (Hillis-Steele, blockDim <= 1024).
  for (int off = 1; off < blockDim.x; off <<= 1) {
    int32_t v = threadIdx.x >= off ? sh_part[threadIdx.x - off] : 0;
    __syncthreads();
    sh_part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t base = sh_part[threadIdx.x] - local;
  for (int c = c0; c < c1; ++c) {
    offsets[b * (k + 1) + c] = base;
    for (int ch0 = 0; ch0 < nchunks; ch0 += CB) {
      int32_t v[CB];
#pragma unroll
      for (int u = 0; u < CB; ++u) v[u] = ch0 + u < nchunks ? cnt[(int64_t)(ch0 + u) * k + c] : 0;
#pragma unroll
      for (int u = 0; u < CB; ++u)
        if (ch0 + u < nchunks) cnt[(int64_t)(ch0 + u) * k + c] = v[u] + base;
    }
    base += sizes[b * k + c];
  }
  if (threadIdx.x == blockDim.x - 1) offsets[b * (k + 1) + k] = sh_part[threadIdx.x];
}

// One warp per chunk writes token ids in label order; within a label the
// tokens keep ascending id order (warp match + lane-rank), so the sort is stable.
__global__ void label_scatter_kernel(const int32_t* __restrict__ labels, int64_t n, int k, int nchunks,
                                     const int32_t* __restrict__ starts, int32_t* __restrict__ order,
                                     const int* __restrict__ done) {
  if (done && *done) return;
  extern __shared__ int32_t sh_cur[];
  const int chunk = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int lane = threadIdx.x;
  const int32_t* st = starts + b * (int64_t)k * nchunks;
  for (int c = lane; c < k; c += 32) sh_cur[c] = st[(int64_t)chunk * k + c];
  __syncwarp();
  const int64_t t0 = (int64_t)chunk * kSortChunk;
  const int64_t t1 = min(n, t0 + kSortChunk);
  const int32_t* lab = labels + b * n;
  int32_t* ord = order + b * n;
  const unsigned lt_mask = (1u << lane) - 1u;
  // Labels of eight 32-token steps are loaded before the steps run, so the
  // global-load latency is paid once per eight steps.
  constexpr int PF = 8;
  for (int64_t g0 = t0; g0 < t1; g0 += 32 * PF) {
    int lv[PF];
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int64_t t = g0 + 32 * u + lane;
      lv[u] = t < t1 ? lab[t] : -1 - lane;  // invalid lanes never match a real label
    }
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int64_t t = g0 + 32 * u + lane;
      const bool valid = t < t1;
      const int l = lv[u];
      const unsigned peers = __match_any_sync(0xffffffffu, l);
      const int rank = __popc(peers & lt_mask);
      int pos = 0;
      if (valid) pos = sh_cur[l] + rank;
      __syncwarp();
      if (valid && rank == 0) sh_cur[l] += __popc(peers);
      __syncwarp();
      if (valid) ord[pos] = (int32_t)t;
    }
  }
}

// ---------------------------------------------------------------------------
// Segmented mean over the sorted order (optionally fused with the permute).
// `wpc` warps of one block per cluster (a power of two dividing the block's
// warps); warp w of a cluster takes rows beg + w*rpw + sub + m*(wpc*rpw),
// each lane streaming one 16-byte chunk of a row.  Large clusters thus spread
// their gather over several warps instead of one serial chain, and the
// partial sums are reduced in a fixed order (row groups, then warps), so the
// result does not depend on scheduling.
// ---------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
  }
}

// mode 0: original-space means (fallback or zero for empty clusters).
// mode 1: k-means update: empty -> old centroid (= fallback), shift = max
//         ||new-old||, optional rounding of the new centroid to `round_dtype`.
template <typename T>
__global__ void segmented_mean_kernel(const T* __restrict__ x, const int32_t* __restrict__ order,
                                      const int32_t* __restrict__ offsets, int64_t n, int d, int k,
                                      const float* __restrict__ fallback, float* __restrict__ means,
                                      T* __restrict__ x_perm, int mode, int round_dtype,
                                      float* __restrict__ shift_out, const int* __restrict__ done,
                                      int64_t total, int wpc) {
  if (done && *done) return;  // launch-uniform
  constexpr int E = 16 / sizeof(T);
  extern __shared__ float sh_acc[];  // [warps][d]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int wi = warp & (wpc - 1);  // warp within its cluster
  const int64_t gc = ((int64_t)blockIdx.x * warps + warp) / wpc;
  const bool valid = gc < total;    // warp-uniform; every warp still reaches the block barrier
  const int64_t b = valid ? gc / k : 0;
  const int c = valid ? (int)(gc % k) : 0;
  float* acc_sh = sh_acc + warp * d;
  const int cpr = d / E;                // 16-byte chunks per row
  const int rpw = 32 / cpr;             // rows per warp step
  const int sub = lane / cpr, ch = lane % cpr;
  const bool active = valid && sub < rpw;
  const int32_t beg = valid ? offsets[b * (k + 1) + c] : 0;
  const int32_t end = valid ? offsets[b * (k + 1) + c + 1] : 0;
  const T* xb = x + b * n * d;
  const int32_t* ob = order + b * n;
  float acc[E];
#pragma unroll
  for (int i = 0; i < E; ++i) acc[i] = 0.f;
  if (active) {
    // Four rows per lane group in flight: the indices first, then the rows
    // (the gather is latency-bound), accumulated in token order.
    // The next batch's row indices are loaded while this batch's rows are in
    // flight, so each batch waits for one memory round trip instead of two.
    constexpr int U = 4;
    const int stride = rpw * wpc;
    int32_t tn[U];
    {
      const int32_t s0 = beg + wi * rpw + sub;
#pragma unroll
      for (int u = 0; u < U; ++u) tn[u] = s0 + u * stride < end ? ob[s0 + u * stride] : -1;
    }
    for (int32_t s0 = beg + wi * rpw + sub; s0 < end; s0 += U * stride) {
      int32_t tt[U];
      uint4 vv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) tt[u] = tn[u];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (tt[u] >= 0) vv[u] = reinterpret_cast<const uint4*>(xb + (int64_t)tt[u] * d)[ch];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int32_t s = s0 + U * stride + u * stride;
        tn[u] = s < end ? ob[s] : -1;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (tt[u] < 0) break;
        if (x_perm) reinterpret_cast<uint4*>(x_perm + b * n * d + (int64_t)(s0 + u * stride) * d)[ch] = vv[u];
        float f[E];
        unpack16<T>(vv[u], f);
#pragma unroll
        for (int i = 0; i < E; ++i) acc[i] += f[i];
      }
    }
  }
  // Reduce the rpw row groups of this warp through shared memory in a fixed order.
  for (int i = lane; i < d; i += 32) acc_sh[i] = 0.f;
  __syncwarp();
  for (int g = 0; g < rpw; ++g) {
    if (active && sub == g) {
#pragma unroll
      for (int i = 0; i < E; ++i) acc_sh[ch * E + i] += acc[i];
    }
    __syncwarp();
  }
  if (wpc > 1) __syncthreads();  // block-uniform
  if (!valid || wi != 0) return;
  const int32_t cnt = end - beg;
  float* out = means + (b * k + c) * (int64_t)d;
  float local_shift = 0.f;
  for (int i = lane; i < d; i += 32) {
    float sum = acc_sh[i];
    for (int w = 1; w < wpc; ++w) sum += acc_sh[w * d + i];  // the cluster's warps in order
    float v;
    if (cnt > 0) {
      v = sum / (float)cnt;
    } else {
      v = fallback ? fallback[(b * k + c) * (int64_t)d + i] : 0.f;
    }
    if (mode == 1) {
      if (cnt > 0 && round_dtype == SPR_BF16) v = __bfloat162float(__float2bfloat16(v));
      if (cnt > 0 && round_dtype == SPR_F16) v = __half2float(__float2half(v));
      const float dv = v - fallback[(b * k + c) * (int64_t)d + i];
      local_shift += dv * dv;
    }
    out[i] = v;
  }
  if (mode == 1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local_shift += __shfl_xor_sync(0xffffffffu, local_shift, o);
    if (lane == 0) atomicMax(reinterpret_cast<int*>(shift_out), __float_as_int(sqrtf(local_shift)));
  }
}

// Adopt the new centroids unless the shift fell below tol (then stop).
// Blocks that observe `done` set by block 0 in this same launch only happen
// when the run converged, in which case no copy is wanted anyway.
__global__ void kmeans_finalize_kernel(float* __restrict__ centroids, const float* __restrict__ next,
                                       int64_t count, const float* __restrict__ shift, float tol,
                                       int* __restrict__ done, int32_t* __restrict__ iters_done) {
  if (*done) return;
  const bool conv = *shift < tol;
  if (!conv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
      centroids[i] = next[i];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    iters_done[0] += 1;
    if (conv) *done = 1;
  }
}

}  // namespace spr

using namespace spr;

static int sort_chunks(int64_t n) { return (int)((n + kSortChunk - 1) / kSortChunk); }

// Workspace layout shared by the k-means entry points.
struct KmeansWs {
  int* err;          // device status word of the last call (0 = ok)
  int* done;         // convergence flag
  float* shifts;     // per-iteration max centroid shift
  float* csq;        // |c|^2 per centroid (padded to whole 128-centroid tiles)
  float* xsq;        // |x|^2 per point (fp32 points, register path)
  float* xmax;       // max |x|^2 per problem (TMA path)
  float* bias;       // (B, base) per problem, then centroid-norm scratch (TMA path)
  int32_t* counts;   // per-(cluster, chunk) counts / starts of the label sort
  float* next;       // updated centroids
  float* caug;       // augmented centroid rows of the folded-bias assignment (may be empty)
  __nv_bfloat16* cbf;  // bf16 centroid operands of the bf16 assignment path
};

static KmeansWs carve_kmeans(Carver& c, int64_t bh, int64_t n, int d, int k) {
  KmeansWs w;
  w.err = c.take<int>(16);
  w.done = c.take<int>(4);
  w.shifts = c.take<float>(1024);
  w.csq = c.take<float>(centroid_sq_pad_count(bh, k));
  w.xsq = c.take<float>((size_t)bh * n);
  // xmax and bias are contiguous (5 * bh floats, cleared by one memset).
  w.xmax = c.take<float>((size_t)bh * 5);
  w.bias = w.xmax + bh;
  w.counts = c.take<int32_t>((size_t)bh * k * sort_chunks(n));
  w.next = c.take<float>((size_t)bh * k * d);
  const size_t naug = d > 0 ? centroid_aug_count(bh, d, k) : 0;
  w.caug = naug ? c.take<float>(naug) : nullptr;
  w.cbf = d > 0 ? c.take<__nv_bfloat16>((size_t)bh * k * d) : nullptr;
  return w;
}

extern "C" size_t spr_kmeans_workspace_bytes(int64_t bh, int64_t n, int d, int k) {
  Carver c(nullptr, 0);
  carve_kmeans(c, bh, n, d, k);
  return c.off + 256;
}

static int launch_label_sort(const int32_t* labels, int64_t bh, int64_t n, int k, int32_t* sizes,
                             int32_t* offsets, int32_t* order, int32_t* counts, const int* done,
                             cudaStream_t st) {
  const int nch = sort_chunks(n);
  dim3 grid(nch, (unsigned)bh);
  label_hist_kernel<<<grid, 256, k * sizeof(int32_t), st>>>(labels, n, k, nch, counts, done);
  label_scan_kernel<<<(unsigned)bh, 1024, 0, st>>>(counts, k, nch, sizes, offsets, done);
  label_scatter_kernel<<<grid, 32, k * sizeof(int32_t), st>>>(labels, n, k, nch, counts, order, done);
  return check_launch("label sort");
}

template <typename T>
static int launch_segmented_mean(const T* x, const int32_t* order, const int32_t* offsets, int64_t bh,
                                 int64_t n, int d, int k, const float* fallback, float* means, T* x_perm,
                                 int mode, int round_dtype, float* shift, const int* done, cudaStream_t st) {
  // Warps per cluster: about one per 48 rows of an average cluster, a power of two <= 8.
  const int warps = 8;
  const int64_t avg = n / k;
  int wpc = 1;
  while (wpc < warps && avg >= 48 * 2 * wpc) wpc *= 2;
  const int64_t total = bh * k;
  const int64_t cpb = warps / wpc;  // clusters per block
  dim3 grid((unsigned)((total + cpb - 1) / cpb));
  segmented_mean_kernel<T><<<grid, warps * 32, warps * d * sizeof(float), st>>>(
      x, order, offsets, n, d, k, fallback, means, x_perm, mode, round_dtype, shift, done, total, wpc);
  return check_launch("segmented mean");
}

static int validate_kmeans(int x_dtype, int64_t bh, int64_t n, int d, int k) {
  if (bh <= 0 || n <= 0 || k <= 0 || bh > 65535)
    return fail(SPR_ERR_SHAPE, "k-means: bh=%lld n=%lld k=%d must be positive (bh <= 65535)", (long long)bh,
                (long long)n, k);
  if (n > INT32_MAX) return fail(SPR_ERR_SHAPE, "k-means: n=%lld exceeds int32", (long long)n);
  if (k > 8192) return fail(SPR_ERR_SHAPE, "k-means: k=%d exceeds 8192", k);
  if (x_dtype != SPR_F32 && x_dtype != SPR_BF16 && x_dtype != SPR_F16)
    return fail(SPR_ERR_DTYPE, "k-means: unsupported dtype %d", x_dtype);
  if (!assign_supported_dim(d)) return fail(SPR_ERR_SHAPE, "k-means: d=%d unsupported (multiple of 4, at most 128)", d);
  return SPR_OK;
}

template <typename T>
static int seg_mean_any(int x_dtype, const void* x, const int32_t* order, const int32_t* offsets, int64_t bh,
                        int64_t n, int d, int k, const float* fallback, float* means, void* x_perm, int mode,
                        int round_dtype, float* shift, const int* done, cudaStream_t st) {
  return launch_segmented_mean<T>((const T*)x, order, offsets, bh, n, d, k, fallback, means, (T*)x_perm, mode,
                                  round_dtype, shift, done, st);
}

static int seg_mean_dispatch(int x_dtype, const void* x, const int32_t* order, const int32_t* offsets, int64_t bh,
                             int64_t n, int d, int k, const float* fallback, float* means, void* x_perm, int mode,
                             int round_dtype, float* shift, const int* done, cudaStream_t st) {
  if (x_dtype == SPR_F32)
    return seg_mean_any<float>(x_dtype, x, order, offsets, bh, n, d, k, fallback, means, x_perm, mode, round_dtype,
                               shift, done, st);
  if (x_dtype == SPR_BF16)
    return seg_mean_any<__nv_bfloat16>(x_dtype, x, order, offsets, bh, n, d, k, fallback, means, x_perm, mode,
                                       round_dtype, shift, done, st);
  if (x_dtype == SPR_F16)
    return seg_mean_any<__half>(x_dtype, x, order, offsets, bh, n, d, k, fallback, means, x_perm, mode, round_dtype,
                                shift, done, st);
  return fail(SPR_ERR_DTYPE, "segmented mean: unsupported dtype %d", x_dtype);
}

static int check_kmeans_alignment(const void* x, const float* centroids, const void* workspace) {
  // Rows are read with 8/16-byte vector loads or TMA (d is a multiple of 4);
  // the workspace's |c|^2 tiles are bulk-copied.
  if (!aligned(x, 16) || !aligned(centroids, 16))
    return fail(SPR_ERR_ALIGN, "k-means: x and centroids must be 16-byte aligned");
  if (!aligned(workspace, 16)) return fail(SPR_ERR_ALIGN, "k-means: workspace must be 16-byte aligned");
  return SPR_OK;
}

extern "C" int spr_kmeans_assign(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k,
                                 const float* centroids, int precision, int32_t* labels, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  int s = validate_kmeans(x_dtype, bh, n, d, k);
  if (s) return s;
  if ((s = check_kmeans_alignment(x, centroids, workspace))) return s;
  if (precision != SPR_KMEANS_TF32 && precision != SPR_KMEANS_FP32)
    return fail(SPR_ERR_ARG, "k-means: unknown precision %d", precision);
  Carver c(workspace, workspace_bytes);
  KmeansWs w = carve_kmeans(c, bh, n, d, k);
  if (!c.ok() || !workspace) return fail(SPR_ERR_WORKSPACE, "k-means assign: workspace %zu < %zu", workspace_bytes, c.off);
  cudaStream_t st = (cudaStream_t)stream;
  cudaMemsetAsync(w.err, 0, sizeof(int), st);
  if ((s = launch_point_sq(x, x_dtype, precision, bh, n, d, w.xsq, w.xmax, st))) return s;
  return launch_assign(x, x_dtype, bh, n, d, k, centroids, w.xsq, w.xmax, w.csq, w.bias, w.caug, precision, labels, nullptr, w.err, st);
}

extern "C" int spr_label_sort(const int32_t* labels, int64_t bh, int64_t n, int k, int32_t* sizes,
                              int32_t* offsets, int32_t* order, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (bh <= 0 || n <= 0 || k <= 0 || k > 8192 || bh > 65535) return fail(SPR_ERR_SHAPE, "label sort: bad shape");
  Carver c(workspace, workspace_bytes);
  KmeansWs w = carve_kmeans(c, bh, n, 0, k);
  if (!c.ok() || !workspace)
    return fail(SPR_ERR_WORKSPACE, "label sort: workspace %zu < %zu", workspace_bytes, c.off);
  return launch_label_sort(labels, bh, n, k, sizes, offsets, order, w.counts, nullptr, (cudaStream_t)stream);
}

extern "C" int spr_kmeans_lloyd(const void* x, int x_dtype, int64_t bh, int64_t n, int d, int k, int iters,
                                float tol, int centroid_round_dtype, int precision, float* centroids, int32_t* labels,
                                int32_t* sizes, int32_t* offsets, int32_t* order, int32_t* iters_done,
                                void* workspace, size_t workspace_bytes, void* stream) {
  int s = validate_kmeans(x_dtype, bh, n, d, k);
  if (s) return s;
  if ((s = check_kmeans_alignment(x, centroids, workspace))) return s;
  if (iters < 1 || iters > 1024) return fail(SPR_ERR_ARG, "k-means: iters=%d must be in [1,1024]", iters);
  if (precision != SPR_KMEANS_TF32 && precision != SPR_KMEANS_FP32)
    return fail(SPR_ERR_ARG, "k-means: unknown precision %d", precision);
  cudaStream_t st = (cudaStream_t)stream;
  Carver c(workspace, workspace_bytes);
  KmeansWs w = carve_kmeans(c, bh, n, d, k);
  if (!c.ok() || !workspace) return fail(SPR_ERR_WORKSPACE, "k-means: workspace %zu < %zu", workspace_bytes, c.off);
  int32_t* counts = w.counts;
  float* next = w.next;
  float* shifts = w.shifts;
  int* done = w.done;
  // err, done and shifts are adjacent: one memset clears them.
  cudaMemsetAsync(w.err, 0, (size_t)((char*)(w.shifts + 1024) - (char*)w.err), st);
  cudaMemsetAsync(iters_done, 0, sizeof(int32_t), st);
  const int64_t count = bh * k * (int64_t)d;
  // bf16 points whose centroids are rounded to bf16 after every update (the
  // standalone flash_kmeans contract): bf16 tensor-core distances.
  const bool cbf_ok = x_dtype == SPR_BF16 && centroid_round_dtype == SPR_BF16 && d % 8 == 0;
  if ((s = launch_point_sq(x, x_dtype, precision, bh, n, d, w.xsq, w.xmax, st, cbf_ok))) return s;
  for (int it = 0; it < iters; ++it) {
    if ((s = launch_assign(x, x_dtype, bh, n, d, k, centroids, w.xsq, w.xmax, w.csq, w.bias, w.caug, precision, labels,
                           done, w.err, st, cbf_ok ? w.cbf : nullptr)))
      return s;
    if ((s = launch_label_sort(labels, bh, n, k, sizes, offsets, order, counts, done, st))) return s;
    if ((s = seg_mean_dispatch(x_dtype, x, order, offsets, bh, n, d, k, centroids, next, nullptr, 1,
                               centroid_round_dtype, shifts + it, done, st)))
      return s;
    const int blocks = (int)std::min<int64_t>((count + 255) / 256, 148 * 8);
    kmeans_finalize_kernel<<<blocks, 256, 0, st>>>(centroids, next, count, shifts + it, tol, done, iters_done);
    if ((s = check_launch("k-means finalize"))) return s;
  }
  return SPR_OK;
}

extern "C" int spr_centroid_means(const void* x, int x_dtype, const int32_t* order, const int32_t* offsets,
                                  int64_t bh, int64_t n, int d, int k, const float* fallback, float* means,
                                  void* x_perm, void* stream) {
  if (bh <= 0 || n <= 0 || k <= 0) return fail(SPR_ERR_SHAPE, "centroid means: bad shape");
  const int eb = dtype_bytes(x_dtype);
  if ((d * eb) % 16 != 0 || (d * eb) / 16 > 32)
    return fail(SPR_ERR_SHAPE, "centroid means: row of %d bytes unsupported", d * eb);
  if (!aligned(x, 16) || (x_perm && !aligned(x_perm, 16)))
    return fail(SPR_ERR_ALIGN, "centroid means: rows must be 16-byte aligned");
  return seg_mean_dispatch(x_dtype, x, order, offsets, bh, n, d, k, fallback, means, x_perm, 0, 0, nullptr, nullptr,
                           (cudaStream_t)stream);
}
