// Batched symmetric eigendecomposition of small matrices (n <= 128, even),
// one CTA per matrix, cyclic two-sided Jacobi with a round-robin pair
// ordering (Golub & Van Loan, "Matrix Computations", sym.schur2 rotations and
// the parallel-ordering cyclic Jacobi method).  Used for the role-metric
// factors (128x128) and the repair basis (64x64 row Gram).
//
// Output matches torch.linalg.eigh's convention: eigenvalues ascending,
// eigenvectors in the columns of a row-major [n][n] matrix.
#include "common.cuh"

namespace spr {

constexpr int kEigMax = 128;
constexpr int kEigLd = kEigMax + 1;  // padded row stride: column sweeps are bank-conflict free
constexpr int kEigThreads = 512;

template <int N>
__global__ void __launch_bounds__(kEigThreads)
sym_eig_kernel(const float* __restrict__ a_in, float* __restrict__ evals, float* __restrict__ evecs,
               int max_sweeps, float rel_tol) {
  constexpr int n = N;
  extern __shared__ float sh[];
  float* A = sh;                        // [n][kEigLd]
  float* V = sh + kEigMax * kEigLd;     // [n][kEigLd]
  __shared__ float s_c[kEigMax / 2], s_s[kEigMax / 2];
  __shared__ int s_p[kEigMax / 2], s_q[kEigMax / 2];
  __shared__ int s_rank[kEigMax];
  __shared__ float s_red[kEigThreads / 32][2];
  __shared__ int s_stop;
  const int64_t b = blockIdx.x;
  const float* src = a_in + b * (int64_t)n * n;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    A[i * kEigLd + j] = 0.5f * (src[i * n + j] + src[j * n + i]);
    V[i * kEigLd + j] = i == j ? 1.f : 0.f;
  }
  const int half = n / 2;
  __syncthreads();
  for (int sweep = 0; sweep < max_sweeps; ++sweep) {
    // Convergence test: off-diagonal mass relative to the total.
    float off = 0.f, tot = 0.f;
    for (int idx = tid; idx < n * n; idx += blockDim.x) {
      const int i = idx / n, j = idx % n;
      const float x = A[i * kEigLd + j];
      tot += x * x;
      if (i != j) off += x * x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      off += __shfl_xor_sync(0xffffffffu, off, o);
      tot += __shfl_xor_sync(0xffffffffu, tot, o);
    }
    if ((tid & 31) == 0) { s_red[tid >> 5][0] = off; s_red[tid >> 5][1] = tot; }
    __syncthreads();
    if (tid == 0) {
      float so = 0.f, st = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { so += s_red[w][0]; st += s_red[w][1]; }
      s_stop = so <= rel_tol * rel_tol * st;
    }
    __syncthreads();
    if (s_stop) break;
    for (int round = 0; round < n - 1; ++round) {
      if (tid < half) {
        // Round-robin schedule: slot 0 holds index 0, slot i >= 1 holds
        // 1 + (i - 1 + round) mod (n - 1); pair t is (slot t, slot n-1-t).
        auto slot = [&](int i) { return i == 0 ? 0 : 1 + (i - 1 + round) % (n - 1); };
        int p = slot(tid), q = slot(n - 1 - tid);
        if (p > q) { const int t = p; p = q; q = t; }
        const float apq = A[p * kEigLd + q];
        float c = 1.f, s = 0.f;
        if (fabsf(apq) > 1e-30f) {
          const float tau = (A[q * kEigLd + q] - A[p * kEigLd + p]) / (2.f * apq);
          const float t = copysignf(1.f, tau) / (fabsf(tau) + sqrtf(1.f + tau * tau));
          c = rsqrtf(1.f + t * t);
          s = t * c;
        }
        s_p[tid] = p; s_q[tid] = q; s_c[tid] = c; s_s[tid] = s;
      }
      __syncthreads();
      // Rows: A <- J^T A.
      for (int idx = tid; idx < half * n; idx += blockDim.x) {
        const int pr = idx / n, j = idx % n;
        const int p = s_p[pr], q = s_q[pr];
        const float c = s_c[pr], s = s_s[pr];
        const float ap = A[p * kEigLd + j], aq = A[q * kEigLd + j];
        A[p * kEigLd + j] = c * ap - s * aq;
        A[q * kEigLd + j] = s * ap + c * aq;
      }
      __syncthreads();
      // Columns: A <- A J, V <- V J.
      for (int idx = tid; idx < half * n; idx += blockDim.x) {
        const int pr = idx / n, i = idx % n;
        const int p = s_p[pr], q = s_q[pr];
        const float c = s_c[pr], s = s_s[pr];
        const float ap = A[i * kEigLd + p], aq = A[i * kEigLd + q];
        A[i * kEigLd + p] = c * ap - s * aq;
        A[i * kEigLd + q] = s * ap + c * aq;
        const float vp = V[i * kEigLd + p], vq = V[i * kEigLd + q];
        V[i * kEigLd + p] = c * vp - s * vq;
        V[i * kEigLd + q] = s * vp + c * vq;
      }
      __syncthreads();
    }
  }
  // Ascending order of the diagonal (ties by index), eigenvectors follow.
  for (int j = tid; j < n; j += blockDim.x) {
    const float lj = A[j * kEigLd + j];
    int rank = 0;
    for (int i = 0; i < n; ++i) {
      const float li = A[i * kEigLd + i];
      rank += (li < lj) || (li == lj && i < j);
    }
    evals[b * n + rank] = lj;
    s_rank[j] = rank;
  }
  __syncthreads();
  float* out = evecs + b * (int64_t)n * n;
  for (int idx = tid; idx < n * n; idx += blockDim.x) {
    const int i = idx / n, j = idx % n;
    out[i * n + s_rank[j]] = V[i * kEigLd + j];
  }
}

// Same method for the two large sizes (n = 64, 128), restructured so a round
// is one pass: with the pairs of a round (p_a, q_a) and their rotations J_a,
// the rotated matrix J^T A J restricted to the 2x2 block (a, b) is
// J_a^T A_ab J_b, so each thread rotates whole 2x2 blocks (both sides at
// once; diagonal blocks get their exact zero off-diagonal) and the V columns
// of its pairs in the same phase.  Rotation parameters are packed as one
// float4 {c, s, p, q} per pair.  1024 threads, two barriers per round.  V is
// held in registers (see below), so a round moves only A through shared memory.
constexpr int kEigBigThreads = 1024;

// Packed fp32 pairs (sm_100 f32x2 instructions).
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
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}


template <int N>
__global__ void __launch_bounds__(kEigBigThreads, 1)
sym_eig_big_kernel(const float* __restrict__ a_in, float* __restrict__ evals, float* __restrict__ evecs,
                   int max_sweeps, float rel_tol) {
  constexpr int n = N, half = N / 2, ld = N + 1;
  constexpr int kBlocks = half * half / kEigBigThreads;  // 2x2 blocks per thread
  // V lives in registers: thread = (row, run of kPPL consecutive pairs).
  constexpr int kLanesPerRow = kEigBigThreads / n;  // 8 (n = 128) or 16 (n = 64): one row per lane group
  constexpr int kPPL = half / kLanesPerRow;         // pairs per thread
  static_assert(kBlocks >= 1 && kPPL >= 2 && 32 % kLanesPerRow == 0, "size not supported");
  extern __shared__ float sh[];
  float* A = sh;            // [n][ld]
  // Rotation of pair t at s_rot[t + t/8]: the padding keeps the eight lanes of a
  // row group (reading pairs t0..t0+7, t0 = 8 x lane) on different banks.
  __shared__ float4 s_rot[half + half / 8];
  __shared__ int s_rank[N];
  __shared__ float s_red[kEigBigThreads / 32][2];
  __shared__ int s_stop;
  const int64_t b = blockIdx.x;
  const float* src = a_in + b * (int64_t)n * n;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < n * n; idx += kEigBigThreads) {
    const int i = idx / n, j = idx % n;
    A[i * ld + j] = 0.5f * (src[i * n + j] + src[j * n + i]);
  }
  // Pair t of a round holds the matrix indices at circle positions t and
  // n-1-t; vf/vs are this row's V entries at those two positions.  Round 0
  // has position i = index i, and a full sweep (n-1 rounds) returns there.
  const int vrow = tid / kLanesPerRow, t0 = (tid % kLanesPerRow) * kPPL;
  float vf[kPPL], vs[kPPL];
#pragma unroll
  for (int u = 0; u < kPPL; ++u) {
    vf[u] = vrow == t0 + u ? 1.f : 0.f;
    vs[u] = vrow == n - 1 - (t0 + u) ? 1.f : 0.f;
  }
  __syncthreads();
  for (int sweep = 0; sweep < max_sweeps; ++sweep) {
    float off = 0.f, tot = 0.f;
    for (int idx = tid; idx < n * n; idx += kEigBigThreads) {
      const int i = idx / n, j = idx % n;
      const float x = A[i * ld + j];
      tot += x * x;
      if (i != j) off += x * x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      off += __shfl_xor_sync(0xffffffffu, off, o);
      tot += __shfl_xor_sync(0xffffffffu, tot, o);
    }
    if ((tid & 31) == 0) { s_red[tid >> 5][0] = off; s_red[tid >> 5][1] = tot; }
    __syncthreads();
    if (tid == 0) {
      float so = 0.f, st = 0.f;
      for (int w = 0; w < kEigBigThreads / 32; ++w) { so += s_red[w][0]; st += s_red[w][1]; }
      s_stop = so <= rel_tol * rel_tol * st;
    }
    __syncthreads();
    if (s_stop) break;
    for (int round = 0; round < n - 1; ++round) {
      if (tid < half) {
        // Round-robin schedule: slot 0 holds index 0, slot i >= 1 holds
        // 1 + (i - 1 + round) mod (n - 1); pair t is (slot t, slot n-1-t).
        auto slot = [&](int i) { return i == 0 ? 0 : 1 + (i - 1 + round) % (n - 1); };
        const int f = slot(tid), g = slot(n - 1 - tid);
        const int p = min(f, g), q = max(f, g);
        const float apq = A[p * ld + q];
        float c = 1.f, s = 0.f;
        if (fabsf(apq) > 1e-30f) {
          // Approximate divisions shorten the serial step of the round: the
          // angle only steers convergence, and c, s below stay a consistent
          // rotation (c^2 + s^2 = 1 to rounding) whatever t is.
          const float tau = __fdividef(A[q * ld + q] - A[p * ld + p], 2.f * apq);
          const float t = __fdividef(copysignf(1.f, tau), fabsf(tau) + sqrtf(fmaf(tau, tau, 1.f)));
          c = rsqrtf(1.f + t * t);
          s = t * c;
        }
        // Oriented by circle position: with (first, second) = (f, g) the
        // rotation reads row f <- c row f - s' row g, row g <- s' row f + c row g
        // where s' = s when f is the smaller index and -s otherwise.
        s_rot[tid + (tid >> 3)] = make_float4(c, f == p ? s : -s, __int_as_float(f), __int_as_float(g));
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kBlocks; ++k) {
        const int z = tid + k * kEigBigThreads;
        const int ia = z / half, ib = z % half;
        const float4 ra = s_rot[ia + (ia >> 3)], rb = s_rot[ib + (ib >> 3)];
        const int pa = __float_as_int(ra.z), qa = __float_as_int(ra.w);
        const int pb = __float_as_int(rb.z), qb = __float_as_int(rb.w);
        const float x00 = A[pa * ld + pb], x01 = A[pa * ld + qb], x10 = A[qa * ld + pb], x11 = A[qa * ld + qb];
        // Rows (J_a^T): row p <- c row p - s row q, row q <- s row p + c row q,
        // as packed pairs over the block's two columns.
        const unsigned long long r0 = pk2(x00, x01), r1 = pk2(x10, x11);
        const unsigned long long ca = pk2(ra.x, ra.x), sa = pk2(ra.y, ra.y), nsa = pk2(-ra.y, -ra.y);
        float y00, y01, y10, y11;
        up2(fma2(ca, r0, mul2(nsa, r1)), y00, y01);
        up2(fma2(sa, r0, mul2(ca, r1)), y10, y11);
        // Columns (J_b): the same on columns p, q, packed over each row's pair.
        const unsigned long long cb2 = pk2(rb.x, rb.y), sb2 = pk2(-rb.y, rb.x);  // [c, s], [-s, c]
        float z00, z01, z10, z11;
        up2(fma2(pk2(y00, y00), cb2, mul2(pk2(y01, y01), sb2)), z00, z01);
        up2(fma2(pk2(y10, y10), cb2, mul2(pk2(y11, y11), sb2)), z10, z11);
        if (ia == ib) z01 = z10 = 0.f;  // the rotated pair's own off-diagonal
        A[pa * ld + pb] = z00;
        A[pa * ld + qb] = z01;
        A[qa * ld + pb] = z10;
        A[qa * ld + qb] = z11;
      }
      // V <- V J on this row's pairs (registers), then advance the circle:
      // every position except 0 takes the content of the next position
      // (position i+1 -> i, position 1 -> n-1), a neighbour exchange between
      // consecutive pairs: within the thread or one shuffle away.
#pragma unroll
      for (int u = 0; u < kPPL; ++u) {
        const int t = t0 + u;
        const float4 r = s_rot[t + (t >> 3)];  // oriented: first = position t
        // [first, second] <- first * [c, s] + second * [-s, c]
        up2(fma2(pk2(vf[u], vf[u]), pk2(r.x, r.y), mul2(pk2(vs[u], vs[u]), pk2(-r.y, r.x))), vf[u], vs[u]);
      }
      {
        const float next_first = __shfl_down_sync(0xffffffffu, vf[0], 1);
        const float prev_second = __shfl_up_sync(0xffffffffu, vs[kPPL - 1], 1);
        float nf[kPPL], ns[kPPL];
#pragma unroll
        for (int u = 0; u < kPPL; ++u) {
          const int t = t0 + u;
          nf[u] = t == 0 ? vf[0] : (t == half - 1 ? vs[u] : (u + 1 < kPPL ? vf[u + 1] : next_first));
          ns[u] = t == 0 ? vf[1] : (u > 0 ? vs[u - 1] : prev_second);
        }
#pragma unroll
        for (int u = 0; u < kPPL; ++u) {
          vf[u] = nf[u];
          vs[u] = ns[u];
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < n; j += kEigBigThreads) {
    const float lj = A[j * ld + j];
    int rank = 0;
    for (int i = 0; i < n; ++i) {
      const float li = A[i * ld + i];
      rank += (li < lj) || (li == lj && i < j);
    }
    evals[b * n + rank] = lj;
    s_rank[j] = rank;
  }
  __syncthreads();
  // Whole sweeps only, so positions are back to indices: pair t = (t, n-1-t).
  float* out = evecs + b * (int64_t)n * n;
#pragma unroll
  for (int u = 0; u < kPPL; ++u) {
    out[vrow * n + s_rank[t0 + u]] = vf[u];
    out[vrow * n + s_rank[n - 1 - (t0 + u)]] = vs[u];
  }
}

}  // namespace spr

using namespace spr;

extern "C" int spr_sym_eig(const float* a, int64_t batch, int n, int max_sweeps, float* evals, float* evecs,
                           void* stream) {
  if (batch <= 0 || batch > 65535 || n < 2 || n > kEigMax || (n & 1))
    return fail(SPR_ERR_SHAPE, "sym_eig: need 0 < batch <= 65535 and even 2 <= n <= 128, got batch=%lld n=%d",
                (long long)batch, n);
  if (max_sweeps < 1 || max_sweeps > 64) return fail(SPR_ERR_ARG, "sym_eig: max_sweeps=%d must be in [1,64]", max_sweeps);
  // Stop once the off-diagonal Frobenius mass is below 1e-6 of the total: the
  // level fp32 rotations settle at (a tighter bound is never reached and only
  // adds sweeps).
  const float tol = 1e-6f;
  const int smem = 2 * kEigMax * kEigLd * (int)sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 64 || n == 128) {
    const int big = n * (n + 1) * (int)sizeof(float);
    auto kern = n == 64 ? sym_eig_big_kernel<64> : sym_eig_big_kernel<128>;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
    if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "sym_eig: shared-memory opt-in: %s", cudaGetErrorString(e));
    kern<<<(unsigned)batch, kEigBigThreads, big, st>>>(a, evals, evecs, max_sweeps, tol);
    return check_launch("sym_eig");
  }
  switch (n) {
#define SPR_EIG_CASE(NN)                                                                                      \
  case NN:                                                                                                    \
    cudaFuncSetAttribute(sym_eig_kernel<NN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);             \
    sym_eig_kernel<NN><<<(unsigned)batch, kEigThreads, smem, st>>>(a, evals, evecs, max_sweeps, tol);        \
    return check_launch("sym_eig");
    SPR_EIG_CASE(2) SPR_EIG_CASE(4) SPR_EIG_CASE(8) SPR_EIG_CASE(16) SPR_EIG_CASE(32) SPR_EIG_CASE(48)
    SPR_EIG_CASE(96)
#undef SPR_EIG_CASE
    default:
      return fail(SPR_ERR_SHAPE, "sym_eig: n=%d not compiled (2,4,8,16,32,48,64,96,128)", n);
  }
}

