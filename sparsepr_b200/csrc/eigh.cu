// Batched symmetric eigendecomposition of small matrices (n <= 128, even),
// one CTA per matrix.  n = 64 and 128 (the role-metric factors, 128x128, and
// the repair basis, 64x64 row Gram) take the tridiagonal route
// (sym_eig_tri_kernel: Householder reduction, multisection, twisted
// factorisation, back-transformation, one Newton-Schulz step), optionally
// forming only the top eigenvectors; a matrix it hands back (repeated
// eigenvalues) and every other n use cyclic two-sided Jacobi with a
// round-robin pair ordering (Golub & Van Loan, "Matrix Computations",
// sym.schur2 rotations and the parallel-ordering cyclic Jacobi method).
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
                   int max_sweeps, float rel_tol, int only_flagged) {
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
  // Second pass after sym_eig_tri_kernel: only the matrices it handed back
  // (first eigenvalue set to NaN).  Block-uniform.
  if (only_flagged && !isnan(evals[b * n])) return;
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


// ---------------------------------------------------------------------------
// Tridiagonal route for n = 64, 128 (one CTA of 512 threads per matrix):
//  1. Householder reduction Q^T A Q = T in shared memory (Golub & Van Loan,
//     "Matrix Computations", Algorithm 8.3.1): per column k the reflector
//     v (stored in column k below the diagonal), p = beta A' v,
//     w = p - (beta/2)(p.v) v, A' -= v w^T + w v^T.
//  2. All eigenvalues of T by multisection on the Sturm count (the number of
//     negative pivots of the LDL^T factorisation of T - x I), G = 512/n threads
//     per eigenvalue each testing one of G interior points per round.
//  3. Eigenvectors of T by a twisted factorisation (Dhillon & Parlett): the
//     forward and backward pivots of T - lambda I meet at the index r where
//     |gamma_r| is smallest; x_r = 1 and the two bidiagonal factors propagate x
//     outwards.  One thread per eigenvalue.
//  4. Vectors of eigenvalues closer than 1e-3 ||T|| are re-orthogonalised
//     (classical Gram-Schmidt, twice) in index order.
//  5. V = H_0 H_1 ... H_{n-3} Z.
// A matrix whose vectors collapse in step 4 (repeated eigenvalues) or come out
// non-finite is handed back: its first eigenvalue is written as NaN and the
// Jacobi kernel, launched next with only_flagged = 1, solves it instead.
constexpr int kTriThreads = 512;

template <int N>
__global__ void __launch_bounds__(kTriThreads, 1)
sym_eig_tri_kernel(const float* __restrict__ a_in, float* __restrict__ evals, float* __restrict__ evecs, int top) {
  constexpr int n = N, ld = N + 1, G = kTriThreads / N;  // G: row groups / threads per eigenvalue
  static_assert(G >= 2 && 32 % G == 0, "size not supported");
  extern __shared__ float sh[];
  float* A = sh;            // [n][ld]; reflectors below the diagonal
  float* Z = sh + n * ld;   // [n][ld]; eigenvectors (columns)
  __shared__ float s_d[N], s_e[N], s_e2[N], s_beta[N], s_v[N], s_p[N], s_lam[N];
  __shared__ float s_part[kTriThreads];  // [row group][column] partial sums
  __shared__ float s_scal[4];
  __shared__ int s_bad;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col = tid % N, grp = tid / N;  // column / row-group mapping: conflict-free row accesses
  const float* src = a_in + b * (int64_t)n * n;
  for (int idx = tid; idx < n * n; idx += kTriThreads) {
    const int i = idx / n, j = idx % n;
    A[i * ld + j] = 0.5f * (src[i * n + j] + src[j * n + i]);
  }
  if (tid == 0) s_bad = 0;
  __syncthreads();

  // 1. Householder tridiagonalisation.
  for (int k = 0; k < n - 2; ++k) {
    const int m = n - 1 - k;  // length of the reflector
    if (warp == 0) {
      float sig = 0.f;
      for (int i = 1 + lane; i < m; i += 32) {
        const float x = A[(k + 1 + i) * ld + k];
        sig = fmaf(x, x, sig);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sig += __shfl_xor_sync(0xffffffffu, sig, o);
      if (lane == 0) {
        const float x0 = A[(k + 1) * ld + k];
        float beta = 0.f, v0 = 0.f, alpha = x0;
        if (sig > 0.f) {
          const float nrm = sqrtf(fmaf(x0, x0, sig));
          alpha = x0 >= 0.f ? -nrm : nrm;
          v0 = x0 - alpha;
          beta = 2.f / fmaf(v0, v0, sig);
        }
        s_d[k] = A[k * ld + k];
        s_e[k] = alpha;
        s_beta[k] = beta;
        s_scal[0] = v0;
      }
    }
    __syncthreads();
    const float beta = s_beta[k];
    if (tid < m) {
      const float vi = tid == 0 ? s_scal[0] : A[(k + 1 + tid) * ld + k];
      s_v[tid] = vi;
    }
    __syncthreads();
    if (tid == 0) A[(k + 1) * ld + k] = s_scal[0];  // column k keeps v (rows k+1..)
    if (beta == 0.f) continue;                      // block-uniform: column already reduced
    {  // p = beta A' v as column sums of the symmetric A': row group grp, column col
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      if (col < m) {
        const float* ac = A + (k + 1) * ld + (k + 1 + col);
        int r = grp;
        for (; r + 3 * G < m; r += 4 * G) {
          a0 = fmaf(ac[r * ld], s_v[r], a0);
          a1 = fmaf(ac[(r + G) * ld], s_v[r + G], a1);
          a2 = fmaf(ac[(r + 2 * G) * ld], s_v[r + 2 * G], a2);
          a3 = fmaf(ac[(r + 3 * G) * ld], s_v[r + 3 * G], a3);
        }
        for (; r < m; r += G) a0 = fmaf(ac[r * ld], s_v[r], a0);
      }
      s_part[grp * N + col] = (a0 + a1) + (a2 + a3);
    }
    __syncthreads();
    if (warp == 0) {  // p, then K = (beta/2) p.v
      float kk = 0.f;
      for (int i = lane; i < m; i += 32) {
        float pi = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) pi += s_part[g * N + i];
        pi *= beta;
        s_p[i] = pi;
        kk = fmaf(pi, s_v[i], kk);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kk += __shfl_xor_sync(0xffffffffu, kk, o);
      const float K = 0.5f * beta * kk;
      for (int i = lane; i < m; i += 32) s_p[i] = fmaf(-K, s_v[i], s_p[i]);  // w = p - K v
    }
    __syncthreads();
    {  // A' -= v w^T + w v^T
      if (col < m) {
        const float vc = s_v[col], wc = s_p[col];
        float* ac = A + (k + 1) * ld + (k + 1 + col);
#pragma unroll 4
        for (int r = grp; r < m; r += G) ac[r * ld] = fmaf(-s_v[r], wc, fmaf(-s_p[r], vc, ac[r * ld]));
      }
    }
    __syncthreads();
  }
  if (tid == 0) {
    s_d[n - 2] = A[(n - 2) * ld + (n - 2)];
    s_d[n - 1] = A[(n - 1) * ld + (n - 1)];
    s_e[n - 2] = A[(n - 1) * ld + (n - 2)];
    s_e[n - 1] = 0.f;
    s_beta[n - 2] = 0.f;
  }
  __syncthreads();
  if (tid < n) s_e2[tid] = s_e[tid] * s_e[tid];
  if (warp == 0) {  // Gershgorin interval and ||T||
    float lo = INFINITY, hi = -INFINITY, e2max = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float r = fabsf(s_e[i]) + (i > 0 ? fabsf(s_e[i - 1]) : 0.f);
      lo = fminf(lo, s_d[i] - r);
      hi = fmaxf(hi, s_d[i] + r);
      e2max = fmaxf(e2max, s_e[i] * s_e[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
      e2max = fmaxf(e2max, __shfl_xor_sync(0xffffffffu, e2max, o));
    }
    if (lane == 0) {
      const float tn = fmaxf(fabsf(lo), fabsf(hi));
      const float pad = 2.f * 1.2e-7f * tn * n + 1e-30f;
      s_scal[0] = lo - pad;
      s_scal[1] = hi + pad;
      s_scal[2] = tn;
      s_scal[3] = fmaxf(1e-30f, 1e-30f * e2max);  // pivmin
    }
  }
  __syncthreads();
  const float tnorm = s_scal[2], pivmin = s_scal[3];

  // 2. Eigenvalue j (ascending) by multisection: G consecutive lanes per eigenvalue.
  {
    const int j = tid / G, t = tid % G;
    float a = s_scal[0], bnd = s_scal[1];
    const unsigned gmask = ((1u << G) - 1u) << ((lane / G) * G);
    const float atol = 2.4e-7f * tnorm;
    // Each thread tests two interior points (2G per round, two independent
    // Sturm chains): points x_u = a + (b - a)(u + 1)/(2G + 1), u = t and G + t.
    for (int round = 0; round < 64; ++round) {
      if (bnd - a <= fmaxf(atol, 1.2e-7f * fmaxf(fabsf(a), fabsf(bnd)))) break;  // group-uniform
      const float h = (bnd - a) / (float)(2 * G + 1);
      const float x0 = a + h * (float)(t + 1), x1 = a + h * (float)(G + t + 1);
      float q0 = s_d[0] - x0, q1 = s_d[0] - x1;
      int c0 = q0 < 0.f, c1 = q1 < 0.f;
      for (int i = 1; i < n; ++i) {
        if (fabsf(q0) < pivmin) q0 = -pivmin;
        if (fabsf(q1) < pivmin) q1 = -pivmin;
        const float e2 = s_e2[i - 1], di = s_d[i];
        q0 = (di - x0) - __fdividef(e2, q0);
        q1 = (di - x1) - __fdividef(e2, q1);
        c0 += q0 < 0.f;
        c1 += q1 < 0.f;
      }
      const int base = (lane / G) * G;
      const int nb = __popc(__ballot_sync(gmask, c0 <= j) & gmask) + __popc(__ballot_sync(gmask, c1 <= j) & gmask);
      // Points left of lambda_j: u < nb.  New bracket [x_{nb-1}, x_{nb}].
      const int ua = nb - 1, ub = nb;
      const float xa = __shfl_sync(gmask, ua >= G ? x1 : x0, base + (ua >= G ? ua - G : max(ua, 0)));
      const float xb = __shfl_sync(gmask, ub >= G ? x1 : x0, base + (ub >= G ? min(ub - G, G - 1) : ub));
      if (nb > 0) a = xa;
      if (nb < 2 * G) bnd = xb;
    }
    if (t == 0) s_lam[j] = 0.5f * (a + bnd);
  }
  __syncthreads();

  // 3. Eigenvector of T for lambda_j (thread j), written to column j of Z;
  // only the `top` largest (columns n-top .. n-1) when fewer are wanted.
  const int jlo = n - top;
  if (tid >= jlo && tid < n) {
    const int j = tid;
    const float lam = s_lam[j];
    float lp[N], um[N], dpv[N];
    float dp = s_d[0] - lam;
    for (int i = 0; i < n - 1; ++i) {
      if (fabsf(dp) < pivmin) dp = -pivmin;
      dpv[i] = dp;
      lp[i] = s_e[i] / dp;
      dp = (s_d[i + 1] - lam) - lp[i] * s_e[i];
    }
    if (fabsf(dp) < pivmin) dp = -pivmin;
    dpv[n - 1] = dp;
    float dm = s_d[n - 1] - lam;
    if (fabsf(dm) < pivmin) dm = -pivmin;
    float best = fabsf(dpv[n - 1]);
    int r = n - 1;
    for (int i = n - 2; i >= 0; --i) {
      um[i] = s_e[i] / dm;
      dm = (s_d[i] - lam) - um[i] * s_e[i];
      if (fabsf(dm) < pivmin) dm = -pivmin;
      const float g = fabsf(dpv[i] + dm - (s_d[i] - lam));
      if (g < best) { best = g; r = i; }
    }
    float x = 1.f, nrm2 = 1.f;
    Z[r * ld + j] = 1.f;
    for (int i = r - 1; i >= 0; --i) {
      x = -lp[i] * x;
      Z[i * ld + j] = x;
      nrm2 = fmaf(x, x, nrm2);
    }
    x = 1.f;
    for (int i = r; i < n - 1; ++i) {
      x = -um[i] * x;
      Z[(i + 1) * ld + j] = x;
      nrm2 = fmaf(x, x, nrm2);
    }
    const float inv = rsqrtf(nrm2);
    if (!(inv > 0.f) || !isfinite(inv)) s_bad = 1;
    for (int i = 0; i < n; ++i) Z[i * ld + j] *= inv;
  }
  __syncthreads();

  // 4. Re-orthogonalise groups of (nearly) repeated eigenvalues (block-uniform
  // loops); a vector that collapses into its group hands the matrix back.
  {
    const float gtol = fmaxf(1e-5f * tnorm, 4.f * pivmin);  // (near-)repeated eigenvalues only
    int g0 = jlo;
    while (g0 < n) {
      int g1 = g0 + 1;
      while (g1 < n && s_lam[g1] - s_lam[g1 - 1] <= gtol) ++g1;
      for (int j = g0 + 1; j < g1; ++j) {
        for (int pass = 0; pass < 2; ++pass) {
          // dots with the earlier members: one warp per member
          for (int i = g0 + warp; i < j; i += kTriThreads / 32) {
            float dt = 0.f;
            for (int rr = lane; rr < n; rr += 32) dt = fmaf(Z[rr * ld + i], Z[rr * ld + j], dt);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dt += __shfl_xor_sync(0xffffffffu, dt, o);
            if (lane == 0) s_p[i] = dt;
          }
          __syncthreads();
          if (tid < n) {
            float z = Z[tid * ld + j];
            for (int i = g0; i < j; ++i) z = fmaf(-s_p[i], Z[tid * ld + i], z);
            Z[tid * ld + j] = z;
          }
          __syncthreads();
          if (warp == 0) {
            float nn = 0.f;
            for (int rr = lane; rr < n; rr += 32) nn = fmaf(Z[rr * ld + j], Z[rr * ld + j], nn);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) nn += __shfl_xor_sync(0xffffffffu, nn, o);
            if (lane == 0) {
              if (pass == 0 && nn < 0.25f) s_bad = 1;  // the vector collapsed into its neighbours
              s_scal[0] = nn > 0.f ? rsqrtf(nn) : 0.f;
            }
          }
          __syncthreads();
          if (tid < n) Z[tid * ld + j] *= s_scal[0];
          __syncthreads();
        }
      }
      g0 = g1;
    }
  }

  // 5. Back-transformation Z <- H_k Z, k = n-3 .. 0 (H_k acts on rows k+1..).
  for (int k = n - 3; k >= 0; --k) {
    const float beta = s_beta[k];
    if (beta == 0.f) continue;  // block-uniform
    const int m = n - 1 - k;
    if (col >= jlo) {  // y_col = v . Z[k+1.., col]: row group grp
      const float* vk = A + (k + 1) * ld + k;
      const float* zc = Z + (k + 1) * ld + col;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int i = grp;
      for (; i + 3 * G < m; i += 4 * G) {
        a0 = fmaf(vk[i * ld], zc[i * ld], a0);
        a1 = fmaf(vk[(i + G) * ld], zc[(i + G) * ld], a1);
        a2 = fmaf(vk[(i + 2 * G) * ld], zc[(i + 2 * G) * ld], a2);
        a3 = fmaf(vk[(i + 3 * G) * ld], zc[(i + 3 * G) * ld], a3);
      }
      for (; i < m; i += G) a0 = fmaf(vk[i * ld], zc[i * ld], a0);
      s_part[grp * N + col] = (a0 + a1) + (a2 + a3);
    }
    __syncthreads();
    if (col >= jlo) {
      float y = 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) y += s_part[g * N + col];
      y *= beta;
      const float* vk = A + (k + 1) * ld + k;
      float* zc = Z + (k + 1) * ld + col;
#pragma unroll 4
      for (int i = grp; i < m; i += G) zc[i * ld] = fmaf(-vk[i * ld], y, zc[i * ld]);
    }
    __syncthreads();
  }

  // 6. One Newton-Schulz step towards the nearest orthogonal matrix,
  // Z <- Z (3I - Z^T Z) / 2: an orthogonality error E becomes O(E^2).  The
  // reflectors are no longer needed, so A holds C = (3I - Z^T Z) / 2.
  if (top < n) {
    // Only the top columns: C = (3I - Zt^T Zt)/2 (top x top) in A, then Zt C.
    for (int idx = tid; idx < top * top; idx += kTriThreads) {
      const int i = idx / top, j = idx % top;
      float g = 0.f;
      for (int r = 0; r < n; ++r) g = fmaf(Z[r * ld + jlo + i], Z[r * ld + jlo + j], g);
      A[i * ld + j] = (i == j ? 1.5f : 0.f) - 0.5f * g;
    }
    __syncthreads();
    float nz[(N * N + kTriThreads - 1) / kTriThreads];
    int cnt = 0;
    for (int idx = tid; idx < n * top; idx += kTriThreads, ++cnt) {
      const int r = idx / top, j = idx % top;
      float acc = 0.f;
      for (int c = 0; c < top; ++c) acc = fmaf(Z[r * ld + jlo + c], A[c * ld + j], acc);
      nz[cnt] = acc;
    }
    __syncthreads();
    cnt = 0;
    for (int idx = tid; idx < n * top; idx += kTriThreads, ++cnt) Z[(idx / top) * ld + jlo + idx % top] = nz[cnt];
  } else {
    // Register tiles: thread (ib, jb) = (warp * 2 + lane / 16, lane % 16) owns
    // rows ib + 32v (v < n/32) and columns jb + 16u (u < n/16); for a fixed u
    // a half-warp reads 16 consecutive columns, the other operand is a broadcast.
    constexpr int VI = N / 32, UJ = N / 16;
    const int ib = warp * 2 + (lane >> 4), jb = lane & 15;
    float acc[VI][UJ];
#pragma unroll
    for (int v = 0; v < VI; ++v)
#pragma unroll
      for (int u = 0; u < UJ; ++u) acc[v][u] = 0.f;
    if (ib < 32) {
      for (int r = 0; r < n; ++r) {  // Z^T Z
        float zi[VI], zj[UJ];
#pragma unroll
        for (int v = 0; v < VI; ++v) zi[v] = Z[r * ld + ib + 32 * v];
#pragma unroll
        for (int u = 0; u < UJ; ++u) zj[u] = Z[r * ld + jb + 16 * u];
#pragma unroll
        for (int v = 0; v < VI; ++v)
#pragma unroll
          for (int u = 0; u < UJ; ++u) acc[v][u] = fmaf(zi[v], zj[u], acc[v][u]);
      }
#pragma unroll
      for (int v = 0; v < VI; ++v)
#pragma unroll
        for (int u = 0; u < UJ; ++u) {
          const int i = ib + 32 * v, j = jb + 16 * u;
          A[i * ld + j] = (i == j ? 1.5f : 0.f) - 0.5f * acc[v][u];
        }
    }
    __syncthreads();
#pragma unroll
    for (int v = 0; v < VI; ++v)
#pragma unroll
      for (int u = 0; u < UJ; ++u) acc[v][u] = 0.f;
    if (ib < 32) {
      for (int c = 0; c < n; ++c) {  // Z C
        float zr[VI], cj[UJ];
#pragma unroll
        for (int v = 0; v < VI; ++v) zr[v] = Z[(ib + 32 * v) * ld + c];
#pragma unroll
        for (int u = 0; u < UJ; ++u) cj[u] = A[c * ld + jb + 16 * u];
#pragma unroll
        for (int v = 0; v < VI; ++v)
#pragma unroll
          for (int u = 0; u < UJ; ++u) acc[v][u] = fmaf(zr[v], cj[u], acc[v][u]);
      }
    }
    __syncthreads();  // every thread has read the old Z
    if (ib < 32) {
#pragma unroll
      for (int v = 0; v < VI; ++v)
#pragma unroll
        for (int u = 0; u < UJ; ++u) Z[(ib + 32 * v) * ld + jb + 16 * u] = acc[v][u];
    }
  }
  __syncthreads();

  float* ev = evals + b * n;
  float* out = evecs + b * (int64_t)n * n;
  const bool bad = s_bad != 0;
  for (int idx = tid; idx < n * n; idx += kTriThreads) {
    const int i = idx / n, j = idx % n;
    out[i * n + j] = j >= jlo ? Z[i * ld + j] : 0.f;
  }
  if (tid < n) ev[tid] = (bad && tid == 0) ? __int_as_float(0x7fc00000) : s_lam[tid];
}

}  // namespace spr

using namespace spr;

static int sym_eig_launch(const float* a, int64_t batch, int n, int top, int max_sweeps, float* evals,
                          float* evecs, void* stream) {
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
    // Tridiagonal route first; the Jacobi kernel then redoes only the matrices
    // it handed back (repeated eigenvalues), in the same stream.
    const int tri_smem = 2 * n * (n + 1) * (int)sizeof(float);
    auto tri = n == 64 ? sym_eig_tri_kernel<64> : sym_eig_tri_kernel<128>;
    cudaError_t e = cudaFuncSetAttribute(tri, cudaFuncAttributeMaxDynamicSharedMemorySize, tri_smem);
    if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "sym_eig: shared-memory opt-in: %s", cudaGetErrorString(e));
    tri<<<(unsigned)batch, kTriThreads, tri_smem, st>>>(a, evals, evecs, top);
    const int big = n * (n + 1) * (int)sizeof(float);
    auto kern = n == 64 ? sym_eig_big_kernel<64> : sym_eig_big_kernel<128>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
    if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "sym_eig: shared-memory opt-in: %s", cudaGetErrorString(e));
    kern<<<(unsigned)batch, kEigBigThreads, big, st>>>(a, evals, evecs, max_sweeps, tol, 1);
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


extern "C" int spr_sym_eig(const float* a, int64_t batch, int n, int max_sweeps, float* evals, float* evecs,
                           void* stream) {
  return sym_eig_launch(a, batch, n, n, max_sweeps, evals, evecs, stream);
}

extern "C" int spr_sym_eig_top(const float* a, int64_t batch, int n, int top, int max_sweeps, float* evals,
                               float* evecs, void* stream) {
  if (top < 1 || top > n) return fail(SPR_ERR_ARG, "sym_eig_top: top=%d must be in [1, n=%d]", top, n);
  return sym_eig_launch(a, batch, n, top, max_sweeps, evals, evecs, stream);
}
