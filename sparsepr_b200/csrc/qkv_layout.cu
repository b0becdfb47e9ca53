// Wan Q/K/V producer step before SparsePR: full-channel RMSNorm of Q and K
// (one mean of squares over all C = H*D channels of a token), the norm weight,
// rounding to the model dtype, complex RoPE on channel pairs (2i, 2i+1) of
// each head with the token's frequencies, rounding again, and the [B,L,C] ->
// [B,H,L,D] layout change (V: layout only).  Behaviour of the reference's
// wan_qkv_norm_rope_layout (n8_ops.cu:16-105).
//
// HBM-bound: each token row is read twice (the second read hits L1/L2) and
// written once.  One CTA per token; a thread handles 16-byte chunks (8 bf16),
// which never straddle a head because D is a multiple of the chunk.
#include "common.cuh"

namespace spr {

namespace {

constexpr int kQkvThreads = 256;

template <typename T>
struct Vec16 {
  static constexpr int E = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load_f32(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int e = 0; e < Vec16<T>::E; ++e) f[e] = to_f32(h[e]);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

template <typename T>
__global__ void __launch_bounds__(kQkvThreads)
wan_qkv_norm_rope_layout_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                const T* __restrict__ qw, const T* __restrict__ kw,
                                const float* __restrict__ fre, const float* __restrict__ fim, int64_t tokens,
                                int channels, int heads, float eps, T* __restrict__ qo, T* __restrict__ ko,
                                T* __restrict__ vo) {
  constexpr int E = Vec16<T>::E;
  __shared__ float s_red[kQkvThreads / 32][2];
  const int64_t row = blockIdx.x;  // (batch, token)
  const int64_t b = row / tokens, tok = row % tokens;
  const int hd = channels / heads;
  const int nch = channels / E;
  const T* qr = q + row * channels;
  const T* kr = k + row * channels;
  // Pass 1: mean of squares of Q and K over all channels (fp32).
  float sq = 0.f, sk = 0.f;
  for (int c = threadIdx.x; c < nch; c += kQkvThreads) {
    float fq[E], fk[E];
    load_f32(qr + c * E, fq);
    load_f32(kr + c * E, fk);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      sq = fmaf(fq[e], fq[e], sq);
      sk = fmaf(fk[e], fk[e], sk);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_red[threadIdx.x >> 5][0] = sq;
    s_red[threadIdx.x >> 5][1] = sk;
  }
  __syncthreads();
  sq = 0.f;
  sk = 0.f;
#pragma unroll
  for (int w = 0; w < kQkvThreads / 32; ++w) {
    sq += s_red[w][0];
    sk += s_red[w][1];
  }
  const float q_inv = rsqrtf(sq / (float)channels + eps);
  const float k_inv = rsqrtf(sk / (float)channels + eps);
  // Pass 2: norm * weight -> model dtype -> RoPE -> model dtype, BHLD store.
  for (int c = threadIdx.x; c < nch; c += kQkvThreads) {
    const int ch0 = c * E;
    const int head = ch0 / hd, d0 = ch0 % hd;
    const int64_t ob = ((b * heads + head) * tokens + tok) * hd + d0;
    *reinterpret_cast<uint4*>(vo + ob) = *reinterpret_cast<const uint4*>(v + row * channels + ch0);
    float fq[E], fk[E], wq[E], wk[E];
    load_f32(qr + ch0, fq);
    load_f32(kr + ch0, fk);
    load_f32(qw + ch0, wq);
    load_f32(kw + ch0, wk);
    const float* fr = fre + tok * (hd / 2) + d0 / 2;
    const float* fi = fim + tok * (hd / 2) + d0 / 2;
    alignas(16) T oq[E], ok[E];
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      // The normalised value is rounded to the model dtype before RoPE.
      const float q0 = to_f32(from_f32<T>(fq[e] * q_inv * wq[e]));
      const float q1 = to_f32(from_f32<T>(fq[e + 1] * q_inv * wq[e + 1]));
      const float k0 = to_f32(from_f32<T>(fk[e] * k_inv * wk[e]));
      const float k1 = to_f32(from_f32<T>(fk[e + 1] * k_inv * wk[e + 1]));
      const float cr = fr[e / 2], ci = fi[e / 2];
      oq[e] = from_f32<T>(q0 * cr - q1 * ci);
      oq[e + 1] = from_f32<T>(q0 * ci + q1 * cr);
      ok[e] = from_f32<T>(k0 * cr - k1 * ci);
      ok[e + 1] = from_f32<T>(k0 * ci + k1 * cr);
    }
    *reinterpret_cast<uint4*>(qo + ob) = *reinterpret_cast<const uint4*>(oq);
    *reinterpret_cast<uint4*>(ko + ob) = *reinterpret_cast<const uint4*>(ok);
  }
}

template <typename T>
int launch_qkv(const void* q, const void* k, const void* v, const void* qw, const void* kw, const float* fre,
               const float* fim, int64_t batch, int64_t tokens, int channels, int heads, float eps, void* qo,
               void* ko, void* vo, cudaStream_t st) {
  wan_qkv_norm_rope_layout_kernel<T><<<(unsigned)(batch * tokens), kQkvThreads, 0, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)qw, (const T*)kw, fre, fim, tokens, channels, heads, eps,
      (T*)qo, (T*)ko, (T*)vo);
  return check_launch("wan qkv norm/rope/layout");
}

}  // namespace

}  // namespace spr

using namespace spr;

extern "C" int spr_wan_qkv_norm_rope_layout(const void* q, const void* k, const void* v, const void* q_weight,
                                            const void* k_weight, const float* freq_real, const float* freq_imag,
                                            int dtype, int64_t batch, int64_t tokens, int channels, int heads,
                                            float epsilon, void* q_out, void* k_out, void* v_out, void* stream) {
  if (batch <= 0 || tokens <= 0 || channels <= 0 || heads <= 0 || channels % heads)
    return fail(SPR_ERR_SHAPE, "wan qkv: channels=%d must be a positive multiple of heads=%d", channels, heads);
  if (batch * tokens > 0x7fffffffLL) return fail(SPR_ERR_SHAPE, "wan qkv: batch*tokens too large");
  const int eb = dtype == SPR_F32 ? 4 : (dtype == SPR_BF16 || dtype == SPR_F16) ? 2 : 0;
  if (!eb) return fail(SPR_ERR_DTYPE, "wan qkv: unsupported dtype %d", dtype);
  const int hd = channels / heads;
  if (hd % 2 || hd % (16 / eb))
    return fail(SPR_ERR_SHAPE, "wan qkv: head_dim=%d must be even and a multiple of %d", hd, 16 / eb);
  const void* ptrs[] = {q, k, v, q_weight, k_weight, q_out, k_out, v_out};
  for (const void* p : ptrs)
    if (!aligned(p, 16)) return fail(SPR_ERR_ALIGN, "wan qkv: tensors must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == SPR_BF16)
    return launch_qkv<__nv_bfloat16>(q, k, v, q_weight, k_weight, freq_real, freq_imag, batch, tokens, channels,
                                     heads, epsilon, q_out, k_out, v_out, st);
  if (dtype == SPR_F16)
    return launch_qkv<__half>(q, k, v, q_weight, k_weight, freq_real, freq_imag, batch, tokens, channels, heads,
                              epsilon, q_out, k_out, v_out, st);
  return launch_qkv<float>(q, k, v, q_weight, k_weight, freq_real, freq_imag, batch, tokens, channels, heads,
                           epsilon, q_out, k_out, v_out, st);
}
