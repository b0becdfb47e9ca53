// Role projections of the N8-V6 route on the tensor cores.
//
//   K role:  feat = (K F_k) / rms(K F_k)      one RMS over all tokens and features of a head
//   Q role:  feat = (Q F_q) / rms_row(Q F_q)  one RMS per token row
//
// (n8_v6.py:141-178 normalize_feature_scale / normalize_rows_rms, 659-806;
// role_projection.py:58-103).  X is bf16 [bh][n][128], F fp32 [bh][128][r],
// out fp32 [bh][n][r].
//
// The fp32 factor is split into three bf16 parts F = F1 + F2 + F3 (each the
// bf16 rounding of what the previous parts leave), carrying it to ~2^-24
// relative; the bf16 X times each part is exact in the fp32 accumulator, so
// three kind::f16 MMAs per K step give the projection at fp32 accuracy (the
// reference computes it in TF32 or fp32, by its matmul-precision setting).
//
// One CTA per 128-token tile of one head (4 warps).  Thread 0 loads the tile
// and the three factor parts with TMA (128-byte swizzle) and issues 3 x 8 MMAs
// (M = 128 tokens, N = r, K = 16) into a TMEM accumulator; each thread then
// owns one token row: it reads its r features from TMEM, and either divides
// them by their row RMS (Q) or writes them raw and adds their squares to the
// tile's partial sum (K; a second kernel reduces the partial sums of a head in
// a fixed order and divides in place).  HBM traffic: X read once, features
// written once (K: read and written once more by the scaling pass).
#include "common.cuh"
#include "tc_common.cuh"
#include "tmap.cuh"

namespace spr {

namespace {

constexpr int kPD = 128;  // model head dim
constexpr int kPM = 128;  // tokens per tile
constexpr int kPThreads = 128;
constexpr int kPParts = 3;

__device__ int g_proj_err;

inline int proj_smem_bytes(int r) { return 1024 + kPM * kPD * 2 + kPParts * r * kPD * 2; }

// F [bh][128][r] fp32 -> parts [3][bh][r][128] bf16 (transposed: K-major B operand).
__global__ void factor_split_kernel(const float* __restrict__ f, int64_t bh, int r, __nv_bfloat16* __restrict__ parts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = bh * r * kPD;
  if (i >= total) return;
  const int64_t b = i / (r * kPD);
  const int j = (int)((i / kPD) % r), e = (int)(i % kPD);
  const float v = f[(b * kPD + e) * r + j];
  const __nv_bfloat16 p1 = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(p1);
  const __nv_bfloat16 p2 = __float2bfloat16_rn(r1);
  const __nv_bfloat16 p3 = __float2bfloat16_rn(r1 - __bfloat162float(p2));
  parts[i] = p1;
  parts[total + i] = p2;
  parts[2 * total + i] = p3;
}

template <int R>
__global__ void __launch_bounds__(kPThreads)
role_projection_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap fmap,
                       int64_t bh, int64_t n, int row_mode, float* __restrict__ out, float* __restrict__ partial) {
  constexpr int TC = R <= 32 ? 32 : R <= 64 ? 64 : 128;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full, bar_mma;
  __shared__ uint32_t s_tmem;
  __shared__ float s_red[4];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sx = tc::smem_addr(smem);
  const uint32_t sf = sx + kPM * kPD * 2;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t b = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.x * kPM;
  if (tid == 0) {
    tc::mbar_init(&bar_full, 1);
    tc::mbar_init(&bar_mma, 1);
    tc::mbar_fence_init();
  }
  if (warp == 0) tc::tmem_alloc<TC>(&s_tmem);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (tid == 0) {
    tc::prefetch_tmap(&xmap);
    tc::prefetch_tmap(&fmap);
    tc::mbar_expect_tx(&bar_full, (uint32_t)(kPM * kPD * 2 + kPParts * R * kPD * 2));
    // Two 128-byte column blocks (64 bf16 each) per row, rows past n zero-filled.
    tc::tma_load_3d(sx, &xmap, 0, (int)t0, (int)b, &bar_full);
    tc::tma_load_3d(sx + kPM * 128, &xmap, 64, (int)t0, (int)b, &bar_full);
    for (int p = 0; p < kPParts; ++p) {
      const uint32_t fp = sf + p * R * kPD * 2;
      tc::tma_load_3d(fp, &fmap, 0, 0, (int)(p * bh + b), &bar_full);
      tc::tma_load_3d(fp + R * 128, &fmap, 64, 0, (int)(p * bh + b), &bar_full);
    }
    if (tc::mbar_wait(&bar_full, 0, &g_proj_err, 51)) {
      tc::tc_fence_after();
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kPM, R, 0);
#pragma unroll
      for (int p = 0; p < kPParts; ++p)
#pragma unroll
        for (int kk = 0; kk < kPD / 16; ++kk) {
          const uint32_t kb = kk * 32;  // 16 bf16 per K step
          const uint32_t xo = (kb >> 7) * (kPM * 128) + (kb & 127);
          const uint32_t fo = p * R * kPD * 2 + (kb >> 7) * (R * 128) + (kb & 127);
          tc::mma_f16(tmem, tc::sw128_desc(sx + xo, 16, 1024), tc::sw128_desc(sf + fo, 16, 1024), idesc,
                      (p | kk) != 0);
        }
      tc::mma_commit(&bar_mma);
    } else {
      tc::mbar_drain(&bar_full, 0);
    }
  }
  // A failed tile load leaves bar_mma unsignalled: every thread's bounded wait
  // then gives up and the tile is skipped (status word set).
  const bool done = __all_sync(0xffffffffu, tc::mbar_wait(&bar_mma, 0, &g_proj_err, 52));
  tc::tc_fence_after();
  const int row = tid;  // TMEM lane = token row of the tile
  const int64_t t = t0 + row;
  float ss = 0.f;
  if (done) {
    float v[TC];
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll
    for (int c = 0; c < TC; c += 32) tc::tmem_ld32_async(tmem + lane_base + c, v + c);
    tc::tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < TC; c += 32) tc::reg_fence32(v + c);
#pragma unroll
    for (int j = 0; j < R; ++j) ss = fmaf(v[j], v[j], ss);
    if (t < n) {
      float* o = out + (b * n + t) * R;
      if (row_mode) {
        const float den = fmaxf(sqrtf(ss / (float)R), 1e-6f);
#pragma unroll
        for (int j = 0; j < R; j += 4)
          *reinterpret_cast<float4*>(o + j) =
              make_float4(__fdiv_rn(v[j], den), __fdiv_rn(v[j + 1], den), __fdiv_rn(v[j + 2], den),
                          __fdiv_rn(v[j + 3], den));
      } else {
#pragma unroll
        for (int j = 0; j < R; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    } else {
      ss = 0.f;
    }
  }
  if (!row_mode) {  // partial sum of squares of this tile (fixed order)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) s_red[warp] = ss;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (!row_mode && tid == 0) partial[b * gridDim.x + blockIdx.x] = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc<TC>(tmem);
  }
}

// Per head: scale = max(sqrt(sum of the tile partials / (n r)), 1e-8) in a
// fixed order (fp64), written to scale[b]; then every feature is divided by it.
__global__ void global_scale_kernel(const float* __restrict__ partial, int tiles, int64_t n, int r,
                                    float* __restrict__ scale) {
  __shared__ double s[256];
  const int64_t b = blockIdx.x;
  double acc = 0.0;
  for (int i = threadIdx.x; i < tiles; i += blockDim.x) acc += (double)partial[b * tiles + i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) scale[b] = fmaxf(sqrtf((float)(s[0] / ((double)n * (double)r))), 1e-8f);
}

__global__ void apply_scale_kernel(float* __restrict__ out, int64_t per_head, int64_t total4,
                                   const float* __restrict__ scale) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    const float sc = __ldg(scale + (i * 4) / per_head);
    float4 v = reinterpret_cast<float4*>(out)[i];
    v.x = __fdiv_rn(v.x, sc);
    v.y = __fdiv_rn(v.y, sc);
    v.z = __fdiv_rn(v.z, sc);
    v.w = __fdiv_rn(v.w, sc);
    reinterpret_cast<float4*>(out)[i] = v;
  }
}

struct ProjWs {
  __nv_bfloat16* parts;  // [3][bh][r][128]
  float* partial;        // [bh][tiles]
};

ProjWs carve_proj(Carver& c, int64_t bh, int64_t n, int r) {
  ProjWs w;
  w.parts = c.take<__nv_bfloat16>((size_t)kPParts * bh * r * kPD);
  w.partial = c.take<float>((size_t)bh * ((n + kPM - 1) / kPM));
  return w;
}

template <int R>
int launch_proj(const CUtensorMap& xmap, const CUtensorMap& fmap, int64_t bh, int64_t n, int row_mode, float* out,
                float* partial, cudaStream_t st) {
  auto kern = role_projection_kernel<R>;
  const int smem = proj_smem_bytes(R);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((unsigned)((n + kPM - 1) / kPM), (unsigned)bh);
  kern<<<grid, kPThreads, smem, st>>>(xmap, fmap, bh, n, row_mode, out, partial);
  return check_launch("role projection");
}

}  // namespace

}  // namespace spr

using namespace spr;

extern "C" size_t spr_role_projection_workspace_bytes(int64_t bh, int64_t n, int r) {
  Carver c(nullptr, 0);
  carve_proj(c, bh, n, r);
  return c.off + 256;
}

extern "C" int spr_role_projection(const void* x, const float* factor, int64_t bh, int64_t n, int d, int r, int mode,
                                   float* out, float* scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (d != kPD) return fail(SPR_ERR_SHAPE, "role projection: d=%d unsupported (128 only)", d);
  if (bh <= 0 || bh > 65535 || n <= 0 || n > INT32_MAX)
    return fail(SPR_ERR_SHAPE, "role projection: bh=%lld n=%lld out of range", (long long)bh, (long long)n);
  if (r != 16 && r != 32 && r != 48 && r != 64)
    return fail(SPR_ERR_SHAPE, "role projection: rank r=%d unsupported (16, 32, 48 or 64)", r);
  if (mode != 0 && mode != 1) return fail(SPR_ERR_ARG, "role projection: mode %d (0 global RMS, 1 row RMS)", mode);
  if (mode == 0 && !scale) return fail(SPR_ERR_ARG, "role projection: global-RMS mode needs the scale output");
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(factor, 4))
    return fail(SPR_ERR_ALIGN, "role projection: x and out must be 16-byte aligned");
  Carver c(workspace, workspace_bytes);
  ProjWs w = carve_proj(c, bh, n, r);
  if (!c.ok() || !workspace)
    return fail(SPR_ERR_WORKSPACE, "role projection: workspace %zu < %zu", workspace_bytes, c.off);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t total = bh * r * kPD;
  factor_split_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(factor, bh, r, w.parts);
  int s = check_launch("role projection: factor split");
  if (s) return s;
  CUtensorMap xmap, fmap;
  if ((s = encode_map_3d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, kPD, n, bh, 64, kPM, "role projection X")))
    return s;
  if ((s = encode_map_3d(&fmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.parts, kPD, r, kPParts * bh, 64, r,
                         "role projection factor")))
    return s;
  switch (r) {
    case 16: s = launch_proj<16>(xmap, fmap, bh, n, mode, out, w.partial, st); break;
    case 32: s = launch_proj<32>(xmap, fmap, bh, n, mode, out, w.partial, st); break;
    case 48: s = launch_proj<48>(xmap, fmap, bh, n, mode, out, w.partial, st); break;
    default: s = launch_proj<64>(xmap, fmap, bh, n, mode, out, w.partial, st); break;
  }
  if (s || mode == 1) return s;
  const int tiles = (int)((n + kPM - 1) / kPM);
  global_scale_kernel<<<(unsigned)bh, 256, 0, st>>>(w.partial, tiles, n, r, scale);
  if ((s = check_launch("role projection: global scale"))) return s;
  const int64_t total4 = bh * n * r / 4;
  apply_scale_kernel<<<148 * 8, 256, 0, st>>>(out, n * r, total4, scale);
  return check_launch("role projection: apply scale");
}

extern "C" int spr_role_projection_status(int* out) {
  if (!out) return fail(SPR_ERR_ARG, "role projection status: null output");
  if (cudaMemcpyFromSymbol(out, g_proj_err, sizeof(int)) != cudaSuccess)
    return fail(SPR_ERR_LAUNCH, "role projection status: copy failed");
  return SPR_OK;
}

extern "C" int spr_role_projection_status_async(int32_t* dst, void* stream) {
  if (!dst) return fail(SPR_ERR_ARG, "role projection status: null destination");
  const cudaError_t e = cudaMemcpyFromSymbolAsync(dst, g_proj_err, sizeof(int), 0, cudaMemcpyDeviceToDevice,
                                                  (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "role projection status: %s", cudaGetErrorString(e));
  return SPR_OK;
}
