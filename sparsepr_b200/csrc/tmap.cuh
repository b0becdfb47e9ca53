// Host-side tensor-map encoding for tiled TMA loads.  cuTensorMapEncodeTiled
// is resolved through the runtime's driver entry-point query, so the library
// does not link libcuda itself.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace spr {

// 3-D tiled map over a row-major [outer][rows][inner] tensor with a 128-byte
// swizzle; box = box_inner x box_rows x 1 elements, zero fill out of bounds.
inline int encode_map_3d(CUtensorMap* m, CUtensorMapDataType dtype, int elem_bytes, const void* base, int64_t inner,
                         int64_t rows, int64_t outer, int box_inner, int box_rows, const char* what) {
  using EncodeFn = decltype(&cuTensorMapEncodeTiled);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return fail(SPR_ERR_LAUNCH, "%s: cuTensorMapEncodeTiled is unavailable", what);
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)outer};
  cuuint64_t strides[2] = {(cuuint64_t)(inner * elem_bytes), (cuuint64_t)(rows * inner * elem_bytes)};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPR_ERR_LAUNCH, "%s: tensor map encoding failed (CUresult %d)", what, (int)r);
  return SPR_OK;
}

}  // namespace spr
