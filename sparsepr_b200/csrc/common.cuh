// Shared helpers for the sparsepr_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string.h>
#include <algorithm>

#include "../../include/sparsepr_b200.h"

namespace spr {

// Thread-local message of the last failure (read by spr_last_error()).
void set_error(const char* fmt, ...);

inline int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return status;
}

// Map the result of the launches just issued to a status.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SPR_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return SPR_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int dtype_bytes(int dt) { return dt == SPR_F32 ? 4 : 2; }

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Carves aligned sub-buffers out of one caller-provided workspace.
struct Carver {
  char* base;
  size_t cap;
  size_t off = 0;
  Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <typename T> T* take(size_t count) {
    off = align_up(off, 256);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
  bool ok() const { return off <= cap; }
};

}  // namespace spr
