// Self-test of the bounded device wait every pipeline in this library uses
// (tc::mbar_wait): one thread waits on an mbarrier that nothing arrives on,
// gives up after limit_ns, records its code in the status word and returns.
// The GPU context stays usable; the host reads the status like any other.
#include "tc_common.cuh"

namespace spr {

__global__ void bounded_wait_selftest_kernel(int* err, int code, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_wait(&bar, 0, err, code, limit_ns);
  __syncthreads();
}

}  // namespace spr

using namespace spr;

extern "C" int spr_selftest_bounded_wait(int* err, int code, int64_t limit_ns, void* stream) {
  if (!err || code == 0) return fail(SPR_ERR_ARG, "bounded-wait self-test: need a status word and a non-zero code");
  if (limit_ns <= 0 || limit_ns > 100000000) return fail(SPR_ERR_ARG, "bounded-wait self-test: limit must be in (0, 0.1 s]");
  bounded_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(err, code, (uint64_t)limit_ns);
  return check_launch("bounded-wait self-test");
}
