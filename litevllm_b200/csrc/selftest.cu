// Self-test of the failure path every bounded wait in this library takes:
// one CTA waits on an mbarrier that nothing ever arrives on, with the given
// time limit, and reports LK_STATUS_WAIT_TIMEOUT in *status instead of
// hanging. The kernel then returns normally and the context stays usable.
#include "lk_common.cuh"
#include "lk_host.h"

namespace {

__global__ void wait_timeout_kernel(int32_t* status, uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    lk::mbar_init(&bar, 1);
    lk::fence_barrier_init();
  }
  __syncthreads();
  // parity 0 of a fresh barrier completes only after one arrival: none comes
  if (!lk::mbar_wait(&bar, 0, timeout_ns)) {
    if (threadIdx.x == 0) atomicOr(status, LK_STATUS_WAIT_TIMEOUT);
  }
}

}  // namespace

extern "C" int lk_selftest_wait_timeout(int32_t* status, uint64_t timeout_ns, void* stream) {
  if (!status || timeout_ns == 0 || timeout_ns > 100000000ull) return LK_ERR_INVALID_ARG;
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, timeout_ns);
  return lk::check_launch();
}
