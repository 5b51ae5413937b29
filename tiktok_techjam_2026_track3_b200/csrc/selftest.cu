// Self-test of the bounded-wait machinery: a kernel waits on an mbarrier that
// nothing ever arrives on, gives up after a short limit, records
// kDevTimeoutInjected in the status word and returns.  This exercises the
// failure path every pipeline wait relies on without faulting or hanging the
// GPU (the host then sees TTJ_ERR_DEVICE_TIMEOUT through ttj_read_status).
#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

__global__ void wait_timeout_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Phase 0 never completes: the wait runs out after limit_ns.
  mbar_wait_warp(&bar, 0, status, kDevTimeoutInjected, &abort_flag, limit_ns);
}

}  // namespace

int launch_wait_timeout_selftest(int* status, int64_t limit_us, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(status, (uint64_t)limit_us * 1000ull);
  TTJ_CUDA_TRY(cudaGetLastError());
  return TTJ_OK;
}

}  // namespace ttj
