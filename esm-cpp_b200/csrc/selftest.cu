// Failure-detection self-test of the bounded device waits.
//
// Every mbarrier wait in the kernels of this library gives up after a bound
// (common.cuh: mbar_wait, mbar_wait_abort), records kStatusTimeout in the
// context's status word and unwinds, so a lost arrival ends as
// ESMCU_ERR_TIMEOUT on the host instead of a hung GPU.  This entry point makes
// such a wait run out on purpose, with a short bound and no fault: one CTA
// initialises an mbarrier that expects two arrivals and gives it only one, so
// its phase never completes.  One thread waits with mbar_wait, the others
// with mbar_wait_abort on a shared abort flag, the form the multi-role
// kernels use: the first waiter to reach the bound sets the flag and the rest
// leave through it.  Every wait ends after about limit_us microseconds.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host/context.h"

namespace esmb200 {
namespace {

constexpr int kSelftestThreads = 128;

__global__ void __launch_bounds__(kSelftestThreads)
    bounded_wait_selftest_kernel(uint64_t limit_ns, uint32_t* status, uint32_t* released) {
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(&bar);  // one of the two expected arrivals
  const bool lead = (threadIdx.x & 31) == 0;
  if (!lead) return;
  bool done;
  if (threadIdx.x == 0)
    done = mbar_wait(&bar, 0, status, limit_ns);
  else
    done = mbar_wait_abort(&bar, 0, status, &abort_flag, limit_ns);
  if (!done) atomicAdd(released, 1u);
}

}  // namespace
}  // namespace esmb200

using namespace esmb200;

extern "C" int esmcu_bounded_wait_selftest(esmcu_context* ctx, int limit_us, int* waiters_released) {
  int rc = use_device(ctx);
  if (rc != ESMCU_OK) return rc;
  if (limit_us <= 0 || limit_us > 1000000)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "limit_us must be in (0, 1000000]");
  if (waiters_released == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "waiters_released is null");
  *waiters_released = 0;
  // The released-waiter counter sits in the context scratch (4 bytes).
  rc = ensure_scratch(ctx, sizeof(uint32_t));
  if (rc != ESMCU_OK) return rc;
  uint32_t* released = static_cast<uint32_t*>(ctx->scratch);
  ESMCU_CUDA(cudaMemsetAsync(released, 0, sizeof(uint32_t), ctx->stream));
  bounded_wait_selftest_kernel<<<1, kSelftestThreads, 0, ctx->stream>>>(
      static_cast<uint64_t>(limit_us) * 1000ull, ctx->d_status, released);
  ESMCU_CUDA(cudaGetLastError());
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  uint32_t n = 0;
  ESMCU_CUDA(cudaMemcpy(&n, released, sizeof(n), cudaMemcpyDeviceToHost));
  *waiters_released = static_cast<int>(n);
  return check_device_status(ctx);
}
