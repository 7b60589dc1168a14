// A kernel whose only job is to have its bounded wait run out, for the tests
// of the timeout path every tensor-core kernel here shares: it allocates
// TMEM like the GEMM and attention kernels, waits on an mbarrier nothing
// arrives at for a host-set limit, raises TL_FLAG_TIMEOUT in the device
// status word, frees TMEM and returns.  Nothing traps, faults or spins
// without a bound.
#include "tc_ptx.cuh"
#include "tl_common.cuh"

namespace tl {
namespace {

__global__ void __launch_bounds__(64, 1) wait_timeout_kernel(uint64_t limit_ns, uint32_t *status,
                                                            uint32_t *waited) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);  // one arrival expected; none comes
    ptx::fence_barrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(&tmem_slot, 32);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint64_t t0 = ptx::global_timer_ns();
    const bool got = ptx::mbar_wait_bounded(&bar, 0, limit_ns);
    *waited = static_cast<uint32_t>((ptx::global_timer_ns() - t0) / 1000u);  // microseconds
    if (!got) raise_flag(status, TL_FLAG_TIMEOUT);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 32);
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" int tl_check_wait_timeout(uint64_t limit_ns, uint32_t *waited_us, void *stream) {
  if (!waited_us) return fail(TL_ERR_INVALID, "tl_check_wait_timeout: null output");
  if (limit_ns > 1000000000ull)
    return fail(TL_ERR_RANGE, "tl_check_wait_timeout: limit above one second");
  uint32_t *status = device_status_ptr();
  if (!status) return fail(TL_ERR_CUDA, "tl_check_wait_timeout: no status word");
  wait_timeout_kernel<<<1, 64, 0, as_stream(stream)>>>(limit_ns, status, waited_us);
  return launch_status("tl_check_wait_timeout");
}
