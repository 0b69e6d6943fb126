// Self-test of the bounded-wait path that every mbarrier wait in the GEMM and
// attention kernels relies on: a kernel waits on an mbarrier phase that
// nothing completes, gives up after the caller's limit, records
// DEV_ERR_WAIT_TIMEOUT in the device error word and returns.  The context
// stays usable, so a test can check the error word and go on.  No TMA or
// tensor-core work is in flight while it waits.
#include "sm100.cuh"

namespace q35 {
namespace {

constexpr int kSelftestSite = 901;

__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns, int *err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);  // one arrival completes phase 0; none comes
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_timer_ns();
    if (!sm100::mbar_wait(&bar, 0, limit_ns)) {
      const uint64_t waited_us = (global_timer_ns() - t0) / 1000;
      report_error(err, DEV_ERR_WAIT_TIMEOUT, kSelftestSite,
                   static_cast<int>(waited_us > 0x7fffffff ? 0x7fffffff : waited_us), 0);
    }
  }
}

}  // namespace
}  // namespace q35

extern "C" int q35_selftest_wait_timeout(int64_t limit_ns, q35_stream_t stream) {
  using namespace q35;
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    return fail(Q35_ERR_INVALID, "selftest_wait_timeout: limit %lld ns (0 < limit <= 2 s)",
                (long long)limit_ns);
  int *err = device_error_word();
  if (!err) return fail(Q35_ERR_CUDA, "selftest_wait_timeout: no device error word");
  wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(limit_ns), err);
  Q35_LAUNCH_CHECK("selftest_wait_timeout launch");
  return Q35_OK;
}
