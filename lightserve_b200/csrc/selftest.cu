// Self-test of the failure path every on-chip wait of this library takes.
//
// Each mbarrier wait in the kernels is bounded (sm100.cuh, LSB_WAIT_CYCLES,
// about one second): when the partner never arrives, the waiting thread
// records a code in its translation unit's error word and returns, and the
// kernel winds down instead of hanging the GPU. This entry point runs that
// path on purpose with a one-thread kernel waiting on an mbarrier that nothing
// ever arrives on, so a test can check that the wait gives up, that
// lsb_device_error() reports it and that the context stays usable afterwards.
// It never faults, traps or hangs the GPU.
#include "common.cuh"
#include "sm100.cuh"

namespace lsb {

using namespace sm100;

constexpr int SELFTEST_WAIT_CODE = 0xE01;

__global__ void selftest_bounded_wait_kernel(int* status) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  // Phase 0 of `bar` never completes: no thread arrives on it.
  const bool completed = mbar_wait(&bar, 0, SELFTEST_WAIT_CODE);
  status[0] = completed ? 1 : 0;
}

int selftest_device_error(bool reset) { return tu_device_error(reset); }

}  // namespace lsb

extern "C" int lsb_selftest_bounded_wait(int* status, void* stream) {
  LSB_CHECK_ARG(status != nullptr, "selftest_bounded_wait: null status");
  lsb::selftest_bounded_wait_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(status);
  LSB_CHECK_LAUNCH("selftest_bounded_wait");
  return LSB_OK;
}
