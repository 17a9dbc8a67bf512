// Self-test of the bounded device-side wait that every probe kernel relies on.
//
// One thread arms an mbarrier for 16 transaction bytes that no copy will ever
// deliver, so the barrier's phase cannot complete, and waits on it with the
// library's bounded wait (mbar_wait) and a caller-chosen limit.  The wait must
// give up, write TCB_ERR_TIMEOUT into the status word and let the kernel
// return: no trap, no fault, and the context stays usable.  Nothing is in
// flight when the kernel exits (no copy was ever issued into the barrier).
//
// No counterpart in the reference suite, whose Triton kernels have no
// device-side waits.
#include "tcb_device.cuh"
#include "tcb_host.h"

namespace tcb {
namespace {

__global__ void bounded_wait_selftest_kernel(unsigned long long limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_arrive_expect_tx(&bar, 16);
  if (!mbar_wait(&bar, 0, limit_ns)) report_status(status, TCB_ERR_TIMEOUT);
}

}  // namespace
}  // namespace tcb

using namespace tcb;

extern "C" int tcb_selftest_bounded_wait(long long limit_ns, int* status_dev,
                                         tcb_stream_t stream) {
  // At most one second: the self-test must end quickly whatever it is given.
  if (status_dev == nullptr || limit_ns < 0 || limit_ns > 1000000000LL)
    return TCB_ERR_INVALID_ARGUMENT;
  clear_stale_error();
  bounded_wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_ns), status_dev);
  return launch_status();
}
