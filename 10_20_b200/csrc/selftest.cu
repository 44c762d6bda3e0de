// Failure-detection self test: runs the bounded mbarrier wait every pipelined
// kernel of this library uses, on a barrier that nothing ever arrives at, so the
// wait's time limit expires and the kernel reports V1X_STATUS_TIMEOUT through the
// status word.  The GPU context stays usable afterwards; this is how the timeout
// path is exercised without faulting or hanging a GPU.
#include "common.cuh"
#include "sm100.cuh"

namespace v1x {
namespace {

__global__ void wait_timeout_kernel(uint64_t limit_ns, int32_t* status, uint64_t* elapsed_ns) {
  __shared__ uint64_t bar;
  __shared__ int no_abort;
  if (threadIdx.x != 0) return;
  no_abort = 0;
  sm100::mbar_init(&bar, 1);
  sm100::fence_mbar_init();
  const uint64_t t0 = sm100::globaltimer_ns();
  const bool done = sm100::mbar_wait(&bar, 0, &no_abort, limit_ns);  // nothing arrives
  if (!done) atomicExch(status, V1X_STATUS_TIMEOUT);
  if (elapsed_ns) *elapsed_ns = sm100::globaltimer_ns() - t0;
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_selftest_wait_timeout(int64_t limit_ns, int32_t* status, uint64_t* elapsed_ns, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(limit_ns > 0 && limit_ns <= 10000000000ll, "selftest: limit_ns must be in (0, 10 s]");
  V1X_CHECK_ARG(status != nullptr, "selftest: status word required");
  wait_timeout_kernel<<<1, 32, 0, as_stream(stream)>>>(static_cast<uint64_t>(limit_ns), status, elapsed_ns);
  return launch_status("v1x_selftest_wait_timeout");
}
