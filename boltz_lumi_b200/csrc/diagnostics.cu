// Self-test of the bounded device-side wait that every tensor-core kernel of
// this library uses (tc::mbar_wait): one thread waits on an mbarrier phase.
// With `arrive` the phase completes first and the wait succeeds; without it
// nothing ever completes the phase, so the wait runs out after `limit_ns`,
// records its code in the device status word and returns -- the kernel exits
// normally and the context stays usable.  No fault, trap or hang is involved.
#include "tc.cuh"

namespace bl {
namespace {

// Status code the self-test's wait records when it runs out.
constexpr unsigned int kWaitSelftestCode = 0x7F01;

__global__ void wait_selftest_kernel(int arrive, uint64_t limit_ns, unsigned int *status) {
  __shared__ uint64_t bar;
  tc::mbar_init(&bar, 1);
  tc::fence_mbar_init();
  if (arrive) tc::mbar_arrive(&bar);
  tc::mbar_wait(&bar, 0, status, kWaitSelftestCode, limit_ns);
}

}  // namespace
}  // namespace bl

using namespace bl;

extern "C" int bl_wait_selftest(int arrive, int64_t limit_ns, void *stream) {
  BL_REQUIRE(limit_ns > 0 && limit_ns <= int64_t(tc::kWaitLimitNs),
             "bl_wait_selftest: limit must be in (0, %llu] ns", (unsigned long long)tc::kWaitLimitNs);
  unsigned int *status = device_status_ptr();
  BL_REQUIRE(status, "bl_wait_selftest: device status word unavailable");
  wait_selftest_kernel<<<1, 1, 0, as_stream(stream)>>>(arrive, uint64_t(limit_ns), status);
  BL_LAUNCH_CHECK();
  return BL_OK;
}
