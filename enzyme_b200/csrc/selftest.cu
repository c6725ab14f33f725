// Diagnostic: exercise the bounded-wait paths without a fault.
//
// One thread waits, each for at most limit_ns of %globaltimer, on (1) an
// mbarrier that nothing arrives on -- the wait helper the tcgen05 GEMM and the
// cluster scan use for TMA / bulk-copy completion -- and (2) a global flag that
// nothing sets, polled with acquire loads and backoff as the look-back scan
// polls its predecessors. Each wait must give up and report AXON_E_TIMEOUT in
// the caller's status words; the kernel then exits normally, so the context
// stays usable. This is how the timeout handling is tested on a shared GPU:
// no trap, no fault, no unbounded spin.
#include "common.cuh"
#include "sm100.cuh"

namespace axon {
namespace {

__global__ void bounded_wait_selftest(int64_t limit_ns, int* status, const unsigned* flag) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  sm100::mbar_init(&bar, 1);
  sm100::mbar_init_fence();
  const bool arrived = sm100::mbar_wait_bounded(&bar, 0, static_cast<uint64_t>(limit_ns));
  status[0] = arrived ? AXON_OK : AXON_E_TIMEOUT;

  bool seen = false;
  const uint64_t t0 = sm100::globaltimer_ns();
  while (sm100::globaltimer_ns() - t0 < static_cast<uint64_t>(limit_ns)) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v != 0u) {
      seen = true;
      break;
    }
    __nanosleep(256);
  }
  status[1] = seen ? AXON_OK : AXON_E_TIMEOUT;
}

}  // namespace
}  // namespace axon

using namespace axon;

extern "C" int axon_selftest_bounded_wait(int64_t limit_ns, void* status2, const void* flag, void* stream) {
  if (!status2 || !flag) return fail(AXON_E_ARG, "axon_selftest_bounded_wait: NULL status or flag");
  if (limit_ns <= 0 || limit_ns > 5000000000LL)
    return fail(AXON_E_ARG, "axon_selftest_bounded_wait: limit must be in (0, 5 s]");
  bounded_wait_selftest<<<1, 32, 0, as_stream(stream)>>>(limit_ns, static_cast<int*>(status2),
                                                          static_cast<const unsigned*>(flag));
  return launch_status("axon_selftest_bounded_wait");
}
