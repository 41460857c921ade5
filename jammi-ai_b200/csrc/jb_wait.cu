// A bounded device-side wait on a flag in device memory: the building block
// every spin in the library's kernels follows (limit on %globaltimer, then an
// error bit the host reads as JB_ERR_TIMEOUT, the context left usable), as
// a single op so failure detection can be exercised without a fault: a wait
// on a flag that nothing sets runs out and reports, it never hangs.
#include <cstdint>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

__global__ void flag_wait_kernel(const volatile int* flag, int expect, uint64_t limit_ns, int* err) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = global_timer_ns();
  while (*flag != expect) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicOr(err, kErrTimeout);
      return;
    }
    __nanosleep(1000);
  }
}

}  // namespace

cudaError_t launch_flag_wait(const int* flag, int expect, int limit_ms, int* err, cudaStream_t s) {
  const uint64_t limit_ns = static_cast<uint64_t>(limit_ms) * 1000000ull;
  flag_wait_kernel<<<1, 32, 0, s>>>(flag, expect, limit_ns, err);
  return cudaGetLastError();
}

}  // namespace jb
