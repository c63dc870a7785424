// Profiling helper: a one-thread kernel that holds its stream until the host
// has enqueued a whole plan (it spins on a host-mapped flag, at most ~1 s, then
// records DEV_TIMEOUT_GRID and returns), so the per-op timing events that
// follow measure back-to-back kernels instead of host launch gaps.
#include "kernels.h"
#include "tc100.cuh"

namespace emx {

__global__ void hold_kernel(const volatile int* flag, int seq, int* err) {
  const uint64_t t0 = globaltimer_ns();
  while (*flag < seq) {
    if (globaltimer_ns() - t0 > 1000000000ull) {
      record_error(err, DEV_TIMEOUT_GRID);
      return;
    }
    __nanosleep(200);
  }
}

void launch_hold(const int* flag, int seq, int* err, cudaStream_t stream) {
  hold_kernel<<<1, 1, 0, stream>>>(flag, seq, err);
}

}  // namespace emx
