// Self-test of the bounded-wait error path (dmx_selftest_wait_timeout).
//
// Every wait in this library's tensor-core kernels (on an mbarrier, or a peer)
// gives up after a fixed time, raises the handle's device error flag and lets
// the kernel return, so the host reports DMX_ERR_TIMEOUT and the CUDA context
// stays usable. Those waits only run out when something is broken, so this
// file provides one wait that always runs out: a single warp waits on a device
// flag that nothing ever sets, with a caller-chosen limit, then raises the
// same error flag with its own code. No trap, fault or unbounded loop.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace dmx {

namespace {

// Never written by anything: the condition the self-test waits for.
__device__ int g_never_set = 0;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void selftest_wait_kernel(uint64_t limit_ns, int code, int* __restrict__ err) {
  const uint64_t t0 = globaltimer_ns();
  while (*reinterpret_cast<volatile int*>(&g_never_set) == 0) {
    if (globaltimer_ns() - t0 > limit_ns) {
      if (threadIdx.x == 0) atomicExch(err, code);
      return;
    }
    __nanosleep(20000);
  }
}

}  // namespace

void launch_selftest_wait(uint64_t limit_ns, int code, int* err, cudaStream_t s) {
  selftest_wait_kernel<<<1, 32, 0, s>>>(limit_ns, code, err);
}

}  // namespace dmx
