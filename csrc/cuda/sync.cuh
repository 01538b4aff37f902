// System-scope flag operations for cross-GPU signalling over NVLink peer memory, and a
// bounded wait that never hangs: after `timeout_ns` it records an error bit and returns.
#pragma once
#include <stdint.h>

namespace syn {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Waits until *flag == want (flags are monotone sequence numbers: >= also accepted).
// Returns false (and sets `err_bit` in *status) on timeout.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t want, uint64_t timeout_ns,
                                          int* status, int err_bit) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    const uint32_t v = ld_acquire_sys(flag);
    if ((int32_t)(v - want) >= 0) return true;
    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > timeout_ns) {
      if (status) atomicOr(status, 1 << err_bit);
      return false;
    }
    __nanosleep(64);
  }
}

}  // namespace syn
