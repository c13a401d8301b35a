// Bounded device-side waits: the polling primitive behind every cross-CTA and
// cross-rank wait of the fused step, and behind hv_wait_probe.
//
// A wait never spins forever: it gives up after a limit measured on %globaltimer (or as
// soon as another party has reported a failure in *status), records HV_E_TIMEOUT in
// *status (first failure wins) and returns false, so the kernel can unwind and the host
// reads an error instead of finding a hung GPU.
#pragma once

#include <cstdint>

#include "hive_b200.h"
#include "hv_common.cuh"

namespace hv {

HV_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

HV_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

HV_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Poll *w (acquire; system scope with kSys, for words other GPUs write) until
// (value & mask) == want. False when a failure is already reported in *status, or after
// limit_ns (then *status = HV_E_TIMEOUT unless another failure got there first). The
// status and the clock are checked every 32 polls.
template <bool kSys>
HV_DEV bool poll_word_until(const unsigned* w, unsigned mask, unsigned want, int* status,
                            unsigned long long limit_ns) {
  const unsigned long long t0 = global_ns();
  for (unsigned n = 1;; ++n) {
    const unsigned v = kSys ? ld_acquire_sys(w) : ld_acquire(w);
    if ((v & mask) == want) return true;
    if ((n & 31) == 0) {
      if (*(volatile int*)status != 0) return false;
      if (global_ns() - t0 > limit_ns) {
        atomicCAS(status, 0, HV_E_TIMEOUT);
        return false;
      }
    }
  }
}

}  // namespace hv
