// gdn_wait.cuh -- the bounded mbarrier wait every kernel of this library uses
// for TMA, bulk-copy and MMA completion: a wait never spins forever; when its
// cycle budget runs out it records device status 2 (read by
// gdn_b200_read_device_status) and reports failure, and the caller skips its
// remaining work, waits (bounded) for its own copies in flight, frees any TMEM
// it holds and returns.
#pragma once
#include "gdn_common.cuh"
#include "sm100.cuh"

namespace gdn {
using namespace sm100;

// Cycle budget of one bounded wait: 2^33 SM cycles (about 4 s at the B200's
// top clock, longer at lower clocks).  The index-checked debug build reads it
// from a device variable instead, so that a test can shorten it and make a
// wait run out (gdn_b200_debug_wait_timeout_probe).
#ifdef GDN_DEBUG_CHECKS
__device__ long long g_wait_limit_cycles = 1ll << 33;
__device__ __forceinline__ long long wait_limit_cycles() {
  return *reinterpret_cast<volatile long long *>(&g_wait_limit_cycles);
}
#else
__device__ __forceinline__ constexpr long long wait_limit_cycles() { return 1ll << 33; }
#endif

// Slow path of wait_phase: keep polling, give up after wait_limit_cycles()
// or at once when another thread of the CTA already gave up; records device
// status 2.  A CTA that gave up finishes its loop without waiting again and
// still deallocates its TMEM.
__device__ __noinline__ bool wait_phase_slow(uint32_t mbar, uint32_t parity, volatile int *broken) {
  const long long t0 = clock64();
  const long long limit = wait_limit_cycles();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(mbar, parity)) return true;
    if (*broken) return false;
    if (clock64() - t0 > limit) {
      *broken = 1;
      set_device_status(kDevStatusWaitTimeout);
      return false;
    }
  }
}

// Wait for an mbarrier phase: one try_wait (which itself suspends the warp
// for a while) covers the common case; only a still-pending phase takes the
// bounded slow path.
__device__ __forceinline__ bool wait_phase(uint32_t mbar, uint32_t parity, volatile int *broken) {
  if (mbar_try_wait(mbar, parity)) return true;
  if (*broken) return false;
  return wait_phase_slow(mbar, parity, broken);
}

// The same bounded wait, with acquire at cluster scope (phases completed by
// the other CTA of a cluster).
__device__ __noinline__ bool wait_phase_cluster_slow(uint32_t mbar, uint32_t parity,
                                                     volatile int *broken) {
  const long long t0 = clock64();
  const long long limit = wait_limit_cycles();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(mbar, parity)) return true;
    if (*broken) return false;
    if (clock64() - t0 > limit) {
      *broken = 1;
      set_device_status(kDevStatusWaitTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ bool wait_phase_cluster(uint32_t mbar, uint32_t parity,
                                                   volatile int *broken) {
  if (mbar_try_wait_cluster(mbar, parity)) return true;
  if (*broken) return false;
  return wait_phase_cluster_slow(mbar, parity, broken);
}

}  // namespace gdn
