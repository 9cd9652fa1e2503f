// gdn_common.cuh -- geometry constants and small helpers shared by the GDN
// decode and prefill kernels (fixed geometry qk4_v8_d128_k_last).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace gdn {

constexpr int kHQK = 4;      // q/k heads
constexpr int kHV = 8;       // v heads; v-head h reads q/k head h / 2
constexpr int kD = 128;      // head dim (K = V = 128)
constexpr int kChunk = 64;   // prefill chunk length (reference BT = 64)

// Device status codes (see gdn_b200_read_device_status).
constexpr int kDevStatusBadSeqlens = 1;
constexpr int kDevStatusWaitTimeout = 2;
constexpr int kDevStatusBadSlot = 3;  // a state-pool slot index out of range
constexpr int kDevStatusIndexCheck = 4;  // a debug-build index check failed

// Per-device status word (the library is one translation unit, gdn_b200.cu).
__device__ int g_device_status = 0;

__device__ __forceinline__ void set_device_status(int code) {
  atomicCAS(&g_device_status, 0, code);
}

// Index checks of the debug build (compile with -DGDN_DEBUG_CHECKS, see
// build.py): a failed check records device status 4 and execution goes on;
// nothing traps.  In the regular build they compile to nothing.
#ifdef GDN_DEBUG_CHECKS
#define GDN_DCHECK(cond)                                          \
  do {                                                            \
    if (!(cond)) ::gdn::set_device_status(::gdn::kDevStatusIndexCheck); \
  } while (0)
#else
#define GDN_DCHECK(cond) \
  do {                   \
  } while (0)
#endif

__device__ __forceinline__ float bf16_lo(uint32_t packed) {
  return __uint_as_float(packed << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t packed) {
  return __uint_as_float(packed & 0xFFFF0000u);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
// Round-to-nearest-even pack of two floats into bf16x2 (lo in bits 0..15).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}

// softplus with threshold 20 -- reference decode kernel.py:21-23.
__device__ __forceinline__ float softplus_thr20(float x) {
  return x <= 20.0f ? logf(1.0f + expf(x)) : x;
}
// overflow-safe softplus -- reference prefill kernel.py:1714-1720.
__device__ __forceinline__ float softplus_stable(float x) {
  return x > 0.0f ? x + logf(1.0f + expf(-x)) : logf(1.0f + expf(x));
}

}  // namespace gdn
