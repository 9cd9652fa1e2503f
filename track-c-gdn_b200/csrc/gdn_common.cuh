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

// Packed fp32 pairs for the sm_100 f32x2 instructions (mul/fma/add.rn.f32x2:
// two independent round-to-nearest fp32 operations per instruction, results
// identical to the scalar instructions on the same operands).  A pair is a
// 64-bit register {lo, hi}.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t x) {
  float lo;
  asm("{\n\t.reg .f32 hi;\n\tmov.b64 {%0, hi}, %1;\n\t}" : "=f"(lo) : "l"(x));
  return lo;
}
__device__ __forceinline__ float f2_hi(uint64_t x) {
  float hi;
  asm("{\n\t.reg .f32 lo;\n\tmov.b64 {lo, %0}, %1;\n\t}" : "=f"(hi) : "l"(x));
  return hi;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// a * b + c, each half fused (one rounding)
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
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
