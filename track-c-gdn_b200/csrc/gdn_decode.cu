// gdn_decode.cu -- fused single-token GDN decode step for sm_100a.
//
// Computes, per (request b, v-head hv) -- reference decode kernel.py:26-79 --
//   g    = exp(-exp(A_log[hv]) * softplus20(a[b,hv] + dt_bias[hv]))
//   beta = sigmoid(b[b,hv])
//   for every state row v (k-last layout S[v, :]):
//     h      = g * S[v, :]
//     delta  = beta * (v[b,hv,v] - h . k)
//     S'[v,:] = h + delta * k
//     out[v] = S'[v,:] . (scale * q)
//
// The step is bound by HBM bandwidth: every (request, v-head) streams its
// 64 KiB fp32 state in and 64 KiB out, against ~0.8 KiB of vectors.  Layout:
// one warp owns a state row (512 contiguous bytes = one float4 per lane, a
// single fully coalesced 128-bit access per row); each warp keeps four rows'
// loads in flight and reduces h.k and S'.q with butterfly shuffles.  A CTA of
// 8 warps covers 32 rows of one head, so a head is spread over 4 CTAs and
// even batch 16 puts 512 CTAs on the 148 SMs.  State traffic uses streaming
// (evict-first) loads/stores: it is touched exactly once per step.
// new_state may alias state (in-place update): every element is read and
// then written by the same thread.
#include "gdn_common.cuh"

namespace gdn {

constexpr int kDecWarps = 8;
constexpr int kDecRowsPerWarp = 4;
constexpr int kDecRowsPerCta = kDecWarps * kDecRowsPerWarp;  // 32
constexpr int kDecCtasPerHead = kD / kDecRowsPerCta;         // 4

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__global__ void __launch_bounds__(kDecWarps * 32)
gdn_decode_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                  const uint16_t *__restrict__ v, const float *state,
                  const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                  const float *__restrict__ dt_bias, const uint16_t *__restrict__ b,
                  float scale, uint16_t *__restrict__ out, float *new_state) {
  const int64_t head = blockIdx.x / kDecCtasPerHead;  // request * 8 + v-head
  const int part = blockIdx.x % kDecCtasPerHead;
  const int64_t req = head / kHV;
  const int hv = static_cast<int>(head % kHV);
  const int hqk = hv >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = part * kDecRowsPerCta + warp * kDecRowsPerWarp;  // first v index
  const int64_t sbase = head * kD * kD;

  // Issue the state loads first: they are the long-latency part.
  float4 s[kDecRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kDecRowsPerWarp; ++i) {
    if (state != nullptr) {
      s[i] = __ldcs(reinterpret_cast<const float4 *>(state + sbase + (row0 + i) * kD) + lane);
    } else {
      s[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  // Lane l owns k-columns 4l .. 4l+3.
  const int64_t qk_off = (req * kHQK + hqk) * kD + 4 * lane;
  const uint2 qr = *reinterpret_cast<const uint2 *>(q + qk_off);
  const uint2 kr = *reinterpret_cast<const uint2 *>(k + qk_off);
  const float q0 = bf16_lo(qr.x) * scale, q1 = bf16_hi(qr.x) * scale;
  const float q2 = bf16_lo(qr.y) * scale, q3 = bf16_hi(qr.y) * scale;
  const float k0 = bf16_lo(kr.x), k1 = bf16_hi(kr.x), k2 = bf16_lo(kr.y), k3 = bf16_hi(kr.y);

  // Gates (kernel.py:59-65).
  const float a_val = bf16_to_f32(a[head]);
  const float b_val = bf16_to_f32(b[head]);
  const float g = expf(-expf(A_log[hv]) * softplus_thr20(a_val + dt_bias[hv]));
  const float beta = 1.0f / (1.0f + expf(-b_val));

  // v values of this warp's four rows (row0 is a multiple of 4: 8-byte load).
  const uint2 vr = *reinterpret_cast<const uint2 *>(v + head * kD + row0);
  const float vv[4] = {bf16_lo(vr.x), bf16_hi(vr.x), bf16_lo(vr.y), bf16_hi(vr.y)};

  float old[kDecRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kDecRowsPerWarp; ++i) {
    s[i].x *= g;
    s[i].y *= g;
    s[i].z *= g;
    s[i].w *= g;
    old[i] = s[i].x * k0 + s[i].y * k1 + s[i].z * k2 + s[i].w * k3;
  }
#pragma unroll
  for (int i = 0; i < kDecRowsPerWarp; ++i) old[i] = warp_sum(old[i]);

  float o[kDecRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kDecRowsPerWarp; ++i) {
    const float delta = beta * (vv[i] - old[i]);
    s[i].x += k0 * delta;
    s[i].y += k1 * delta;
    s[i].z += k2 * delta;
    s[i].w += k3 * delta;
    o[i] = s[i].x * q0 + s[i].y * q1 + s[i].z * q2 + s[i].w * q3;
    __stcs(reinterpret_cast<float4 *>(new_state + sbase + (row0 + i) * kD) + lane, s[i]);
  }
#pragma unroll
  for (int i = 0; i < kDecRowsPerWarp; ++i) o[i] = warp_sum(o[i]);

  if (lane == 0) {
    uint2 packed;
    packed.x = pack_bf16x2(o[0], o[1]);
    packed.y = pack_bf16x2(o[2], o[3]);
    *reinterpret_cast<uint2 *>(out + head * kD + row0) = packed;
  }
}

cudaError_t launch_decode(const void *q, const void *k, const void *v, const float *state,
                          const float *A_log, const void *a, const float *dt_bias,
                          const void *b, float scale, int64_t batch, void *out,
                          float *new_state, cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  const int64_t blocks = batch * kHV * kDecCtasPerHead;
  gdn_decode_kernel<<<static_cast<unsigned>(blocks), kDecWarps * 32, 0, stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(v), state, A_log, static_cast<const uint16_t *>(a), dt_bias,
      static_cast<const uint16_t *>(b), scale, static_cast<uint16_t *>(out), new_state);
  return cudaGetLastError();
}

}  // namespace gdn
