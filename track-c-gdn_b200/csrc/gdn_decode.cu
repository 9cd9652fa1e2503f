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
// even batch 16 puts 512 CTAs on the 148 SMs.  The per-row arithmetic runs
// on packed fp32 pairs (sm_100 f32x2 instructions), half the FP instructions.
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

// State element access for the fp32 state and the bf16 state variant (the
// latter: 8 bytes per lane per row, widened to fp32 on load and rounded to
// nearest even on store; all arithmetic stays fp32).
template <bool kBf16>
struct StateIO;
// Every state element is read once, by the thread that later writes it (in
// place or not), so the read-only data path is safe for the loads; plain
// loads and stores measured ~1 % faster on B200 than evict-first hints.
template <>
struct StateIO<false> {
  using T = float;
  static __device__ __forceinline__ float4 load(const float *row, int lane) {
    return __ldg(reinterpret_cast<const float4 *>(row) + lane);
  }
  static __device__ __forceinline__ void store(float *row, int lane, float4 x) {
    reinterpret_cast<float4 *>(row)[lane] = x;
  }
  static __device__ __forceinline__ float4 round(float4 x) { return x; }
};
template <>
struct StateIO<true> {
  using T = uint16_t;
  static __device__ __forceinline__ float4 load(const uint16_t *row, int lane) {
    const uint2 r = __ldg(reinterpret_cast<const uint2 *>(row) + lane);
    return make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
  }
  static __device__ __forceinline__ void store(uint16_t *row, int lane, float4 x) {
    reinterpret_cast<uint2 *>(row)[lane] = make_uint2(pack_bf16x2(x.x, x.y), pack_bf16x2(x.z, x.w));
  }
  // the value a bf16 state holds after a store
  static __device__ __forceinline__ float4 round(float4 x) {
    const uint32_t lo = pack_bf16x2(x.x, x.y), hi = pack_bf16x2(x.z, x.w);
    return make_float4(bf16_lo(lo), bf16_hi(lo), bf16_lo(hi), bf16_hi(hi));
  }
};

// Sums v[i] (one value per state row, i < 8) across the warp with a
// transposing butterfly: at offsets 16, 8 and 4 each lane keeps half of its
// values and adds the partner's half, then offsets 2 and 1 finish the sum --
// 9 shuffles instead of 8 x 5.  Every lane returns the total of row
// (lane >> 2) & 7.  Each row's additions pair the same lanes at the same
// offsets as warp_sum, and fp32 addition is commutative, so the totals equal
// warp_sum's bit for bit.
__device__ __forceinline__ float warp_sum8_transposed(const float (&v)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float send = b4 ? v[j] : v[j + 4];
    const float keep = b4 ? v[j + 4] : v[j];
    w[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float x[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float send = b3 ? w[j] : w[j + 2];
    const float keep = b3 ? w[j + 2] : w[j];
    x[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float send = b2 ? x[0] : x[1];
  const float keep = b2 ? x[1] : x[0];
  float y = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  y += __shfl_xor_sync(0xffffffffu, y, 2);
  y += __shfl_xor_sync(0xffffffffu, y, 1);
  return y;
}
// One lane's slice of a state row, k = 4 lane .. 4 lane + 3, as two packed
// fp32 pairs (x, y) and (z, w).  Both decode kernels do their per-row
// arithmetic through the two functions below, so the multi-token kernel
// stays bit-identical to repeated single-token steps.
struct RowSlice {
  uint64_t xy, zw;
};

__device__ __forceinline__ RowSlice to_slice(float4 x) {
  return RowSlice{f2_pack(x.x, x.y), f2_pack(x.z, x.w)};
}
__device__ __forceinline__ float4 to_float4(const RowSlice &r) {
  return make_float4(f2_lo(r.xy), f2_hi(r.xy), f2_lo(r.zw), f2_hi(r.zw));
}

// h = g S (in place) and this lane's part of h . k: (x k0 + z k2) + (y k1 + w k3).
__device__ __forceinline__ float decay_dot(RowSlice &s, uint64_t gg, uint64_t kxy, uint64_t kzw) {
  s.xy = f2_mul(s.xy, gg);
  s.zw = f2_mul(s.zw, gg);
  const uint64_t t = f2_fma(s.zw, kzw, f2_mul(s.xy, kxy));
  return f2_lo(t) + f2_hi(t);
}

// S' = h + delta k (in place) and this lane's part of S' . (scale q).
__device__ __forceinline__ float update_dot(RowSlice &s, float delta, uint64_t kxy, uint64_t kzw,
                                            uint64_t qxy, uint64_t qzw) {
  const uint64_t dd = f2_pack(delta, delta);
  s.xy = f2_fma(kxy, dd, s.xy);
  s.zw = f2_fma(kzw, dd, s.zw);
  const uint64_t t = f2_fma(s.zw, qzw, f2_mul(s.xy, qxy));
  return f2_lo(t) + f2_hi(t);
}

// q (scaled) and k of this lane's four k-columns as packed pairs.
__device__ __forceinline__ void qk_pairs(uint2 qr, uint2 kr, float scale, uint64_t &qxy,
                                         uint64_t &qzw, uint64_t &kxy, uint64_t &kzw) {
  qxy = f2_pack(bf16_lo(qr.x) * scale, bf16_hi(qr.x) * scale);
  qzw = f2_pack(bf16_lo(qr.y) * scale, bf16_hi(qr.y) * scale);
  kxy = f2_pack(bf16_lo(kr.x), bf16_hi(kr.x));
  kzw = f2_pack(bf16_lo(kr.y), bf16_hi(kr.y));
}

// Single-token step, templated on the state format (fp32 or bf16 storage)
// and the rows per warp R: fp32 uses R = 4 (32 rows per CTA, 4 CTAs per
// head); the bf16 state uses R = 8, so a warp still keeps 2 KiB of state in
// flight, and reduces its rows with the transposing butterfly (same sums, bit
// for bit, as one warp_sum per row).
template <bool kBf16, int R>
__global__ void __launch_bounds__(kDecWarps * 32)
gdn_decode_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                  const uint16_t *__restrict__ v, const typename StateIO<kBf16>::T *state,
                  const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                  const float *__restrict__ dt_bias, const uint16_t *__restrict__ b,
                  float scale, uint16_t *__restrict__ out, typename StateIO<kBf16>::T *new_state,
                  const int32_t *__restrict__ slots, int64_t pool_slots) {
  using IO = StateIO<kBf16>;
  static_assert(R == 4 || R == 8, "4 or 8 rows per warp");
  constexpr int kRowsPerCta = kDecWarps * R;
  constexpr int kCtasPerHead = kD / kRowsPerCta;
  const int64_t head = blockIdx.x / kCtasPerHead;  // request * 8 + v-head
  const int part = blockIdx.x % kCtasPerHead;
  const int64_t req = head / kHV;
  const int hv = static_cast<int>(head % kHV);
  const int hqk = hv >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = part * kRowsPerCta + warp * R;  // first v index
  // state of this request: dense (row req) or a slot of a state pool
  const int64_t sreq = slots != nullptr ? slots[req] : req;
  if (slots != nullptr && (sreq < 0 || sreq >= pool_slots)) {
    if (threadIdx.x == 0) set_device_status(kDevStatusBadSlot);
    return;
  }
  const int64_t sbase = (sreq * kHV + hv) * kD * kD;

  // Issue the state loads first: they are the long-latency part.
  float4 s4[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    if (state != nullptr) {
      s4[i] = IO::load(state + sbase + (row0 + i) * kD, lane);
    } else {
      s4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  // Lane l owns k-columns 4l .. 4l+3.
  const int64_t qk_off = (req * kHQK + hqk) * kD + 4 * lane;
  uint64_t qxy, qzw, kxy, kzw;
  qk_pairs(*reinterpret_cast<const uint2 *>(q + qk_off), *reinterpret_cast<const uint2 *>(k + qk_off),
           scale, qxy, qzw, kxy, kzw);

  // Gates (kernel.py:59-65).
  const float a_val = bf16_to_f32(a[head]);
  const float b_val = bf16_to_f32(b[head]);
  const float g = expf(-expf(A_log[hv]) * softplus_thr20(a_val + dt_bias[hv]));
  const float beta = 1.0f / (1.0f + expf(-b_val));
  const uint64_t gg = f2_pack(g, g);

  // v values of this warp's rows (row0 is a multiple of 4: 8-byte loads).
  float vv[R];
#pragma unroll
  for (int h = 0; h < R / 4; ++h) {
    const uint2 vr = *reinterpret_cast<const uint2 *>(v + head * kD + row0 + 4 * h);
    vv[4 * h] = bf16_lo(vr.x);
    vv[4 * h + 1] = bf16_hi(vr.x);
    vv[4 * h + 2] = bf16_lo(vr.y);
    vv[4 * h + 3] = bf16_hi(vr.y);
  }

  RowSlice s[R];
  float old[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    s[i] = to_slice(s4[i]);
    old[i] = decay_dot(s[i], gg, kxy, kzw);
  }
  if constexpr (R == 8) {
    const float tot = warp_sum8_transposed(old, lane);
#pragma unroll
    for (int i = 0; i < R; ++i) old[i] = __shfl_sync(0xffffffffu, tot, 4 * i);
  } else {
#pragma unroll
    for (int i = 0; i < R; ++i) old[i] = warp_sum(old[i]);
  }

  float o[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const float delta = beta * (vv[i] - old[i]);
    o[i] = update_dot(s[i], delta, kxy, kzw, qxy, qzw);
    IO::store(new_state + sbase + (row0 + i) * kD, lane, to_float4(s[i]));
  }
  if constexpr (R == 8) {
    const float tot = warp_sum8_transposed(o, lane);  // lanes 4 i hold row i's output
    if ((lane & 3) == 0)
      out[head * kD + row0 + (lane >> 2)] = __bfloat16_as_ushort(__float2bfloat16_rn(tot));
  } else {
#pragma unroll
    for (int i = 0; i < R; ++i) o[i] = warp_sum(o[i]);
    if (lane == 0) {
      uint2 packed;
      packed.x = pack_bf16x2(o[0], o[1]);
      packed.y = pack_bf16x2(o[2], o[3]);
      *reinterpret_cast<uint2 *>(out + head * kD + row0) = packed;
    }
  }
}

// Multi-token decode (speculative verify / MTP): T tokens per request, the
// same step applied T times in order -- exactly T calls of the single-token
// kernel above (same fp32 operations in the same order), with the state kept
// in registers between tokens.  State traffic is that of one step (64 KiB in
// + 64 KiB out per head); each extra token adds only its vectors.  Because a
// CTA now lives through T tokens' dependent reductions, each warp owns 8 rows
// (a CTA 64 rows, 2 CTAs per head): twice the state bytes in flight per CTA
// and 8 independent reduction chains to interleave, which keeps the kernel
// on the HBM roofline.  Token t of request r is row r * T + t of the [B*T, ...]
// inputs and outputs.  `inter` (optional) receives the state after every
// token, [B, T, 8, 128, 128] fp32, for rolling back rejected tokens.  All T
// tokens' vectors for the CTA (q, k of its q/k head, v of its 64 rows, a, b:
// ~0.6 KiB per token) are staged into shared memory in one round trip that
// overlaps the state loads, so the token loop never waits on global memory.
constexpr int kMtpRowsPerWarp = 8;

constexpr int kMtpRowsPerCta = kDecWarps * kMtpRowsPerWarp;  // 64
constexpr int kMtpCtasPerHead = kD / kMtpRowsPerCta;         // 2

// kInter: the per-token states are written (`inter` non-null); the
// instantiation without them keeps that pointer and its addressing out of the
// token loop's registers.
template <bool kBf16State, bool kInter>
__global__ void __launch_bounds__(kDecWarps * 32, 4)
gdn_decode_mtp_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                      const uint16_t *__restrict__ v,
                      const typename StateIO<kBf16State>::T *state,
                      const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                      const float *__restrict__ dt_bias, const uint16_t *__restrict__ b,
                      float scale, int T, uint16_t *__restrict__ out,
                      typename StateIO<kBf16State>::T *new_state,
                      typename StateIO<kBf16State>::T *__restrict__ inter,
                      const int32_t *__restrict__ slots, int64_t pool_slots) {
  using IO = StateIO<kBf16State>;
  constexpr int R = kMtpRowsPerWarp;
  const int64_t head = blockIdx.x / kMtpCtasPerHead;  // request * 8 + v-head
  const int part = blockIdx.x % kMtpCtasPerHead;
  const int64_t req = head / kHV;
  const int hv = static_cast<int>(head % kHV);
  const int hqk = hv >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = part * kMtpRowsPerCta + warp * R;
  const int64_t sreq = slots != nullptr ? slots[req] : req;
  if (slots != nullptr && (sreq < 0 || sreq >= pool_slots)) {
    if (threadIdx.x == 0) set_device_status(kDevStatusBadSlot);
    return;
  }
  const int64_t sbase = (sreq * kHV + hv) * kD * kD;

  RowSlice s[R];
#pragma unroll
  for (int i = 0; i < R; ++i)
    s[i] = to_slice(state != nullptr ? IO::load(state + sbase + (row0 + i) * kD, lane)
                                     : make_float4(0.f, 0.f, 0.f, 0.f));

  // Stage every token's vectors (8-byte pieces: q/k/v are only guaranteed
  // 8-byte aligned): per token 32 + 32 pieces of q, k, 16 of v (this CTA's 64
  // rows); and each token's gates g and beta, computed once here rather than
  // by every warp (the same expressions as the single-token kernel).
  extern __shared__ uint2 mtp_smem[];
  uint2 *qs = mtp_smem;                 // [T][32]
  uint2 *ks = qs + 32 * T;              // [T][32]
  uint2 *vs = ks + 32 * T;              // [T][16]
  float *gs = reinterpret_cast<float *>(vs + 16 * T);  // [T][2]: g, beta
  for (int idx = threadIdx.x; idx < 80 * T; idx += kDecWarps * 32) {
    const int t = idx / 80, p = idx % 80;
    const int64_t tok = req * T + t;
    if (p < 32) {
      qs[t * 32 + p] = reinterpret_cast<const uint2 *>(q + (tok * kHQK + hqk) * kD)[p];
    } else if (p < 64) {
      ks[t * 32 + p - 32] = reinterpret_cast<const uint2 *>(k + (tok * kHQK + hqk) * kD)[p - 32];
    } else {
      vs[t * 16 + p - 64] = reinterpret_cast<const uint2 *>(
          v + (tok * kHV + hv) * kD + part * kMtpRowsPerCta)[p - 64];
    }
  }
  for (int t = threadIdx.x; t < T; t += kDecWarps * 32) {
    const int64_t tok = req * T + t;
    const float a_val = bf16_to_f32(a[tok * kHV + hv]);
    const float b_val = bf16_to_f32(b[tok * kHV + hv]);
    gs[2 * t] = expf(-expf(A_log[hv]) * softplus_thr20(a_val + dt_bias[hv]));
    gs[2 * t + 1] = 1.0f / (1.0f + expf(-b_val));
  }
  __syncthreads();

  for (int t = 0; t < T; ++t) {
    const uint2 v0 = vs[t * 16 + 2 * warp], v1 = vs[t * 16 + 2 * warp + 1];
    const float2 gb = *reinterpret_cast<const float2 *>(gs + 2 * t);
    const int64_t tok = req * T + t;
    uint64_t qxy, qzw, kxy, kzw;
    qk_pairs(qs[t * 32 + lane], ks[t * 32 + lane], scale, qxy, qzw, kxy, kzw);
    const uint64_t gg = f2_pack(gb.x, gb.x);
    const float beta = gb.y;
    const float vv[R] = {bf16_lo(v0.x), bf16_hi(v0.x), bf16_lo(v0.y), bf16_hi(v0.y),
                         bf16_lo(v1.x), bf16_hi(v1.x), bf16_lo(v1.y), bf16_hi(v1.y)};

    float old[R];
#pragma unroll
    for (int i = 0; i < R; ++i) old[i] = decay_dot(s[i], gg, kxy, kzw);
    {
      const float tot = warp_sum8_transposed(old, lane);
#pragma unroll
      for (int i = 0; i < R; ++i) old[i] = __shfl_sync(0xffffffffu, tot, 4 * i);
    }

    float o[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const float delta = beta * (vv[i] - old[i]);
      o[i] = update_dot(s[i], delta, kxy, kzw, qxy, qzw);
      if constexpr (kInter)
        IO::store(inter + ((tok * kHV + hv) * kD + row0 + i) * kD, lane, to_float4(s[i]));
      // a bf16 state carries its rounded value into the next token, as T
      // separate steps would (the output above used the unrounded update)
      if constexpr (kBf16State) s[i] = to_slice(IO::round(to_float4(s[i])));
    }
    {
      // lanes 4 i hold row i's output
      const float tot = warp_sum8_transposed(o, lane);
      if ((lane & 3) == 0)
        out[(tok * kHV + hv) * kD + row0 + (lane >> 2)] =
            __bfloat16_as_ushort(__float2bfloat16_rn(tot));
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) IO::store(new_state + sbase + (row0 + i) * kD, lane, to_float4(s[i]));
}

cudaError_t launch_decode_mtp(const void *q, const void *k, const void *v, const float *state,
                              const float *A_log, const void *a, const float *dt_bias,
                              const void *b, float scale, int64_t batch, int num_tokens,
                              void *out, float *new_state, float *inter, const int32_t *slots,
                              int64_t pool_slots, cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  const int64_t blocks = batch * kHV * kMtpCtasPerHead;
  const size_t smem = static_cast<size_t>(num_tokens) * (80 * sizeof(uint2) + 2 * sizeof(float));
  auto kernel = inter != nullptr ? gdn_decode_mtp_kernel<false, true>
                                 : gdn_decode_mtp_kernel<false, false>;
  kernel<<<static_cast<unsigned>(blocks), kDecWarps * 32, smem, stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(v), state, A_log, static_cast<const uint16_t *>(a), dt_bias,
      static_cast<const uint16_t *>(b), scale, num_tokens, static_cast<uint16_t *>(out),
      new_state, inter, slots, pool_slots);
  return cudaGetLastError();
}

// bf16 state variant: T >= 1 tokens, state (dense [B,8,128,128] or a pool with
// slots) updated in place in bf16.
cudaError_t launch_decode_bf16_state(const void *q, const void *k, const void *v, void *state,
                                     const float *A_log, const void *a, const float *dt_bias,
                                     const void *b, float scale, int64_t batch, int num_tokens,
                                     void *out, const int32_t *slots, int64_t pool_slots,
                                     cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  uint16_t *st = static_cast<uint16_t *>(state);
  if (num_tokens == 1) {
    const int64_t blocks = batch * kHV * (kD / (kDecWarps * 8));
    gdn_decode_kernel<true, 8><<<static_cast<unsigned>(blocks), kDecWarps * 32, 0, stream>>>(
        static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
        static_cast<const uint16_t *>(v), st, A_log, static_cast<const uint16_t *>(a), dt_bias,
        static_cast<const uint16_t *>(b), scale, static_cast<uint16_t *>(out), st, slots,
        pool_slots);
    return cudaGetLastError();
  }
  const int64_t blocks = batch * kHV * kMtpCtasPerHead;
  const size_t smem = static_cast<size_t>(num_tokens) * (80 * sizeof(uint2) + 2 * sizeof(float));
  gdn_decode_mtp_kernel<true, false><<<static_cast<unsigned>(blocks), kDecWarps * 32, smem, stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(v), st, A_log, static_cast<const uint16_t *>(a), dt_bias,
      static_cast<const uint16_t *>(b), scale, num_tokens, static_cast<uint16_t *>(out), st,
      nullptr, slots, pool_slots);
  return cudaGetLastError();
}

cudaError_t launch_decode(const void *q, const void *k, const void *v, const float *state,
                          const float *A_log, const void *a, const float *dt_bias,
                          const void *b, float scale, int64_t batch, void *out,
                          float *new_state, const int32_t *slots, int64_t pool_slots,
                          cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  const int64_t blocks = batch * kHV * kDecCtasPerHead;
  gdn_decode_kernel<false, kDecRowsPerWarp><<<static_cast<unsigned>(blocks), kDecWarps * 32, 0,
                                              stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(v), state, A_log, static_cast<const uint16_t *>(a), dt_bias,
      static_cast<const uint16_t *>(b), scale, static_cast<uint16_t *>(out), new_state, slots,
      pool_slots);
  return cudaGetLastError();
}

}  // namespace gdn
