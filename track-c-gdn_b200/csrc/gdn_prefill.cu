// gdn_prefill.cu -- chunk-64 Gated DeltaNet prefill for sm_100a.
//
// Semantics: per sequence and v-head, the token recurrence
//     S <- g_t S ;  S <- S + beta_t (v_t - S k_t) k_t^T ;  o_t = scale S q_t
// (reference solution/triton/kernel.py:1762-1802 and the chunked kernels
// :473-1542 it calls), evaluated in the chunk-64 WY form.  With, per chunk,
//   G      chunk-local cumsum of log g          (kernel.py:1712-1722)
//   A      strict_lower(beta_i e^{G_i-G_j} K K^T)          (kernel.py:506-525)
//   Ainv   (I + A)^-1                           (kernel.py:665-737)
//   P      tril_incl(e^{G_i-G_j} Q K^T)         (kernel.py:1447-1490)
// the reference forms W = Ainv (beta e^G K) and U = Ainv (beta V) and scans
// v_new = U - W S^T (kernel.py:1179-1211).  Here the same quantity is
// re-associated so that W and U are never formed:
//   X      = beta * (V - e^G * (K S^T))
//   [O_intra ; V_new] = [P Ainv ; Ainv] X          (one M=128 MMA)
//   O      = scale * (e^G * (Q S^T) + O_intra)
//   S      = e^{G_last} S + (e^{G_last - G} V_new)^T K
// so each chunk of the sequential scan costs three dependent tensor-core
// MMAs: Y = [Q;K] S^T, Z = [PA;Ainv] X and dS = K^T V_dec.
//
// Kernels (all on the caller's stream, no host synchronisation):
//   1. gdn_prefill_meta_kernel   (1 CTA)  validates cu_seqlens, builds the
//      chunk offsets, the (sequence, chunk) table and a longest-first order
//      of sequences;
//   2. gdn_prefill_prep_kernel   (one CTA per (chunk, q/k head)) computes G,
//      beta and the 128x64 bf16 matrix [P Ainv ; Ainv] for both v-heads of the
//      q/k head, written to the workspace in the exact shared-memory image the
//      scan kernel feeds to the tensor core;
//   3. gdn_prefill_scan_kernel   (one CTA per (sequence, v-head, v-slice))
//      runs the inter-chunk scan with the fp32 state slice held in registers
//      and a bf16 copy in shared memory as the MMA operand.
#include "gdn_common.cuh"
#include "sm100.cuh"

namespace gdn {
using namespace sm100;

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct PrefillWs {
  size_t meta, chunk_off, seq_order, chunk_tab, gcum, beta, m2, total;
  int64_t nt_max;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr size_t kM2Bytes = 128 * 128;  // [PA ; Ainv] 128 rows x 64 bf16

inline PrefillWs prefill_ws_layout(int64_t T, int64_t N) {
  PrefillWs w;
  w.nt_max = (T + kChunk - 1) / kChunk + N;
  size_t off = 0;
  w.meta = off;
  off = align_up(off + 4 * sizeof(int), 256);
  w.chunk_off = off;
  off = align_up(off + (N + 1) * sizeof(int), 256);
  w.seq_order = off;
  off = align_up(off + N * sizeof(int), 256);
  w.chunk_tab = off;
  off = align_up(off + w.nt_max * sizeof(int2), 256);
  w.gcum = off;
  off = align_up(off + T * kHV * sizeof(float), 256);
  w.beta = off;
  off = align_up(off + T * kHV * sizeof(float), 1024);
  w.m2 = off;
  off = align_up(off + static_cast<size_t>(w.nt_max) * kHV * kM2Bytes, 1024);
  w.total = off;
  return w;
}

// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t lmin(int64_t x, int64_t y) { return x < y ? x : y; }

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for an mbarrier phase; gives up after ~4 s (or at once when another
// thread of the CTA already gave up), records device status 2 and returns
// false.  A CTA that gave up finishes its loop without waiting again and
// still deallocates its TMEM.
__device__ __noinline__ bool wait_phase(uint32_t mbar, uint32_t parity, volatile int *broken) {
  if (*broken) return false;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(mbar, parity)) return true;
    if (*broken) return false;
    if (globaltimer_ns() - t0 > 4000000000ull) {
      *broken = 1;
      set_device_status(kDevStatusWaitTimeout);
      return false;
    }
  }
}

// Copy rows of q (rows 0..63) and k (rows 64..127) of one chunk into the
// [Q;K] operand tile: two 64-wide d-blocks of 128 rows x 128 bytes each,
// 128-byte swizzled.  Rows past the chunk's valid length are zero.
__device__ __forceinline__ void load_qk_tile(uint8_t *qk, const uint16_t *__restrict__ q,
                                             const uint16_t *__restrict__ k, int64_t t0, int L,
                                             int hqk, int tid, int nthreads) {
  for (int idx = tid; idx < 128 * 16; idx += nthreads) {
    const int r = idx >> 4, ch = idx & 15, tok = r & 63;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (tok < L) {
      const uint16_t *src = (r < 64 ? q : k) + ((t0 + tok) * kHQK + hqk) * kD + ch * 8;
      val = __ldg(reinterpret_cast<const uint4 *>(src));
    }
    *reinterpret_cast<uint4 *>(qk + (ch >> 3) * 16384 + sw128(r, ch & 7)) = val;
  }
}

// ---------------------------------------------------------------------------
// 1. metadata
// ---------------------------------------------------------------------------
constexpr int kMetaThreads = 1024;
constexpr int kLptMaxSeqs = 2048;

__global__ void __launch_bounds__(kMetaThreads)
gdn_prefill_meta_kernel(const int64_t *__restrict__ cu, int N, int64_t T, int64_t nt_max,
                        int *meta, int *chunk_off, int *seq_order, int2 *chunk_tab) {
  __shared__ int s_wtot[32];
  __shared__ int s_carry;
  __shared__ int s_nc[kLptMaxSeqs];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  int bad = 0;
  for (int i = tid; i < N; i += kMetaThreads)
    if (cu[i + 1] < cu[i]) bad = 1;
  if (tid == 0 && (cu[0] != 0 || cu[N] != T)) bad = 1;
  if (__syncthreads_or(bad)) {
    if (tid == 0) {
      meta[0] = 0;
      meta[1] = 1;
      set_device_status(kDevStatusBadSeqlens);
    }
    return;
  }

  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < N; base += kMetaThreads) {
    const int i = base + tid;
    const int nc = i < N ? static_cast<int>((cu[i + 1] - cu[i] + kChunk - 1) / kChunk) : 0;
    if (i < N && i < kLptMaxSeqs) s_nc[i] = nc;
    int x = nc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_wtot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = s_wtot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_wtot[lane] = w;  // inclusive prefix of warp totals
    }
    __syncthreads();
    const int excl = s_carry + (warp > 0 ? s_wtot[warp - 1] : 0) + x - nc;
    if (i < N) chunk_off[i] = excl;
    __syncthreads();
    if (tid == 0) s_carry += s_wtot[31];
    __syncthreads();
  }
  const int nt = s_carry;
  if (tid == 0) {
    chunk_off[N] = nt;
    const bool ok = nt <= nt_max;
    meta[0] = ok ? nt : 0;
    meta[1] = ok ? 0 : 1;
    if (!ok) set_device_status(kDevStatusBadSeqlens);
  }
  if (nt > nt_max) return;
  __syncthreads();
  for (int i = tid; i < N; i += kMetaThreads) {
    const int off = chunk_off[i], nc = chunk_off[i + 1] - off;
    for (int c = 0; c < nc; ++c) chunk_tab[off + c] = make_int2(i, c);
  }
  // Longest-first order of sequences (ties by index) so that the scan's
  // longest recurrences start first.
  if (N <= kLptMaxSeqs) {
    for (int i = tid; i < N; i += kMetaThreads) {
      const int ni = s_nc[i];
      int r = 0;
      for (int j = 0; j < N; ++j) {
        const int nj = s_nc[j];
        r += (nj > ni) || (nj == ni && j < i);
      }
      seq_order[r] = i;
    }
  } else {
    for (int i = tid; i < N; i += kMetaThreads) seq_order[i] = i;
  }
}

// ---------------------------------------------------------------------------
// 2. chunk-parallel preparation
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 128;
// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kPrepQK = 0;         // [Q;K] tile 32 KB; later the fp32 A matrices
constexpr int kPrepPP = 32768;     // [P_0 ; P_1] bf16, K-major 128 x 64, 16 KB
constexpr int kPrepM2 = 49152;     // two [PA ; Ainv] images, 2 x 16 KB
constexpr int kPrepG = 81920;      // float G[2][64]
constexpr int kPrepB = 82432;      // float beta[2][64]
constexpr int kPrepWt = 82944;     // float warp totals[4]
constexpr int kPrepBar = 82960;    // mbarrier (8 B)
constexpr int kPrepTmem = 82968;   // TMEM base address (4 B)
constexpr int kPrepBroken = 82972; // wait-timeout flag
// + 1024 for aligning the base, + 16 KiB guard after the last operand
constexpr int kPrepSmem = 83008 + 1024 + 16384;

__global__ void __launch_bounds__(kPrepThreads)
gdn_prefill_prep_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                        const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                        const float *__restrict__ dt_bias, const uint16_t *__restrict__ b,
                        const int64_t *__restrict__ cu, const int *__restrict__ meta,
                        const int2 *__restrict__ chunk_tab, float *__restrict__ gcum_ws,
                        float *__restrict__ beta_ws, uint8_t *__restrict__ m2_ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(align_up(reinterpret_cast<size_t>(smem_raw), 1024));
  const int gchunk = blockIdx.x, hqk = blockIdx.y;
  if (meta[1] != 0 || gchunk >= meta[0]) return;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 e = chunk_tab[gchunk];
  const int64_t bos = cu[e.x];
  const int64_t t0 = bos + static_cast<int64_t>(e.y) * kChunk;
  const int L = static_cast<int>(lmin(kChunk, cu[e.x + 1] - t0));

  uint8_t *qk = smem + kPrepQK;
  uint8_t *pp = smem + kPrepPP;
  uint8_t *m2 = smem + kPrepM2;
  float *Gs = reinterpret_cast<float *>(smem + kPrepG);
  float *Bs = reinterpret_cast<float *>(smem + kPrepB);
  float *wt = reinterpret_cast<float *>(smem + kPrepWt);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + kPrepBroken);
  const uint32_t bar = smem_u32(smem + kPrepBar);

  if (warp == 0) tmem_alloc(smem_u32(smem + kPrepTmem), 256);
  if (tid == 0) {
    *broken = 0;
    mbar_init(bar, 1);
    mbar_init_fence();
  }

  load_qk_tile(qk, q, k, t0, L, hqk, tid, kPrepThreads);

  // Gates for v-heads 2*hqk + j (j = tid / 64), token t = tid % 64.
  {
    const int j = tid >> 6, t = tid & 63, hv = 2 * hqk + j;
    const bool valid = t < L;
    float gl = 0.f, bt = 0.f;
    if (valid) {
      const int64_t idx = (t0 + t) * kHV + hv;
      gl = -expf(A_log[hv]) * softplus_stable(bf16_to_f32(a[idx]) + dt_bias[hv]);
      bt = 1.0f / (1.0f + expf(-bf16_to_f32(b[idx])));
    }
    float x = gl;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wt[warp] = x;
    __syncthreads();
    if (warp & 1) x += wt[warp - 1];
    Gs[j * 64 + t] = x;
    Bs[j * 64 + t] = bt;
    if (valid) {
      const int64_t idx = (t0 + t) * kHV + hv;
      gcum_ws[idx] = x;
      beta_ws[idx] = bt;
    }
  }

  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + kPrepTmem);

  // D[128 x 64] = [Q;K] K^T : rows 0..63 Q K^T, rows 64..127 K K^T.
  if (tid == 0) {
    const uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
    const uint32_t base = smem_u32(qk);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
      umma_bf16(tmem, umma_desc_sw128(base + off, 16, 1024),
                umma_desc_sw128(base + 8192 + off, 16, 1024), idesc, ks > 0);
    }
    umma_commit(bar);
  }
  wait_phase(bar, 0, broken);
  tc_fence_after();

  {
    float acc[64];
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    tmem_ld32(trow, *reinterpret_cast<float(*)[32]>(acc));
    tmem_ld32(trow + 32, *reinterpret_cast<float(*)[32]>(acc + 32));
    tmem_wait_ld();
    const int i = (warp & 1) * 32 + lane;
    if (warp >= 2) {
      // A_j rows (fp32) into the retired [Q;K] region, 16-byte chunks
      // swizzled by (row & 15) so the row-per-thread stores do not conflict.
      float *Abuf = reinterpret_cast<float *>(smem + kPrepQK);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float Gi = Gs[j * 64 + i], bi = Bs[j * 64 + i];
        float *Arow = Abuf + (j * 64 + i) * 64;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          float vals[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = 4 * m + u;
            vals[u] = col < i ? acc[col] * expf(Gi - Gs[j * 64 + col]) * bi : 0.f;
          }
          *reinterpret_cast<float4 *>(Arow + 4 * (m ^ (i & 15))) =
              make_float4(vals[0], vals[1], vals[2], vals[3]);
        }
      }
    } else {
      // P_j rows (bf16) into the [P_0 ; P_1] operand.
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float Gi = Gs[j * 64 + i];
        const bool rv = i < L;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float vals[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int col = 8 * cc + u;
            vals[u] = (rv && col <= i) ? acc[col] * expf(Gi - Gs[j * 64 + col]) : 0.f;
          }
          uint4 pk;
          pk.x = pack_bf16x2(vals[0], vals[1]);
          pk.y = pack_bf16x2(vals[2], vals[3]);
          pk.z = pack_bf16x2(vals[4], vals[5]);
          pk.w = pack_bf16x2(vals[6], vals[7]);
          *reinterpret_cast<uint4 *>(pp + sw128(j * 64 + i, cc)) = pk;
        }
      }
    }
  }
  __syncthreads();

  // Forward substitution: thread (j, c) solves column c of (I + A_j)^-1 in
  // fp32; the rows of A_j are broadcast reads from shared memory.
  {
    const int j = tid >> 6, c = tid & 63;
    const float *Aj = reinterpret_cast<const float *>(smem + kPrepQK) + j * 64 * 64;
    float x[64];
#pragma unroll
    for (int r = 0; r < 64; ++r) x[r] = 0.f;
    if (c == 0) x[0] = 1.f;
#pragma unroll
    for (int r = 1; r < 64; ++r) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int m = 0; m < (r + 3) / 4; ++m) {
        const float4 av = *reinterpret_cast<const float4 *>(Aj + r * 64 + 4 * (m ^ (r & 15)));
        s0 += av.x * x[4 * m + 0];
        s1 += av.y * x[4 * m + 1];
        s2 += av.z * x[4 * m + 2];
        s3 += av.w * x[4 * m + 3];
      }
      x[r] = -((s0 + s1) + (s2 + s3));
      if (r == c) x[r] = 1.f;
      if (r < c) x[r] = 0.f;
    }
    // Column c of Ainv_j -> rows 64..127 of the j-th [PA ; Ainv] image.
    uint8_t *img = m2 + j * 16384;
#pragma unroll
    for (int r = 0; r < 64; ++r) {
      const uint32_t R = 64 + r;
      *reinterpret_cast<__nv_bfloat16 *>(img + R * 128 + (((c >> 3) ^ (R & 7)) << 4) +
                                         (c & 7) * 2) = __float2bfloat16_rn(x[r]);
    }
  }

  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // D_j[128 x 64] = [P_0 ; P_1] Ainv_j  (B = Ainv_j, MN-major: rows = K index).
  if (tid == 0) {
    const uint32_t idesc = umma_idesc_bf16(128, 64, false, true);
    const uint32_t pbase = smem_u32(pp);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t bbase = smem_u32(m2 + j * 16384 + 8192);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma_bf16(tmem + 64 + 64 * j, umma_desc_sw128(pbase + ks * 32, 16, 1024),
                  umma_desc_sw128(bbase + ks * 2048, 8192, 1024), idesc, ks > 0);
      }
    }
    umma_commit(bar);
  }
  wait_phase(bar, 1, broken);
  tc_fence_after();

  {
    // warps 0,1: rows 0..63 of D_0 = P_0 Ainv_0; warps 2,3: rows 64..127 of
    // D_1 = P_1 Ainv_1.
    const int j = warp >> 1, i = (warp & 1) * 32 + lane;
    float acc[64];
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64 + 64 * j;
    tmem_ld32(trow, *reinterpret_cast<float(*)[32]>(acc));
    tmem_ld32(trow + 32, *reinterpret_cast<float(*)[32]>(acc + 32));
    tmem_wait_ld();
    uint8_t *img = m2 + j * 16384;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint4 pk;
      pk.x = pack_bf16x2(acc[8 * cc + 0], acc[8 * cc + 1]);
      pk.y = pack_bf16x2(acc[8 * cc + 2], acc[8 * cc + 3]);
      pk.z = pack_bf16x2(acc[8 * cc + 4], acc[8 * cc + 5]);
      pk.w = pack_bf16x2(acc[8 * cc + 6], acc[8 * cc + 7]);
      *reinterpret_cast<uint4 *>(img + sw128(i, cc)) = pk;
    }
  }
  tc_fence_before();
  __syncthreads();

  // Both images -> workspace (image index = chunk * 8 + v-head).
  {
    uint4 *dst = reinterpret_cast<uint4 *>(m2_ws + (static_cast<size_t>(gchunk) * kHV + 2 * hqk) * kM2Bytes);
    const uint4 *src = reinterpret_cast<const uint4 *>(m2);
    for (int idx = tid; idx < 2 * 1024; idx += kPrepThreads) dst[idx] = src[idx];
  }
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// 3. sequential inter-chunk scan
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 256;

template <int VS>
struct ScanSmem {
  static constexpr int kQK = 0;                       // [Q;K] tile, 32 KB
  static constexpr int kM2 = 32768;                   // [PA ; Ainv], 16 KB
  static constexpr int kS = 49152;                    // bf16 S slice, MN-major
  static constexpr int kSGroup = 16384;               // 128 K-rows x 128 B
  static constexpr int kX = kS + (VS / 64) * kSGroup; // X / V_dec, MN-major
  static constexpr int kXGroup = 8192;                // 64 K-rows x 128 B
  static constexpr int kG = kX + (VS / 64) * kXGroup; // float G[64]
  static constexpr int kB = kG + 256;                 // float beta[64]
  static constexpr int kBar = kB + 256;
  static constexpr int kTmem = kBar + 8;
  static constexpr int kBroken = kBar + 12;
  static constexpr int kBytes = kBar + 64 + 1024 + 16384;  // align slack + guard
  static constexpr uint32_t kTmemCols = 2 * VS;
};

// Write n8 chunks of 8 bf16 (from fp32 vals) into row `row` of a 128-byte
// swizzled operand whose 64-column groups are `gstride` bytes apart,
// starting at column col0 (a multiple of 8).
template <int NV>
__device__ __forceinline__ void store_row_bf16(uint8_t *base, int row, int col0, const float *vals,
                                               int gstride) {
#pragma unroll
  for (int i = 0; i < NV / 8; ++i) {
    const int col = col0 + 8 * i;
    uint4 pk;
    pk.x = pack_bf16x2(vals[8 * i + 0], vals[8 * i + 1]);
    pk.y = pack_bf16x2(vals[8 * i + 2], vals[8 * i + 3]);
    pk.z = pack_bf16x2(vals[8 * i + 4], vals[8 * i + 5]);
    pk.w = pack_bf16x2(vals[8 * i + 6], vals[8 * i + 7]);
    *reinterpret_cast<uint4 *>(base + (col >> 6) * gstride + sw128(row, (col & 63) >> 3)) = pk;
  }
}

template <int VS>
__global__ void __launch_bounds__(kScanThreads, 1)
gdn_prefill_scan_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                        const uint16_t *__restrict__ v, const float *h0,
                        const int64_t *__restrict__ cu, const int *__restrict__ meta,
                        const int *__restrict__ chunk_off, const int *__restrict__ seq_order,
                        const float *__restrict__ gcum_ws, const float *__restrict__ beta_ws,
                        const uint8_t *__restrict__ m2_ws, float scale, uint16_t *__restrict__ out,
                        float *final_state) {
  using SM = ScanSmem<VS>;
  constexpr int NSL = kD / VS;   // v-slices per head
  constexpr int HALF = VS / 2;   // columns per thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(align_up(reinterpret_cast<size_t>(smem_raw), 1024));
  if (meta[1] != 0) return;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hc = warp >> 2;
  const int rank = blockIdx.x / (kHV * NSL);
  const int rem = blockIdx.x % (kHV * NSL);
  const int hv = rem / NSL, slice = rem % NSL;
  const int hqk = hv >> 1;
  const int n = seq_order[rank];
  const int64_t bos = cu[n];
  const int64_t len = cu[n + 1] - bos;
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);
  const int gbase = chunk_off[n];
  const int v0 = slice * VS;
  const int vcol0 = hc * HALF;          // this thread's first column within the slice
  const int drow = 32 * quad + lane;    // state k-index owned for dS / S

  uint8_t *qk = smem + SM::kQK;
  uint8_t *m2 = smem + SM::kM2;
  uint8_t *sop = smem + SM::kS;
  uint8_t *xv = smem + SM::kX;
  float *Gs = reinterpret_cast<float *>(smem + SM::kG);
  float *Bs = reinterpret_cast<float *>(smem + SM::kB);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + SM::kBroken);
  const uint32_t bar = smem_u32(smem + SM::kBar);

  if (warp == 0) tmem_alloc(smem_u32(smem + SM::kTmem), SM::kTmemCols);
  if (tid == 0) {
    *broken = 0;
    mbar_init(bar, 1);
    mbar_init_fence();
  }

  // fp32 state slice S[v0 + vcol0 + jj][drow] in registers.
  float s[HALF];
  const int64_t state_base = ((static_cast<int64_t>(n) * kHV + hv) * kD + v0 + vcol0) * kD + drow;
#pragma unroll
  for (int jj = 0; jj < HALF; ++jj) s[jj] = h0 != nullptr ? h0[state_base + jj * kD] : 0.f;
  store_row_bf16<HALF>(sop, drow, vcol0, s, SM::kSGroup);

  const uint32_t qk_s = smem_u32(qk), m2_s = smem_u32(m2), sop_s = smem_u32(sop),
                 xv_s = smem_u32(xv);
  const uint32_t idesc_y = umma_idesc_bf16(128, VS, false, true);
  const uint32_t idesc_ds = umma_idesc_bf16(128, VS, true, true);
  uint32_t phase = 0;
  uint32_t tmem = 0;

  for (int c = 0; c < nchunks; ++c) {
    const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk));
    const int64_t gidx = gbase + c;

    // ---- stage this chunk's operands ----
    load_qk_tile(qk, q, k, t0, L, hqk, tid, kScanThreads);
    {
      const uint4 *src = reinterpret_cast<const uint4 *>(m2_ws + (gidx * kHV + hv) * kM2Bytes);
      uint4 *dst = reinterpret_cast<uint4 *>(m2);
      for (int idx = tid; idx < 1024; idx += kScanThreads) dst[idx] = __ldg(src + idx);
    }
    const float g_last = gcum_ws[(t0 + L - 1) * kHV + hv];
    if (tid < 64) {
      const bool valid = tid < L;
      Gs[tid] = valid ? gcum_ws[(t0 + tid) * kHV + hv] : g_last;
      Bs[tid] = valid ? beta_ws[(t0 + tid) * kHV + hv] : 0.f;
    }
    // V row of this thread's token (quadrants 2,3), kept as packed bf16
    // pairs until X is formed; the loads overlap MMA 1.
    uint4 vpk[HALF / 8];
    const int tok = 32 * (quad & 1) + lane;
    if (quad >= 2) {
      const uint4 *src = reinterpret_cast<const uint4 *>(
          v + ((t0 + tok) * kHV + hv) * kD + v0 + vcol0);
#pragma unroll
      for (int i = 0; i < HALF / 8; ++i)
        vpk[i] = tok < L ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem = *reinterpret_cast<volatile uint32_t *>(smem + SM::kTmem);
    const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * quad) << 16);

    // ---- MMA 1: Y[128 x VS] = [Q;K] S^T ----
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
        umma_bf16(tmem, umma_desc_sw128(qk_s + aoff, 16, 1024),
                  umma_desc_sw128(sop_s + ks * 2048, SM::kSGroup, 1024), idesc_y, ks > 0);
      }
      umma_commit(bar);
    }
    wait_phase(bar, phase, broken);
    phase ^= 1;
    tc_fence_after();

    if (quad >= 2) {
      // X = beta * (V - e^G * (K S^T)) for token `tok`, 32 columns at a time
      const float eg = expf(Gs[tok]), bt = Bs[tok];
#pragma unroll
      for (int p = 0; p < HALF / 32; ++p) {
        float y[32];
        tmem_ld32(tlane + vcol0 + 32 * p, y);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 w = vpk[4 * p + i];
          const float vv[8] = {bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y),
                               bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)};
#pragma unroll
          for (int u = 0; u < 8; ++u) y[8 * i + u] = bt * (vv[u] - eg * y[8 * i + u]);
        }
        store_row_bf16<32>(xv, tok, vcol0 + 32 * p, y, SM::kXGroup);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA 2: Z[128 x VS] = [PA ; Ainv] X ----
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma_bf16(tmem + VS, umma_desc_sw128(m2_s + ks * 32, 16, 1024),
                  umma_desc_sw128(xv_s + ks * 2048, SM::kXGroup, 1024), idesc_y, ks > 0);
      }
      umma_commit(bar);
    }
    wait_phase(bar, phase, broken);
    phase ^= 1;
    tc_fence_after();

    if (quad < 2) {
      // O = scale * (e^G * (Q S^T) + P Ainv X) for token `tok`
      const float eg = expf(Gs[tok]);
      uint4 *dst = reinterpret_cast<uint4 *>(out + ((t0 + tok) * kHV + hv) * kD + v0 + vcol0);
#pragma unroll
      for (int p = 0; p < HALF / 32; ++p) {
        float y[32], z[32];
        tmem_ld32(tlane + vcol0 + 32 * p, y);
        tmem_ld32(tlane + VS + vcol0 + 32 * p, z);
        tmem_wait_ld();
        if (tok < L) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float o8[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) o8[u] = scale * (eg * y[8 * i + u] + z[8 * i + u]);
            uint4 pk;
            pk.x = pack_bf16x2(o8[0], o8[1]);
            pk.y = pack_bf16x2(o8[2], o8[3]);
            pk.z = pack_bf16x2(o8[4], o8[5]);
            pk.w = pack_bf16x2(o8[6], o8[7]);
            dst[4 * p + i] = pk;
          }
        }
      }
    } else {
      // V_dec = e^{G_last - G} * V_new, zero past the chunk's end
      const float dec = tok < L ? expf(g_last - Gs[tok]) : 0.f;
#pragma unroll
      for (int p = 0; p < HALF / 32; ++p) {
        float z[32];
        tmem_ld32(tlane + VS + vcol0 + 32 * p, z);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] *= dec;
        store_row_bf16<32>(xv, tok, vcol0 + 32 * p, z, SM::kXGroup);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA 3: dS^T[128 (k) x VS] = K^T V_dec ----
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma_bf16(tmem, umma_desc_sw128(qk_s + 8192 + ks * 2048, 16384, 1024),
                  umma_desc_sw128(xv_s + ks * 2048, SM::kXGroup, 1024), idesc_ds, ks > 0);
      }
      umma_commit(bar);
    }
    wait_phase(bar, phase, broken);
    phase ^= 1;
    tc_fence_after();
    {
      const float eg_last = expf(g_last);
#pragma unroll
      for (int p = 0; p < HALF / 32; ++p) {
        float ds[32];
        tmem_ld32(tlane + vcol0 + 32 * p, ds);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * p + i] = eg_last * s[32 * p + i] + ds[i];
        store_row_bf16<32>(sop, drow, vcol0 + 32 * p, s + 32 * p, SM::kSGroup);
      }
    }
    tc_fence_before();
    __syncthreads();
  }

#pragma unroll
  for (int jj = 0; jj < HALF; ++jj) final_state[state_base + jj * kD] = s[jj];

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem = *reinterpret_cast<volatile uint32_t *>(smem + SM::kTmem);
    tmem_dealloc(tmem, SM::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
size_t prefill_workspace_bytes(int64_t T, int64_t N) { return prefill_ws_layout(T, N).total; }

template <int VS>
static cudaError_t launch_scan(const void *q, const void *k, const void *v, const float *state,
                               const int64_t *cu, const int *meta, const int *chunk_off,
                               const int *seq_order, const float *gcum, const float *beta,
                               const uint8_t *m2, float scale, void *out, float *final_state,
                               int64_t N, cudaStream_t stream) {
  using SM = ScanSmem<VS>;
  cudaError_t err = cudaFuncSetAttribute(gdn_prefill_scan_kernel<VS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kBytes);
  if (err != cudaSuccess) return err;
  const int64_t blocks = N * kHV * (kD / VS);
  gdn_prefill_scan_kernel<VS><<<static_cast<unsigned>(blocks), kScanThreads, SM::kBytes, stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(v), state, cu, meta, chunk_off, seq_order, gcum, beta, m2,
      scale, static_cast<uint16_t *>(out), final_state);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const void *q, const void *k, const void *v, const float *state,
                           const float *A_log, const void *a, const float *dt_bias, const void *b,
                           const int64_t *cu_seqlens, int64_t N, int64_t T, float scale,
                           void *out, float *final_state, void *workspace, int num_sms,
                           cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  const PrefillWs w = prefill_ws_layout(T, N);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int *meta = reinterpret_cast<int *>(ws + w.meta);
  int *chunk_off = reinterpret_cast<int *>(ws + w.chunk_off);
  int *seq_order = reinterpret_cast<int *>(ws + w.seq_order);
  int2 *chunk_tab = reinterpret_cast<int2 *>(ws + w.chunk_tab);
  float *gcum = reinterpret_cast<float *>(ws + w.gcum);
  float *beta = reinterpret_cast<float *>(ws + w.beta);
  uint8_t *m2 = ws + w.m2;

  gdn_prefill_meta_kernel<<<1, kMetaThreads, 0, stream>>>(cu_seqlens, static_cast<int>(N), T,
                                                          w.nt_max, meta, chunk_off, seq_order,
                                                          chunk_tab);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  err = cudaFuncSetAttribute(gdn_prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPrepSmem);
  if (err != cudaSuccess) return err;
  if (w.nt_max > 0) {
    dim3 grid(static_cast<unsigned>(w.nt_max), kHQK);
    gdn_prefill_prep_kernel<<<grid, kPrepThreads, kPrepSmem, stream>>>(
        static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k), A_log,
        static_cast<const uint16_t *>(a), dt_bias, static_cast<const uint16_t *>(b), cu_seqlens,
        meta, chunk_tab, gcum, beta, m2);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  // Few recurrences: split each head's 128 v-rows over two CTAs for more
  // parallelism along the sequential scan; otherwise one CTA per head.
  const bool split = N * kHV * 2 <= static_cast<int64_t>(num_sms);
  if (split)
    return launch_scan<64>(q, k, v, state, cu_seqlens, meta, chunk_off, seq_order, gcum, beta,
                           m2, scale, out, final_state, N, stream);
  return launch_scan<128>(q, k, v, state, cu_seqlens, meta, chunk_off, seq_order, gcum, beta, m2,
                          scale, out, final_state, N, stream);
}

}  // namespace gdn
