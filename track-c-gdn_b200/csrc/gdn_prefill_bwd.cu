// gdn_prefill_bwd.cu -- backward pass of the chunked GDN prefill.
//
// No counterpart in the reference, whose prefill is forward-only
// (solution/triton/kernel.py:1).  Gradients of
//     (out, final_state) = prefill(q, k, v, h0, A_log, a, dt_bias, b)
// given d_out and d_final_state, with respect to q, k, v, a, b, A_log,
// dt_bias and h0, for the semantics the forward implements (gdn_prefill.cu).
//
// Per chunk (64 tokens, L of them valid) of one sequence and v-head, with S_0
// the state at the chunk start, G the chunk-local cumsum of log g (G_C its
// value at the last token), delta the solved values (the forward's V_new) and
// X = beta (V - e^G K S_0^T):
//   out_i = scale (e^{G_i} S_0 q_i + sum_{j<=i} P_ij delta_j),  P_ij = e^{G_i-G_j} q_i.k_j
//   S_C   = e^{G_C} S_0 + sum_j e^{G_C-G_j} delta_j k_j^T,   (I + A) delta = X,
//   A_ij  = beta_i e^{G_i-G_j} k_i.k_j (j < i).
// After a recompute of the forward that saves S_0 per chunk and delta per
// token (the prep kernel and gdn_prefill_scan_kernel<true>):
//   bwd_scan  (one CTA per (sequence, v-head), chunks in reverse order)
//             carries dS, the gradient of the chunk-end state:
//               Z   = e^{G_C-G} (dS K^T)                         [v x t]
//               dX  = scale dO^T (P Ainv) + Z Ainv               [v x t]
//               dS <- e^{G_C} dS + scale (e^G dO)^T Q - (beta e^G dX)^T K
//             and stores dS (chunk end) per chunk and dX per token;
//   bwd_chunk (one CTA per (chunk, v-head), all chunks at once):
//               dq = scale e^G (dO S_0) + Mq K
//               dk = Mq^T Q + (Ma + Ma^T) K + e^{G_C-G} (delta dS_C) - beta e^G (dX S_0)
//               dv = beta dX,  dbeta,  dG -> dg (reverse cumsum in the chunk) -> da, db
//             with Mq = scale tril_incl(e^{G_i-G_j} dO_i.delta_j) and
//                  Ma = strict_lower(-(dX_i.delta_j) beta_i e^{G_i-G_j});
//   bwd_reduce: dA_log = sum_t dg_t g_t, ddt_bias = sum_t da_t.
// The two new kernels compute in fp32 on the CUDA cores.  Every sum has a
// fixed order; dq and dk (shared by the two v-heads of a q/k head) are the
// sum of exactly two fp32 atomic additions onto zero, which is
// order-independent, so the whole backward is deterministic.

namespace gdn {

// ---------------------------------------------------------------------------
// workspace
// ---------------------------------------------------------------------------
struct PrefillBwdWs {
  PrefillWs fwd;  // the forward's layout without segmentation (prep, tables)
  size_t states, delta, dsc, dx, dgg, total;
};

inline PrefillBwdWs prefill_bwd_ws_layout(int64_t T, int64_t N) {
  PrefillBwdWs w;
  w.fwd = prefill_ws_layout(T, N, false);
  const size_t chunk_states = static_cast<size_t>(w.fwd.nt_max) * kStateBytes;
  const size_t token_vecs = static_cast<size_t>(T) * kHV * kD * sizeof(float);
  size_t off = align_up(w.fwd.total, 1024);
  w.states = off;  // fp32 [chunks][8][128][128]: state at each chunk start
  off = align_up(off + chunk_states, 1024);
  w.dsc = off;  // fp32 [chunks][8][128][128]: gradient of each chunk-end state
  off = align_up(off + chunk_states, 1024);
  w.delta = off;  // fp32 [T][8][128]
  off = align_up(off + token_vecs, 1024);
  w.dx = off;  // fp32 [T][8][128]
  off = align_up(off + token_vecs, 1024);
  w.dgg = off;  // fp32 [T][8]: dg_t * g_t
  off = align_up(off + static_cast<size_t>(T) * kHV * sizeof(float), 1024);
  w.total = off;
  return w;
}

size_t prefill_bwd_workspace_bytes(int64_t T, int64_t N) {
  return prefill_bwd_ws_layout(T, N).total;
}

__device__ __forceinline__ float bf_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// 8 bf16 -> fp32
__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  f[0] = bf_lo(u.x);
  f[1] = bf_hi(u.x);
  f[2] = bf_lo(u.y);
  f[3] = bf_hi(u.y);
  f[4] = bf_lo(u.z);
  f[5] = bf_hi(u.z);
  f[6] = bf_lo(u.w);
  f[7] = bf_hi(u.w);
}

// ---------------------------------------------------------------------------
// reverse scan over chunks
// ---------------------------------------------------------------------------
constexpr int kBwdScanThreads = 256;

struct BwdScanSmem {
  static constexpr int kK = 0;          // K tile bf16 [64 t][128 k] (q/k head of this v-head)
  static constexpr int kQ = 16384;      // Q tile bf16 [64 t][128 k]
  static constexpr int kDO = 32768;     // dO tile bf16 [64 t][128 v] (this v-head)
  static constexpr int kImg = 49152;    // [P Ainv ; Ainv] bf16 image (prep kernel output)
  static constexpr int kZX = 65536;     // Z, then dX: fp32 [64 t][128 v]
  static constexpr int kEG = 98304;     // e^{G_t} (0 past the end)
  static constexpr int kBT = kEG + 256;  // beta_t (0 past the end)
  static constexpr int kED = kBT + 256;  // e^{G_C - G_t} (0 past the end)
  static constexpr int kEGC = kED + 256;  // e^{G_C}
  static constexpr int kBytes = kEGC + 16 + 128;  // + base alignment slack
};

__global__ void __launch_bounds__(kBwdScanThreads, 2)
gdn_prefill_bwd_scan_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                            const uint16_t *__restrict__ d_out,
                            const float *__restrict__ d_final, const int64_t *__restrict__ cu,
                            const int *__restrict__ meta, const int *__restrict__ chunk_off,
                            const int *__restrict__ seq_order, const float *__restrict__ gcum_ws,
                            const float *__restrict__ beta_ws, const uint8_t *__restrict__ m2_ws,
                            float scale, float *__restrict__ dsc_ws, float *__restrict__ dx_ws,
                            float *__restrict__ d_state) {
  using SM = BwdScanSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<128>(smem_raw);
  if (meta[kMetaError] != 0) return;
  const int n = seq_order[blockIdx.x / kHV];
  const int hv = blockIdx.x % kHV, hqk = hv >> 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hc = warp >> 2, vrow = 32 * (warp & 3) + lane;
  const int64_t bos = cu[n], len = cu[n + 1] - bos;
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);
  const int gbase = chunk_off[n];
  const int64_t hv_off = static_cast<int64_t>(hv) * kD * kD;
  const int64_t srow = static_cast<int64_t>(vrow) * kD + 64 * hc;
  GDN_DCHECK(n >= 0 && n < meta[kMetaN] && gbase + nchunks <= meta[kMetaChunks]);

  const uint16_t *dOt = reinterpret_cast<const uint16_t *>(smem + SM::kDO);
  float *ZX = reinterpret_cast<float *>(smem + SM::kZX);
  float *EG = reinterpret_cast<float *>(smem + SM::kEG);
  float *BT = reinterpret_cast<float *>(smem + SM::kBT);
  float *ED = reinterpret_cast<float *>(smem + SM::kED);
  float *EGC = reinterpret_cast<float *>(smem + SM::kEGC);

  // dS[vrow][64 hc .. 64 hc + 63]
  float ds[64];
  if (d_final != nullptr) {
    const float *src = d_final + static_cast<int64_t>(n) * kHV * kD * kD + hv_off + srow;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 x = *reinterpret_cast<const float4 *>(src + 4 * i);
      ds[4 * i] = x.x;
      ds[4 * i + 1] = x.y;
      ds[4 * i + 2] = x.z;
      ds[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) ds[i] = 0.f;
  }

#pragma unroll 1
  for (int c = nchunks - 1; c >= 0; --c) {
    const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk));
    const int64_t gc = gbase + c;
    {  // the chunk-end gradient, for the chunk-parallel kernel
      float *dst = dsc_ws + gc * kHV * kD * kD + hv_off + srow;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        *reinterpret_cast<float4 *>(dst + 4 * i) =
            make_float4(ds[4 * i], ds[4 * i + 1], ds[4 * i + 2], ds[4 * i + 3]);
    }
    __syncthreads();  // the previous chunk's shared-memory reads are done
    // K, Q (q/k head hqk) and dO (v-head hv) tiles; rows past L are zero
    for (int idx = tid; idx < 3 * 64 * 16; idx += kBwdScanThreads) {
      const int which = idx >> 10, r = (idx >> 4) & 63, ch = idx & 15;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < L) {
        const uint16_t *src = which == 0   ? k + ((t0 + r) * kHQK + hqk) * kD
                              : which == 1 ? q + ((t0 + r) * kHQK + hqk) * kD
                                           : d_out + ((t0 + r) * kHV + hv) * kD;
        val = *reinterpret_cast<const uint4 *>(src + 8 * ch);
      }
      *reinterpret_cast<uint4 *>(smem + which * 16384 + r * 256 + ch * 16) = val;
    }
    {
      const uint4 *src = reinterpret_cast<const uint4 *>(m2_ws + (gc * kHV + hv) * kM2Bytes);
      uint4 *dst = reinterpret_cast<uint4 *>(smem + SM::kImg);
      for (int i = tid; i < static_cast<int>(kM2Bytes / 16); i += kBwdScanThreads) dst[i] = src[i];
    }
    if (tid < 64) {
      const float gC = gcum_ws[(t0 + L - 1) * kHV + hv];
      float eg = 0.f, bt = 0.f, ed = 0.f;
      if (tid < L) {
        const float g = gcum_ws[(t0 + tid) * kHV + hv];
        eg = expf(g);
        bt = beta_ws[(t0 + tid) * kHV + hv];
        ed = expf(gC - g);
      }
      EG[tid] = eg;
      BT[tid] = bt;
      ED[tid] = ed;
      if (tid == 0) EGC[0] = expf(gC);
    }
    __syncthreads();

    // Z[v][t] = e^{G_C - G_t} sum_k dS[v][k] K[t][k], 16 tokens at a time;
    // the two k halves meet in shared memory (stored as ZX[t][v])
#pragma unroll 1
    for (int tg = 0; tg < 4; ++tg) {
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint4 *krow =
            reinterpret_cast<const uint4 *>(smem + SM::kK + (16 * tg + j) * 256 + hc * 128);
        float a = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float kv[8];
          unpack8(krow[u], kv);
#pragma unroll
          for (int e = 0; e < 8; ++e) a += ds[8 * u + e] * kv[e];
        }
        acc[j] = a;
      }
      if (hc == 1) {
#pragma unroll
        for (int j = 0; j < 16; ++j) ZX[(16 * tg + j) * kD + vrow] = acc[j];
      }
      __syncthreads();
      if (hc == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = 16 * tg + j;
          ZX[t * kD + vrow] = ED[t] * (acc[j] + ZX[t * kD + vrow]);
        }
      }
    }
    __syncthreads();

    // dX[v][t] for t in [32 hc, 32 hc + 32):
    //   sum_i scale dO[i][v] (P Ainv)[i][t] + Z[v][i] Ainv[i][t]
    float dx[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) dx[j] = 0.f;
    const uint8_t *img = smem + SM::kImg;
#pragma unroll 1
    for (int i = 0; i < L; ++i) {
      const float a = scale * bf16_to_f32(dOt[i * kD + vrow]);
      const float z = ZX[i * kD + vrow];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float pa[8], ai[8];
        unpack8(*reinterpret_cast<const uint4 *>(img + sw128(i, 4 * hc + u)), pa);
        unpack8(*reinterpret_cast<const uint4 *>(img + sw128(64 + i, 4 * hc + u)), ai);
#pragma unroll
        for (int e = 0; e < 8; ++e) dx[8 * u + e] += a * pa[e] + z * ai[e];
      }
    }
    __syncthreads();  // every thread has read Z
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = 32 * hc + j;
      const float val = t < L ? dx[j] : 0.f;
      ZX[t * kD + vrow] = val;
      if (t < L) dx_ws[((t0 + t) * kHV + hv) * kD + vrow] = val;
    }
    __syncthreads();

    // dS <- e^{G_C} dS + sum_t (scale e^{G_t} dO[t][v]) Q[t] - (beta_t e^{G_t} dX[v][t]) K[t]
    const float egc = EGC[0];
#pragma unroll
    for (int i = 0; i < 64; ++i) ds[i] *= egc;
#pragma unroll 1
    for (int t = 0; t < L; ++t) {
      const float at = scale * EG[t] * bf16_to_f32(dOt[t * kD + vrow]);
      const float bt = BT[t] * EG[t] * ZX[t * kD + vrow];
      const uint4 *qrow = reinterpret_cast<const uint4 *>(smem + SM::kQ + t * 256 + hc * 128);
      const uint4 *krow = reinterpret_cast<const uint4 *>(smem + SM::kK + t * 256 + hc * 128);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float qv[8], kv[8];
        unpack8(qrow[u], qv);
        unpack8(krow[u], kv);
#pragma unroll
        for (int e = 0; e < 8; ++e) ds[8 * u + e] += at * qv[e] - bt * kv[e];
      }
    }
  }

  if (d_state != nullptr) {
    float *dst = d_state + static_cast<int64_t>(n) * kHV * kD * kD + hv_off + srow;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<float4 *>(dst + 4 * i) =
          make_float4(ds[4 * i], ds[4 * i + 1], ds[4 * i + 2], ds[4 * i + 3]);
  }
}

// ---------------------------------------------------------------------------
// chunk-parallel gradients
// ---------------------------------------------------------------------------
constexpr int kBwdChunkThreads = 256;
constexpr int kTP = 68;  // row pitch (floats) of the transposed [128][64] tiles
constexpr int kTT = 65;  // row pitch (floats) of the 64 x 64 matrices

struct BwdChunkSmem {
  // three transposed tiles [128 inner][64 t] (fp32, pitch kTP): first Q^T,
  // K^T; then dO^T, dX^T, delta^T
  static constexpr int kTile = 128 * kTP * 4;
  static constexpr int kR = 0;
  static constexpr int kMat = 3 * kTile;  // QK, KK|Msym, DOD|Mq, DXD|Ma: [64][kTT] fp32
  static constexpr int kMatBytes = 64 * kTT * 4;
  static constexpr int kRed = kMat + 4 * kMatBytes;  // float [3][16][64] partial dot products
  static constexpr int kVec = kRed + 3 * 16 * 64 * 4;  // per-token vectors, 64 floats each
  static constexpr int kNumVec = 16;
  static constexpr int kScalars = kVec + kNumVec * 64 * 4;  // e^{G_C}, <dS_C, S_0>, warp partials
  static constexpr int kBytes = kScalars + 64 * 4 + 128;
};
// per-token vector slots
enum BwdVec : int {
  kVG = 0, kVEG, kVBT, kVED, kVRowWq, kVColWq, kVRowWa, kVColWa, kVDbA, kVDXv, kVZeta,
  kVDG, kVDB
};

__global__ void __launch_bounds__(kBwdChunkThreads, 1)
gdn_prefill_bwd_chunk_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                             const uint16_t *__restrict__ v, const uint16_t *__restrict__ d_out,
                             const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                             const float *__restrict__ dt_bias, const int64_t *__restrict__ cu,
                             const int *__restrict__ meta, const int2 *__restrict__ chunk_tab,
                             const float *__restrict__ gcum_ws, const float *__restrict__ beta_ws,
                             const float *__restrict__ states_ws, const float *__restrict__ dsc_ws,
                             const float *__restrict__ delta_ws, const float *__restrict__ dx_ws,
                             float scale, float *__restrict__ dq, float *__restrict__ dk,
                             float *__restrict__ dv, float *__restrict__ da,
                             float *__restrict__ db, float *__restrict__ dgg_ws) {
  using SM = BwdChunkSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<128>(smem_raw);
  const int g = blockIdx.x, hv = blockIdx.y, hqk = hv >> 1;
  if (meta[kMetaError] != 0 || g >= meta[kMetaChunks]) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 e = chunk_tab[g];
  const int64_t t0 = cu[e.x] + static_cast<int64_t>(e.y) * kChunk;
  const int L = static_cast<int>(lmin(kChunk, cu[e.x + 1] - t0));
  GDN_DCHECK(e.x >= 0 && e.x < meta[kMetaN] && L > 0 && t0 + L <= meta[kMetaT]);
  const int64_t soff = (static_cast<int64_t>(g) * kHV + hv) * kD * kD;
  const float *S0 = states_ws + soff;
  const float *dSC = dsc_ws + soff;

  float *T0 = reinterpret_cast<float *>(smem + SM::kR);
  float *T1 = reinterpret_cast<float *>(smem + SM::kR + SM::kTile);
  float *T2 = reinterpret_cast<float *>(smem + SM::kR + 2 * SM::kTile);
  float *QK = reinterpret_cast<float *>(smem + SM::kMat);
  float *KK = QK + 64 * kTT;  // later Msym = Ma + Ma^T
  float *M1 = KK + 64 * kTT;  // dO_i.delta_j, then Mq
  float *M2 = M1 + 64 * kTT;  // dX_i.delta_j, then Ma
  float *RED = reinterpret_cast<float *>(smem + SM::kRed);
  float *VEC = reinterpret_cast<float *>(smem + SM::kVec);
  float *SC = reinterpret_cast<float *>(smem + SM::kScalars);
  auto vec = [&](int slot) { return VEC + slot * 64; };

  // gates of the chunk
  if (tid < 64) {
    const float gC = gcum_ws[(t0 + L - 1) * kHV + hv];
    float gg = 0.f, eg = 0.f, bt = 0.f, ed = 0.f;
    if (tid < L) {
      gg = gcum_ws[(t0 + tid) * kHV + hv];
      eg = expf(gg);
      bt = beta_ws[(t0 + tid) * kHV + hv];
      ed = expf(gC - gg);
    }
    vec(kVG)[tid] = gg;
    vec(kVEG)[tid] = eg;
    vec(kVBT)[tid] = bt;
    vec(kVED)[tid] = ed;
    if (tid == 0) SC[0] = expf(gC);
  }

  // transposed tile loads: dst[i][t] = row t of the source, 128 values;
  // a warp covers 32 consecutive tokens (conflict-free shared stores)
  auto load_t_bf16 = [&](float *dst, const uint16_t *base, int64_t stride) {
    for (int idx = tid; idx < 64 * 16; idx += kBwdChunkThreads) {
      const int t = idx & 63, ch = idx >> 6;
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (t < L) unpack8(*reinterpret_cast<const uint4 *>(base + (t0 + t) * stride + 8 * ch), f);
#pragma unroll
      for (int u = 0; u < 8; ++u) dst[(8 * ch + u) * kTP + t] = f[u];
    }
  };
  auto load_t_f32 = [&](float *dst, const float *base, int64_t stride) {
    for (int idx = tid; idx < 64 * 32; idx += kBwdChunkThreads) {
      const int t = idx & 63, ch = idx >> 6;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < L) f = *reinterpret_cast<const float4 *>(base + (t0 + t) * stride + 4 * ch);
      dst[(4 * ch + 0) * kTP + t] = f.x;
      dst[(4 * ch + 1) * kTP + t] = f.y;
      dst[(4 * ch + 2) * kTP + t] = f.z;
      dst[(4 * ch + 3) * kTP + t] = f.w;
    }
  };
  // C1 += A1 B^T, C2 += A2 B^T over 128 inner values, thread tile 4 x 4
  // (rows 4 ti.., columns 4 tj..) from transposed tiles
  const int ti = tid & 15, tj = tid >> 4;
  auto tt_products = [&](const float *A1, const float *A2, const float *B, float *C1, float *C2) {
    float c1[4][4], c2[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 4; ++s) c1[r][s] = c2[r][s] = 0.f;
#pragma unroll 4
    for (int x = 0; x < 128; ++x) {
      const float4 a1 = *reinterpret_cast<const float4 *>(A1 + x * kTP + 4 * ti);
      const float4 a2 = *reinterpret_cast<const float4 *>(A2 + x * kTP + 4 * ti);
      const float4 bb = *reinterpret_cast<const float4 *>(B + x * kTP + 4 * tj);
      const float av1[4] = {a1.x, a1.y, a1.z, a1.w}, av2[4] = {a2.x, a2.y, a2.z, a2.w};
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          c1[r][s] += av1[r] * bv[s];
          c2[r][s] += av2[r] * bv[s];
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        C1[(4 * ti + r) * kTT + 4 * tj + s] = c1[r][s];
        C2[(4 * ti + r) * kTT + 4 * tj + s] = c2[r][s];
      }
  };

  // ---- stage 1: Q K^T, K K^T ----
  load_t_bf16(T0, q + hqk * kD, kHQK * kD);
  load_t_bf16(T1, k + hqk * kD, kHQK * kD);
  __syncthreads();
  tt_products(T0, T1, T1, QK, KK);
  __syncthreads();

  // ---- stage 2: dO delta^T, dX delta^T ----
  load_t_bf16(T0, d_out + hv * kD, kHV * kD);
  load_t_f32(T1, dx_ws + hv * kD, kHV * kD);
  load_t_f32(T2, delta_ws + hv * kD, kHV * kD);
  __syncthreads();
  tt_products(T0, T1, T2, M1, M2);
  __syncthreads();

  // ---- stage 3: Mq, Ma and their gate terms (row i per thread) ----
  if (tid < 64) {
    const int i = tid;
    float rwq = 0.f, rwa = 0.f, dba = 0.f;
    const float gi = vec(kVG)[i], bi = vec(kVBT)[i];
    for (int j = 0; j < 64; ++j) {
      float mq = 0.f, ma = 0.f;
      if (i < L && j <= i) {
        const float dec = expf(gi - vec(kVG)[j]);
        mq = scale * dec * M1[i * kTT + j];
        rwq += mq * QK[i * kTT + j];
        if (j < i) {
          const float dA = -M2[i * kTT + j];
          ma = dA * bi * dec;
          rwa += ma * KK[i * kTT + j];
          dba += dA * dec * KK[i * kTT + j];
        }
      }
      M1[i * kTT + j] = mq;
      M2[i * kTT + j] = ma;
    }
    vec(kVRowWq)[i] = rwq;
    vec(kVRowWa)[i] = rwa;
    vec(kVDbA)[i] = dba;
  }
  __syncthreads();
  if (tid < 64) {  // column sums (column j per thread)
    const int j = tid;
    float cwq = 0.f, cwa = 0.f;
    for (int i = 0; i < 64; ++i) {
      cwq += M1[i * kTT + j] * QK[i * kTT + j];
      cwa += M2[i * kTT + j] * KK[i * kTT + j];
    }
    vec(kVColWq)[j] = cwq;
    vec(kVColWa)[j] = cwa;
  }
  __syncthreads();
  if (tid < 64) {  // Msym = Ma + Ma^T over K K^T (no longer needed)
    const int i = tid;
    for (int j = 0; j < 64; ++j) KK[i * kTT + j] = M2[i * kTT + j] + M2[j * kTT + i];
  }
  __syncthreads();

  // ---- stage 4: dq and dk, thread tile 4 tokens x 8 k ----
  const int tg = tid & 15, kg = tid >> 4;
  const int tr0 = 4 * tg, kc0 = 8 * kg;
  const float *dOT = T0, *dXT = T1, *DT = T2;
  const float *EGv = vec(kVEG), *BTv = vec(kVBT), *EDv = vec(kVED);
  const uint16_t *qh = q + hqk * kD + kc0;  // + token * kHQK * kD
  const uint16_t *kh = k + hqk * kD + kc0;
  auto row8 = [&](const uint16_t *base, int t, float (&f)[8]) {
    unpack8(*reinterpret_cast<const uint4 *>(base + (t0 + t) * kHQK * kD), f);
  };
  // acc = A (rows tr0..) x B[128][128] (cols kc0..), A from a transposed tile
  auto big_product = [&](const float *AT, const float *B, float (&acc)[4][8]) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int s = 0; s < 8; ++s) acc[r][s] = 0.f;
#pragma unroll 2
    for (int x = 0; x < 128; ++x) {
      const float4 av = *reinterpret_cast<const float4 *>(AT + x * kTP + tr0);
      const float4 b0 = __ldg(reinterpret_cast<const float4 *>(B + x * kD + kc0));
      const float4 b1 = __ldg(reinterpret_cast<const float4 *>(B + x * kD + kc0 + 4));
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int s = 0; s < 8; ++s) acc[r][s] += ar[r] * bs[s];
    }
  };
  // dot partials of acc rows with q or k rows -> RED[slot][kg][t]
  auto dot_partials = [&](const float (&acc)[4][8], const uint16_t *base, int slot) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = tr0 + r;
      float p = 0.f;
      if (t < L) {
        float f[8];
        row8(base, t, f);
#pragma unroll
        for (int s = 0; s < 8; ++s) p += acc[r][s] * f[s];
      }
      RED[(slot * 16 + kg) * 64 + t] = p;
    }
  };
  float acc[4][8], out[4][8];

  // dq = scale e^G (dO S_0) + Mq K
  big_product(dOT, S0, acc);
  dot_partials(acc, qh, 0);  // rho_t = q_t . (S_0^T dO_t)
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int s = 0; s < 8; ++s) out[r][s] = scale * EGv[tr0 + r] * acc[r][s];
#pragma unroll 1
  for (int j = 0; j < L; ++j) {
    float kv[8];
    row8(kh, j, kv);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float m = M1[(tr0 + r) * kTT + j];
#pragma unroll
      for (int s = 0; s < 8; ++s) out[r][s] += m * kv[s];
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (tr0 + r < L) {
      float *dst = dq + ((t0 + tr0 + r) * kHQK + hqk) * kD + kc0;
#pragma unroll
      for (int s = 0; s < 8; ++s) atomicAdd(dst + s, out[r][s]);
    }

  // dk = -beta e^G (dX S_0) + e^{G_C-G} (delta dS_C) + Mq^T Q + Msym K
  big_product(dXT, S0, acc);
  dot_partials(acc, kh, 1);  // xi_t = k_t . (S_0^T dX_t)
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int s = 0; s < 8; ++s) out[r][s] = -BTv[tr0 + r] * EGv[tr0 + r] * acc[r][s];
  big_product(DT, dSC, acc);
  dot_partials(acc, kh, 2);  // zeta_t = k_t . (dS_C^T delta_t)
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int s = 0; s < 8; ++s) out[r][s] += EDv[tr0 + r] * acc[r][s];
#pragma unroll 1
  for (int j = 0; j < L; ++j) {
    float qv[8], kv[8];
    row8(qh, j, qv);
    row8(kh, j, kv);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float mqt = M1[j * kTT + tr0 + r];   // Mq[j][t]
      const float ms = KK[(tr0 + r) * kTT + j];  // Msym[t][j]
#pragma unroll
      for (int s = 0; s < 8; ++s) out[r][s] += mqt * qv[s] + ms * kv[s];
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (tr0 + r < L) {
      float *dst = dk + ((t0 + tr0 + r) * kHQK + hqk) * kD + kc0;
#pragma unroll
      for (int s = 0; s < 8; ++s) atomicAdd(dst + s, out[r][s]);
    }

  // ---- stage 5: dv, per-token dot products, <dS_C, S_0> ----
  for (int idx = tid; idx < 64 * kD; idx += kBwdChunkThreads) {
    const int t = idx >> 7, vv = idx & 127;
    if (t < L) dv[((t0 + t) * kHV + hv) * kD + vv] = BTv[t] * dXT[vv * kTP + t];
  }
  {  // dX_t . v_t: four threads per token, 32 values each
    const int t = tid >> 2, part = tid & 3;
    float p = 0.f;
    if (t < L) {
      const uint16_t *vr = v + ((t0 + t) * kHV + hv) * kD + 32 * part;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4 *>(vr + 8 * u), f);
#pragma unroll
        for (int s = 0; s < 8; ++s) p += f[s] * dXT[(32 * part + 8 * u + s) * kTP + t];
      }
    }
    p += __shfl_xor_sync(0xffffffffu, p, 1);
    p += __shfl_xor_sync(0xffffffffu, p, 2);
    if (part == 0) vec(kVDXv)[t] = p;
  }
  {  // <dS_C, S_0>: 64 consecutive values per thread, then a fixed-order reduction
    const float4 *x = reinterpret_cast<const float4 *>(S0 + tid * 64);
    const float4 *y = reinterpret_cast<const float4 *>(dSC + tid * 64);
    float p = 0.f;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const float4 a4 = x[i], b4 = y[i];
      p += a4.x * b4.x + a4.y * b4.y + a4.z * b4.z + a4.w * b4.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if (lane == 0) SC[8 + warp] = p;
  }
  __syncthreads();
  if (tid < 64) {
    const int t = tid;
    float rho = 0.f, xi = 0.f, zeta = 0.f;
    for (int s = 0; s < 16; ++s) {
      rho += RED[(0 * 16 + s) * 64 + t];
      xi += RED[(1 * 16 + s) * 64 + t];
      zeta += RED[(2 * 16 + s) * 64 + t];
    }
    const float eg = EGv[t], bt = BTv[t], ed = EDv[t];
    float dG = 0.f, dB = 0.f;
    if (t < L) {
      dB = vec(kVDXv)[t] - eg * xi + vec(kVDbA)[t];
      dG = scale * eg * rho + vec(kVRowWq)[t] - vec(kVColWq)[t] + vec(kVRowWa)[t] -
           vec(kVColWa)[t] - bt * eg * xi - ed * zeta;
    }
    vec(kVZeta)[t] = t < L ? zeta : 0.f;
    vec(kVDG)[t] = dG;
    vec(kVDB)[t] = dB;
  }
  __syncthreads();
  if (tid == 0) {  // the chunk-end state depends on G_C
    float sds = 0.f;
    for (int w = 0; w < kBwdChunkThreads / 32; ++w) sds += SC[8 + w];
    float extra = SC[0] * sds;
    for (int j = 0; j < L; ++j) extra += EDv[j] * vec(kVZeta)[j];
    vec(kVDG)[L - 1] += extra;
  }
  __syncthreads();
  if (tid < L) {
    const int t = tid;
    float dg = 0.f;  // g_t enters every G_s, s >= t, of the chunk
    for (int s = t; s < L; ++s) dg += vec(kVDG)[s];
    const int64_t idx = (t0 + t) * kHV + hv;
    const float x = bf16_to_f32(a[idx]) + dt_bias[hv];
    const float ea = expf(A_log[hv]);
    const float sig = 1.0f / (1.0f + expf(-x));  // d softplus / dx
    const float gt = -ea * softplus_stable(x);
    const float bt = BTv[t];
    da[idx] = -dg * ea * sig;
    db[idx] = vec(kVDB)[t] * bt * (1.0f - bt);
    dgg_ws[idx] = dg * gt;
  }
}

// ---------------------------------------------------------------------------
// dA_log and ddt_bias: fixed-order sums over the tokens
// ---------------------------------------------------------------------------
constexpr int kBwdReduceThreads = 256;

__global__ void __launch_bounds__(kBwdReduceThreads)
gdn_prefill_bwd_reduce_kernel(const int *__restrict__ meta, const float *__restrict__ dgg_ws,
                              const float *__restrict__ da, int64_t T, float *__restrict__ dA_log,
                              float *__restrict__ ddt_bias) {
  __shared__ float s1[kBwdReduceThreads / 32], s2[kBwdReduceThreads / 32];
  const int hv = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float x = 0.f, y = 0.f;
  if (meta[kMetaError] == 0)
    for (int64_t t = tid; t < T; t += kBwdReduceThreads) {
      x += dgg_ws[t * kHV + hv];
      y += da[t * kHV + hv];
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    x += __shfl_xor_sync(0xffffffffu, x, o);
    y += __shfl_xor_sync(0xffffffffu, y, o);
  }
  if (lane == 0) {
    s1[warp] = x;
    s2[warp] = y;
  }
  __syncthreads();
  if (tid == 0) {
    float a1 = 0.f, a2 = 0.f;
    for (int w = 0; w < kBwdReduceThreads / 32; ++w) {
      a1 += s1[w];
      a2 += s2[w];
    }
    dA_log[hv] = a1;
    ddt_bias[hv] = a2;
  }
}

// ---------------------------------------------------------------------------
// launcher
// ---------------------------------------------------------------------------
int prefill_bwd_kernel_launches() { return 6; }

cudaError_t launch_prefill_bwd(const void *q, const void *k, const void *v, const float *state,
                               const float *A_log, const void *a, const float *dt_bias,
                               const void *b, const int64_t *cu_seqlens, int64_t N, int64_t T,
                               float scale, const void *d_out, const float *d_final, float *dq,
                               float *dk, float *dv, float *da, float *db, float *dA_log,
                               float *ddt_bias, float *d_state, void *workspace,
                               cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  const PrefillBwdWs w = prefill_bwd_ws_layout(T, N);
  const PrefillWs &f = w.fwd;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int *meta = reinterpret_cast<int *>(ws + f.meta);
  int *chunk_off = reinterpret_cast<int *>(ws + f.chunk_off);
  int *seq_order = reinterpret_cast<int *>(ws + f.seq_order);
  int2 *chunk_tab = reinterpret_cast<int2 *>(ws + f.chunk_tab);
  float *gcum = reinterpret_cast<float *>(ws + f.gcum);
  float *beta = reinterpret_cast<float *>(ws + f.beta);
  uint8_t *m2 = ws + f.m2;
  int4 *items = reinterpret_cast<int4 *>(ws + f.items);
  int *seg_off = reinterpret_cast<int *>(ws + f.seg_off);
  float *states = reinterpret_cast<float *>(ws + w.states);
  float *dsc = reinterpret_cast<float *>(ws + w.dsc);
  float *delta = reinterpret_cast<float *>(ws + w.delta);
  float *dx = reinterpret_cast<float *>(ws + w.dx);
  float *dgg = reinterpret_cast<float *>(ws + w.dgg);

  CUtensorMap tq, tk, tv;
  memset(&tq, 0, sizeof(tq));
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  if (T > 0) {
    if (!make_tmap_2d(&tq, q, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tk, k, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tv, v, kHV * kD, T, kD, 64, false))
      return cudaErrorInvalidValue;
  }
  cudaError_t err;
  if (T > 0) {
    err = cudaMemsetAsync(dq, 0, static_cast<size_t>(T) * kHQK * kD * sizeof(float), stream);
    if (err != cudaSuccess) return err;
    err = cudaMemsetAsync(dk, 0, static_cast<size_t>(T) * kHQK * kD * sizeof(float), stream);
    if (err != cudaSuccess) return err;
  }

  // recompute: tables, gates and [P Ainv ; Ainv], then the scan saving S_0 and delta
  gdn_prefill_meta_kernel<<<1, kMetaThreads, 0, stream>>>(
      cu_seqlens, static_cast<int>(N), T, f.nt_max, meta, chunk_off, seq_order, chunk_tab, 0, 0,
      items, seg_off, nullptr, 0);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(gdn_prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPrepSmem);
  if (err != cudaSuccess) return err;
  if (f.nt_max > 0) {
    dim3 grid(static_cast<unsigned>(f.nt_max), kHQK);
    gdn_prefill_prep_kernel<<<grid, kPrepThreads, kPrepSmem, stream>>>(
        tq, tk, A_log, static_cast<const uint16_t *>(a), dt_bias,
        static_cast<const uint16_t *>(b), cu_seqlens, meta, chunk_tab, gcum, beta, m2);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  err = cudaFuncSetAttribute(gdn_prefill_scan_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, ScanSmem::kBytes);
  if (err != cudaSuccess) return err;
  gdn_prefill_scan_kernel<true><<<static_cast<unsigned>(N * kHV), kScanThreads, ScanSmem::kBytes,
                                  stream>>>(
      tq, tk, tv, state, cu_seqlens, meta, chunk_off, gcum, beta, m2, scale, nullptr, nullptr,
      items, kMetaPass1, int64_t{1} << 40, seg_off, nullptr, nullptr, nullptr, nullptr, states,
      delta);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  // reverse scan
  err = cudaFuncSetAttribute(gdn_prefill_bwd_scan_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, BwdScanSmem::kBytes);
  if (err != cudaSuccess) return err;
  gdn_prefill_bwd_scan_kernel<<<static_cast<unsigned>(N * kHV), kBwdScanThreads,
                                BwdScanSmem::kBytes, stream>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
      static_cast<const uint16_t *>(d_out), d_final, cu_seqlens, meta, chunk_off, seq_order, gcum,
      beta, m2, scale, dsc, dx, d_state);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  // chunk-parallel gradients
  if (f.nt_max > 0) {
    err = cudaFuncSetAttribute(gdn_prefill_bwd_chunk_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, BwdChunkSmem::kBytes);
    if (err != cudaSuccess) return err;
    dim3 grid(static_cast<unsigned>(f.nt_max), kHV);
    gdn_prefill_bwd_chunk_kernel<<<grid, kBwdChunkThreads, BwdChunkSmem::kBytes, stream>>>(
        static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k),
        static_cast<const uint16_t *>(v), static_cast<const uint16_t *>(d_out), A_log,
        static_cast<const uint16_t *>(a), dt_bias, cu_seqlens, meta, chunk_tab, gcum, beta,
        states, dsc, delta, dx, scale, dq, dk, dv, da, db, dgg);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  gdn_prefill_bwd_reduce_kernel<<<kHV, kBwdReduceThreads, 0, stream>>>(meta, dgg, da, T, dA_log,
                                                                      ddt_bias);
  return cudaGetLastError();
}

}  // namespace gdn
