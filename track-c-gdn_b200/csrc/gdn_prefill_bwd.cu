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
//             and stores dS (chunk end) per chunk, dX per token (a bf16
//             operand image) and dv = beta dX;
//   bwd_chunk (persistent; per (chunk, v-head), all chunks at once):
//               dq = scale e^G (dO S_0) + Mq K
//               dk = Mq^T Q + (Ma + Ma^T) K + e^{G_C-G} (delta dS_C) - beta e^G (dX S_0)
//               dbeta,  dG -> dg (reverse cumsum in the chunk) -> da, db
//             with Mq = scale tril_incl(e^{G_i-G_j} dO_i.delta_j) and
//                  Ma = strict_lower(-(dX_i.delta_j) beta_i e^{G_i-G_j});
//   bwd_reduce (two fixed-order stages): dA_log = sum_t dg_t g_t,
//             ddt_bias = sum_t da_t.
// Both kernels run their products on the tensor cores (bf16 operands, fp32
// accumulators, as the forward) and the rest in fp32; the state gradient
// itself is carried in fp32.  Every sum has a
// fixed order; dq and dk (shared by the two v-heads of a q/k head) are one
// fp32 addition of the two v-heads' contributions, exchanged between the two
// CTAs of a cluster, so the whole backward is deterministic.

namespace gdn {

// ---------------------------------------------------------------------------
// workspace
// ---------------------------------------------------------------------------
// token blocks of the first stage of the dA_log / ddt_bias reduction
constexpr int kBwdRedBlocks = 256;

struct PrefillBwdWs {
  PrefillWs fwd;  // the forward's layout without segmentation (prep, tables)
  size_t states, delta, dsc, dx, dgg, red, total;
};

inline PrefillBwdWs prefill_bwd_ws_layout(int64_t T, int64_t N) {
  PrefillBwdWs w;
  w.fwd = prefill_ws_layout(T, N, false);
  const size_t chunk_states = static_cast<size_t>(w.fwd.nt_max) * kHV * kStateImgBytes;
  const size_t chunk_toks = static_cast<size_t>(w.fwd.nt_max) * kHV * kTokImgBytes;
  size_t off = align_up(w.fwd.total, 1024);
  w.states = off;  // [chunks][8] bf16 images (put_state_img_row): state at each chunk start
  off = align_up(off + chunk_states, 1024);
  w.dsc = off;  // [chunks][8] bf16 images: gradient of each chunk-end state
  off = align_up(off + chunk_states, 1024);
  w.delta = off;  // [chunks][8] token images (put_tok_img): delta
  off = align_up(off + chunk_toks, 1024);
  w.dx = off;  // [chunks][8] token images: dX
  off = align_up(off + chunk_toks, 1024);
  w.dgg = off;  // fp32 [T][8]: dg_t * g_t
  off = align_up(off + static_cast<size_t>(T) * kHV * sizeof(float), 1024);
  w.red = off;  // fp32 [kBwdRedBlocks][8][2]: per-block partial sums of dg g and da
  off = align_up(off + static_cast<size_t>(kBwdRedBlocks) * kHV * 2 * sizeof(float), 1024);
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
// reverse scan over chunks (tcgen05)
// ---------------------------------------------------------------------------
// One CTA (256 threads) per (sequence, v-head).  Thread (vrow, hc) keeps
// dS[vrow][64 hc .. 64 hc + 63] in fp32 registers; a bf16 copy in TMEM
// (columns 0..63) is the A operand of MMA a.  Per chunk, three dependent
// MMAs (bf16 operands, fp32 accumulators):
//   a:  Zr = dS K^T                                    [v x t]  cols 128..191
//   b:  dX / scale = dO^T (P Ainv) + (Z / scale) Ainv  [v x t]  cols 192..255
//   c:  dS' = dO^T Q' - (beta e^G dX) K                [v x k]  cols 128..255
// with Z = e^{G_C - G} Zr and Q' = scale e^G Q (built in place over the Q
// tile); dO, the image and Q', K enter MMAs b and c as MN-major operands,
// Z / scale and -beta e^G dX as bf16 A operands in TMEM (columns 64..127).
// Then dS <- e^{G_C} dS + dS'.
constexpr int kBwdScanThreads = 256;

struct BwdScanSmem {
  static constexpr int kQ = 0;        // Q tile, then Q' in place: 2 d-blocks x 64 t x 128 B
  static constexpr int kK0 = 16384;   // K tiles, double buffered (chunks in reverse order)
  static constexpr int kK1 = 32768;
  static constexpr int kDO = 49152;   // dO tile: 2 v-blocks x 64 t x 128 B
  static constexpr int kImg = 65536;  // [P Ainv ; Ainv] image, 128 rows x 128 B
  static constexpr int kEG = 81920;   // e^{G_t} (0 past the end)
  static constexpr int kBT = kEG + 256;   // beta_t (0 past the end)
  static constexpr int kED = kBT + 256;   // e^{G_C - G_t} (0 past the end)
  static constexpr int kEGC = kED + 256;  // e^{G_C}
  static constexpr int kBar = kEGC + 16;  // mma, q, do, img, k0, k1
  static constexpr int kTmem = kBar + 48;
  static constexpr int kBroken = kBar + 52;
  static constexpr int kBytes = kBar + 64 + 1024;  // + base alignment slack
  static constexpr uint32_t kTmemCols = 256;
  // bf16 Z / scale, then -beta e^G dX: the TMEM A operand of MMAs b and c
  // (thread half hc: columns kColZX + 32 hc .. + 15, two tokens per column)
  static constexpr uint32_t kColSb = 0, kColZX = 64, kColA = 128, kColB = 192;
};

__global__ void __launch_bounds__(kBwdScanThreads, 2)
gdn_prefill_bwd_scan_kernel(const __grid_constant__ CUtensorMap tmap_q,
                            const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_do,
                            const float *__restrict__ d_final, const int64_t *__restrict__ cu,
                            const int *__restrict__ meta, const int *__restrict__ chunk_off,
                            const int *__restrict__ seq_order, const float *__restrict__ gcum_ws,
                            const float *__restrict__ beta_ws, const uint8_t *__restrict__ m2_ws,
                            float scale, uint8_t *__restrict__ dsc_ws, uint8_t *__restrict__ dx_ws,
                            float *__restrict__ dv, float *__restrict__ d_state) {
  using SM = BwdScanSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  if (meta[kMetaError] != 0) return;
  const int n = seq_order[blockIdx.x / kHV];
  const int hv = blockIdx.x % kHV, hqk = hv >> 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hc = warp >> 2, vrow = 32 * quad + lane;
  const int64_t bos = cu[n], len = cu[n + 1] - bos;
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);
  const int gbase = chunk_off[n];
  const int64_t hv_off = static_cast<int64_t>(hv) * kD * kD;
  const int64_t srow = static_cast<int64_t>(vrow) * kD + 64 * hc;
  GDN_DCHECK(n >= 0 && n < meta[kMetaN] && gbase + nchunks <= meta[kMetaChunks]);

  float *EG = reinterpret_cast<float *>(smem + SM::kEG);
  float *BT = reinterpret_cast<float *>(smem + SM::kBT);
  float *ED = reinterpret_cast<float *>(smem + SM::kED);
  float *EGC = reinterpret_cast<float *>(smem + SM::kEGC);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + SM::kBroken);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_mma = s_base + SM::kBar, bar_q = bar_mma + 8, bar_do = bar_mma + 16,
                 bar_img = bar_mma + 24, bar_k0 = bar_mma + 32;  // bar_k1 = bar_k0 + 8

  auto chunk_t0 = [&](int c) { return static_cast<int>(bos + static_cast<int64_t>(c) * kChunk); };
  auto issue_tile2 = [&](const void *tm, uint32_t dst, int x, int c, uint32_t bar) {
    mbar_arrive_expect_tx(bar, 16384);
    tma_load_2d(dst, tm, x, chunk_t0(c), bar);
    tma_load_2d(dst + 8192, tm, x + 64, chunk_t0(c), bar);
  };
  auto issue_img = [&](int c) {
    mbar_arrive_expect_tx(bar_img, static_cast<uint32_t>(kM2Bytes));
    bulk_load(s_base + SM::kImg, m2_ws + (static_cast<int64_t>(gbase + c) * kHV + hv) * kM2Bytes,
              static_cast<uint32_t>(kM2Bytes), bar_img);
  };

  if (warp == 0) tmem_alloc(s_base + SM::kTmem, SM::kTmemCols);
  if (tid == 0) {
    *broken = 0;
    for (int i = 0; i < 6; ++i) mbar_init(bar_mma + 8 * i, 1);
    mbar_init_fence();
    if (nchunks > 0) {
      const int c = nchunks - 1;
      issue_tile2(&tmap_q, s_base + SM::kQ, hqk * kD, c, bar_q);
      issue_tile2(&tmap_do, s_base + SM::kDO, hv * kD, c, bar_do);
      issue_img(c);
      issue_tile2(&tmap_k, s_base + ((c & 1) ? SM::kK1 : SM::kK0), hqk * kD, c, bar_k0 + 8 * (c & 1));
      if (c > 0)
        issue_tile2(&tmap_k, s_base + (((c - 1) & 1) ? SM::kK1 : SM::kK0), hqk * kD, c - 1,
                    bar_k0 + 8 * ((c - 1) & 1));
    }
  }

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
  __syncthreads();  // barriers initialised, TMEM address published
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + SM::kTmem);
  const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * quad) << 16);
  auto put_sb = [&]() {  // bf16 copy of dS -> TMEM columns 32 hc .. 32 hc + 31
    uint32_t pk[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pk[j] = pack_bf16x2(ds[2 * j], ds[2 * j + 1]);
    tmem_st32(tlane + SM::kColSb + 32 * hc, pk);
    tmem_wait_st();
  };
  put_sb();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t id_a = umma_idesc_bf16(128, 64, false, false);
  const uint32_t id_b1 = umma_idesc_bf16(128, 64, true, true);
  const uint32_t id_b2 = umma_idesc_bf16(128, 64, false, true);
  const uint32_t id_c1 = umma_idesc_bf16(128, 128, true, true);
  const uint32_t id_c2 = umma_idesc_bf16(128, 128, false, true);
  const float inv_scale = 1.0f / scale;
  uint32_t ph_mma = 0, ph_q = 0, ph_do = 0, ph_img = 0, ph_k = 0;

#pragma unroll 1
  for (int c = nchunks - 1; c >= 0; --c) {
    const int cb = c & 1;
    const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk));
    const int64_t gc = gbase + c;
    const uint32_t kbuf = s_base + (cb ? SM::kK1 : SM::kK0);
    // the chunk-end gradient, as the chunk-parallel kernel's operand image
    put_state_img_row(dsc_ws + (gc * kHV + hv) * kStateImgBytes, vrow, hc, ds);
    if (tid < 64) {
      const float gC = gcum_ws[(t0 + L - 1) * kHV + hv];
      float eg = 0.f, bt = 0.f, ed = 0.f;
      if (tid < L) {
        const float gg = gcum_ws[(t0 + tid) * kHV + hv];
        eg = expf(gg);
        bt = beta_ws[(t0 + tid) * kHV + hv];
        ed = expf(gC - gg);
      }
      EG[tid] = eg;
      BT[tid] = bt;
      ED[tid] = ed;
      if (tid == 0) EGC[0] = expf(gC);
    }
    // every thread sees this chunk's tiles land once; the next loads into
    // each buffer are issued only after a later __syncthreads
    wait_phase(bar_k0 + 8 * cb, (ph_k >> cb) & 1, broken);
    ph_k ^= 1u << cb;
    wait_phase(bar_q, ph_q, broken);
    ph_q ^= 1;
    wait_phase(bar_do, ph_do, broken);
    ph_do ^= 1;
    wait_phase(bar_img, ph_img, broken);
    ph_img ^= 1;
    if (L < kChunk) {
      // the first chunk processed is the only partial one: rows past the
      // sequence end hold the next sequence's tokens (or zero fill)
      const int nz = kChunk - L;
      for (int idx = tid; idx < 6 * nz * 8; idx += kBwdScanThreads) {
        const int ch = idx & 7, r = L + (idx >> 3) % nz, which = (idx >> 3) / nz;  // 0..5
        const uint32_t base = (which >> 1) == 0 ? SM::kQ : ((which >> 1) == 1 ? (cb ? SM::kK1 : SM::kK0) : SM::kDO);
        *reinterpret_cast<uint4 *>(smem + base + (which & 1) * 8192 + r * 128 + ch * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA a: Zr = dS K^T ----
    if (tid == 0) {
      const uint64_t dk = umma_desc_sw128(kbuf, 16, 1024);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t boff = (ks >> 2) * 8192 + (ks & 3) * 32;
        umma_bf16_ts(tmem + SM::kColA, tmem + SM::kColSb + 8 * ks, umma_desc_advance(dk, boff), id_a,
                     ks > 0);
      }
      umma_commit(bar_mma);
    }
    // Q' = scale e^{G_t} Q, in place, while MMA a runs (1024 chunks of 8)
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = tid + kBwdScanThreads * m;
      const int t = (idx >> 3) & 63;
      uint4 *pq = reinterpret_cast<uint4 *>(smem + SM::kQ + (idx >> 9) * 8192 + t * 128 + (idx & 7) * 16);
      float f[8];
      unpack8(*pq, f);
      const float sc = scale * EG[t];
      *pq = make_uint4(pack_bf16x2(sc * f[0], sc * f[1]), pack_bf16x2(sc * f[2], sc * f[3]),
                       pack_bf16x2(sc * f[4], sc * f[5]), pack_bf16x2(sc * f[6], sc * f[7]));
    }
    wait_phase(bar_mma, ph_mma, broken);
    ph_mma ^= 1;
    tc_fence_after();

    // ---- Z / scale -> K-major tile (tokens 32 hc .. 32 hc + 31 of row vrow) ----
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int tb = 32 * hc + 16 * p;
      float z[16];
      tmem_ld16(tlane + SM::kColA + tb, z);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) z[j] *= ED[tb + j] * inv_scale;
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pk[j] = pack_bf16x2(z[2 * j], z[2 * j + 1]);
      tmem_st8(tlane + SM::kColZX + 32 * hc + 8 * p, pk);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA b: dX / scale = dO^T (P Ainv) + (Z / scale) Ainv ----
    if (tid == 0) {
      const uint64_t dmn = umma_desc_sw128(s_base, 8192, 1024);  // MN-major, 8 KB between blocks
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + SM::kColB, umma_desc_advance(dmn, SM::kDO + ks * 2048),
                  umma_desc_advance(dmn, SM::kImg + ks * 2048), id_b1, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16_ts(tmem + SM::kColB, tmem + SM::kColZX + 32 * (ks >> 1) + 8 * (ks & 1),
                     umma_desc_advance(dmn, SM::kImg + 8192 + ks * 2048), id_b2, 1);
      umma_commit(bar_mma);
    }
    wait_phase(bar_mma, ph_mma, broken);
    ph_mma ^= 1;
    tc_fence_after();
    if (tid == 0 && c > 0) issue_img(c - 1);  // the image is consumed

    // ---- dX: dv = beta dX (fp32), dX as the chunk kernel's token image,
    // and -beta e^G dX -> K-major tile ----
    uint8_t *dximg = dx_ws + (gc * kHV + hv) * kTokImgBytes;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int tb = 32 * hc + 16 * p;
      float x[16];
      tmem_ld16(tlane + SM::kColB + tb, x);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = tb + j;
        const float dx = t < L ? scale * x[j] : 0.f;
        put_tok_img(dximg, t, vrow, dx);
        if (t < L) dv[((t0 + t) * kHV + hv) * kD + vrow] = BT[t] * dx;
        x[j] = -BT[t] * EG[t] * dx;
      }
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pk[j] = pack_bf16x2(x[2 * j], x[2 * j + 1]);
      tmem_st8(tlane + SM::kColZX + 32 * hc + 8 * p, pk);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA c: dS' = dO^T Q' - (beta e^G dX) K ----
    if (tid == 0) {
      const uint64_t dmn = umma_desc_sw128(s_base, 8192, 1024);
      const uint64_t dkm = umma_desc_sw128(kbuf, 8192, 1024);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + SM::kColA, umma_desc_advance(dmn, SM::kDO + ks * 2048),
                  umma_desc_advance(dmn, SM::kQ + ks * 2048), id_c1, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16_ts(tmem + SM::kColA, tmem + SM::kColZX + 32 * (ks >> 1) + 8 * (ks & 1),
                     umma_desc_advance(dkm, ks * 2048), id_c2, 1);
      umma_commit(bar_mma);
    }
    wait_phase(bar_mma, ph_mma, broken);
    ph_mma ^= 1;
    tc_fence_after();
    if (tid == 0) {  // Q, dO and this K buffer are consumed
      if (c > 0) {
        issue_tile2(&tmap_q, s_base + SM::kQ, hqk * kD, c - 1, bar_q);
        issue_tile2(&tmap_do, s_base + SM::kDO, hv * kD, c - 1, bar_do);
      }
      if (c > 1) issue_tile2(&tmap_k, kbuf, hqk * kD, c - 2, bar_k0 + 8 * cb);
    }

    // ---- dS <- e^{G_C} dS + dS' ; bf16(dS) -> TMEM ----
    {
      const float egc = EGC[0];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        float d[32];
        tmem_ld32(tlane + SM::kColA + 64 * hc + 32 * p, d);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) ds[32 * p + j] = egc * ds[32 * p + j] + d[j];
      }
      put_sb();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (d_state != nullptr) {
    float *dst = d_state + static_cast<int64_t>(n) * kHV * kD * kD + hv_off + srow;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<float4 *>(dst + 4 * i) =
          make_float4(ds[4 * i], ds[4 * i + 1], ds[4 * i + 2], ds[4 * i + 3]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, SM::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// chunk-parallel gradients (tcgen05)
// ---------------------------------------------------------------------------
// Persistent clusters of two CTAs (256 threads and the whole TMEM each, one
// CTA per SM): a cluster takes the (chunk, q/k head) pairs in turn, its rank
// r the v-head 2 hqk + r, and each CTA fetches the next pair's operands into
// its buffers as they retire.  Per (chunk, v-head), eight MMAs on bf16
// operands, fp32 accumulators in TMEM:
//   (a) [Q;K] K^T      -> QK (lanes 0-63), KK (lanes 64-127)      M=128 N=64 K=128
//   (b) [dO;dX] [delta;V]^T -> dO.delta (lanes 0-63), dX.delta and dX.v
//                          (lanes 64-127; the diagonal of dX.v is dX_t.v_t)  N=128
//   (c) S_0^T dO^T = (dO S_0)^T        lanes k, columns t         M=128 N=64 K=128
//   (d) S_0^T dX^T = (dX S_0)^T
//   (e) dS_C^T delta^T = (delta dS_C)^T
//   (f) K^T Mq^T = (Mq K)^T                                       K=64
//   (g)+(h) Q^T Mq + K^T Msym = (Mq^T Q + Msym K)^T
// S_0, dS_C ([v][k] in memory) and the Q and K tiles ([t][k]) enter (c)-(h)
// as MN-major A operands (k contiguous), so nothing is transposed by hand.
// Every input arrives by TMA (Q, K, dO, V tiles) or bulk copy (the S_0,
// dS_C, delta and dX images the recompute and the reverse scan wrote): the
// images and the dO / V tiles as soon as batch 2 is done with the previous
// pair's, the Q / K tiles once batch 3 and the dot products are, dS_C once the
// dq / dk exchange that borrows its buffer is consumed.
// Mq and Msym come from (a) and (b) by element-wise work on the CUDA cores
// between the two MMA batches.
constexpr int kBwdTcThreads = 256;  // warps w and w + 4 share TMEM lanes 32 (w & 3) ..
// The thread that issues the copies and the MMAs: lane 0 of warp 4, whose
// share of the Mq pass (rows 0..31, columns 32..63) is structurally zero.
constexpr int kBwdTcIssuer = 128;

struct BwdTcSmem {
  static constexpr int kQK = 0;        // [Q;K]: 2 d-blocks x (64 Q rows | 64 K rows) x 128 B (TMA)
  static constexpr int kOX = 32768;    // [dO;dX]: 2 v-blocks x (64 dO rows (TMA) | 64 dX rows) x 128 B
  static constexpr int kDV = 65536;    // [delta;V]: 2 v-blocks x (64 delta rows | 64 V rows (TMA)) x 128 B
  static constexpr int kS0 = 98304;    // S_0 as MN-major A: 2 k-blocks x 128 v rows x 128 B
  static constexpr int kDS = 131072;   // dS_C, same layout
  static constexpr int kMQ = 163840;   // Mq bf16 [64 t][64 j], 128-byte rows
  static constexpr int kMS = 172032;   // Msym bf16 [64][64]
  static constexpr int kMA = 180224;   // Ma fp32 [64][65] (transpose staging)
  static constexpr int kVec = kMA + 64 * 65 * 4;     // per-token vectors: 16 x 64 fp32
  static constexpr int kRed = kVec + 16 * 64 * 4;    // partials [4 lane quadrants][5][64] fp32
  static constexpr int kRow = kRed + 4 * 5 * 64 * 4;  // row-sum halves [2][3][64] fp32
  // 8 mbarriers: qk, rest, m1, m2, m3, xfree, xfull, ds
  static constexpr int kBar = kRow + 2 * 3 * 64 * 4;
  static constexpr int kTmem = kBar + 64;
  static constexpr int kBroken = kBar + 68;
  static constexpr int kScal = kBar + 96;            // 16 fp32 scalars
  static constexpr int kBytes = kScal + 64 + 1024;   // + base alignment slack
};
static_assert(BwdTcSmem::kMA + 64 * 65 * 4 <= BwdTcSmem::kVec, "layout");
static_assert(BwdTcSmem::kBytes <= 227 * 1024, "shared memory");
// TMEM columns
constexpr uint32_t kTcA = 0, kTcB = 64, kTcP1 = 192, kTcP2 = 256, kTcP3 = 320, kTcF = 384,
                   kTcGH = 448, kTcCols = 512;
// per-token vector slots and partial-sum families
enum BwdVec : int {
  kVG = 0, kVEG, kVBT, kVED, kVRowWq, kVRowWa, kVDbA, kVDXv, kVZeta, kVDG, kVDB, kVEGL
};
enum BwdRed : int { kRedRho = 0, kRedXi, kRedZeta, kRedColWq, kRedColWa };

// Sum over the warp's 32 lanes of v[lane]: a transposing butterfly (31
// shuffles for 32 sums, instead of 32 x 5).  v is clobbered.
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

__device__ __forceinline__ uint4 pack8(const float4 a, const float4 b) {
  return make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                    pack_bf16x2(b.z, b.w));
}

// element (row, col) of a bf16 tile with 128-byte rows and 128-byte swizzle
__device__ __forceinline__ float tile_at(const uint8_t *tile, int row, int col) {
  return bf16_to_f32(*reinterpret_cast<const uint16_t *>(
      tile + row * 128 + ((((col >> 3) ^ row) & 7) << 4) + (col & 7) * 2));
}

__global__ void __launch_bounds__(kBwdTcThreads, 1)
gdn_prefill_bwd_chunk_kernel(const __grid_constant__ CUtensorMap tmap_q,
                             const __grid_constant__ CUtensorMap tmap_k,
                             const __grid_constant__ CUtensorMap tmap_do,
                             const __grid_constant__ CUtensorMap tmap_v,
                             const float *__restrict__ A_log,
                             const uint16_t *__restrict__ a, const float *__restrict__ dt_bias,
                             const int64_t *__restrict__ cu, const int *__restrict__ meta,
                             const int4 *__restrict__ chunk_tab, const float *__restrict__ gcum_ws,
                             const float *__restrict__ beta_ws,
                             const uint8_t *__restrict__ states_ws,
                             const uint8_t *__restrict__ dsc_ws,
                             const uint8_t *__restrict__ delta_ws,
                             const uint8_t *__restrict__ dx_ws, float scale, int npairs,
                             float *__restrict__ dq, float *__restrict__ dk,
                             float *__restrict__ da, float *__restrict__ db,
                             float *__restrict__ dgg_ws) {
  using SM = BwdTcSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Persistent: a cluster of two CTAs walks the pairs p = (chunk p / 4, q/k
  // head p % 4), p = cluster, cluster + clusters, ...; rank r of the cluster
  // takes v-head 2 hqk + r.  Both ranks walk the same pairs, so every cluster
  // barrier below is reached by both or by neither.
  const int crank = static_cast<int>(cluster_ctarank());
  const int ncl = static_cast<int>(gridDim.x >> 1);
  const int nchunks = meta[kMetaChunks];
  const bool meta_ok = meta[kMetaError] == 0;
  auto live = [&](int p) { return meta_ok && p < npairs && p / kHQK < nchunks; };

  float *VEC = reinterpret_cast<float *>(smem + SM::kVec);
  float *RED = reinterpret_cast<float *>(smem + SM::kRed);
  float *SC = reinterpret_cast<float *>(smem + SM::kScal);
  float *MA = reinterpret_cast<float *>(smem + SM::kMA);
  float *ROW = reinterpret_cast<float *>(smem + SM::kRow);  // [hh][Wq | Wa | dbA][i]
  volatile int *broken = reinterpret_cast<volatile int *>(smem + SM::kBroken);
  auto vec = [&](int slot) { return VEC + slot * 64; };
  auto red = [&](int w, int f) { return RED + (w * 5 + f) * 64; };
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_qk = s_base + SM::kBar, bar_rest = bar_qk + 8, bar_m1 = bar_qk + 16,
                 bar_m2 = bar_qk + 24, bar_m3 = bar_qk + 32;
  // the dq / dk exchange: the partner arrives on xfree when its exchange area
  // may be written; its stores into this CTA's area complete on xfull.  The
  // area is the dS_C image, whose copy for the next pair (bar_ds) is issued
  // once the exchange is consumed.
  const uint32_t bar_xfree = bar_qk + 40, bar_xfull = bar_qk + 48, bar_ds = bar_qk + 56;
  const uint32_t peer = static_cast<uint32_t>(crank ^ 1);

  // the copies of one pair's operands: the Q and K tiles (bar_qk); the dO and
  // V tiles and the S_0, delta and dX images (bar_rest); the dS_C image (bar_ds)
  auto issue_qk = [&](int hqk, int64_t t0) {
    mbar_arrive_expect_tx(bar_qk, 32768);
    for (int blk = 0; blk < 2; ++blk) {
      const int y = static_cast<int>(t0);
      tma_load_2d(s_base + SM::kQK + blk * 16384, &tmap_q, hqk * kD + 64 * blk, y, bar_qk);
      tma_load_2d(s_base + SM::kQK + blk * 16384 + 8192, &tmap_k, hqk * kD + 64 * blk, y, bar_qk);
    }
  };
  // (bar_rest's copies in two halves, which two threads may issue: the barrier
  // cannot complete before the first half's expect_tx arrival, whichever half's
  // bytes land first)
  auto issue_rest_a = [&](int g, int hv, int64_t t0) {  // expect_tx, S_0, dO and V tiles
    const int64_t soff = (static_cast<int64_t>(g) * kHV + hv) * kStateImgBytes;
    mbar_arrive_expect_tx(bar_rest, 32768 + static_cast<uint32_t>(kStateImgBytes) +
                                        2 * static_cast<uint32_t>(kTokImgBytes));
    bulk_load(s_base + SM::kS0, states_ws + soff, static_cast<uint32_t>(kStateImgBytes), bar_rest);
    for (int blk = 0; blk < 2; ++blk) {
      const int y = static_cast<int>(t0);
      tma_load_2d(s_base + SM::kOX + blk * 16384, &tmap_do, hv * kD + 64 * blk, y, bar_rest);
      tma_load_2d(s_base + SM::kDV + blk * 16384 + 8192, &tmap_v, hv * kD + 64 * blk, y, bar_rest);
    }
  };
  auto issue_rest_b = [&](int g, int hv) {  // the dX and delta images
    const int64_t toff = (static_cast<int64_t>(g) * kHV + hv) * kTokImgBytes;
    for (int blk = 0; blk < 2; ++blk) {
      bulk_load(s_base + SM::kOX + blk * 16384 + 8192, dx_ws + toff + blk * 8192, 8192, bar_rest);
      bulk_load(s_base + SM::kDV + blk * 16384, delta_ws + toff + blk * 8192, 8192, bar_rest);
    }
  };
  auto issue_ds = [&](int g, int hv) {
    const int64_t soff = (static_cast<int64_t>(g) * kHV + hv) * kStateImgBytes;
    mbar_arrive_expect_tx(bar_ds, static_cast<uint32_t>(kStateImgBytes));
    bulk_load(s_base + SM::kDS, dsc_ws + soff, static_cast<uint32_t>(kStateImgBytes), bar_ds);
  };
  // gate inputs of the next pair, loaded a pair ahead into registers (token
  // tid < 64; zero past the chunk's end): G, beta, G_C, a (raw bf16), dt_bias,
  // A_log -- only loaded here, used at the next pair's start, so that no
  // arithmetic waits on the loads now
  float nx_g = 0.f, nx_b = 0.f, nx_gc = 0.f, nx_dtb = 0.f, nx_alog = 0.f;
  uint16_t nx_a = 0;
  auto fetch_gates = [&](const int4 &en, int hvn) {
    if (tid < 64) {
      nx_gc = gcum_ws[(en.z + en.w - 1) * kHV + hvn];
      nx_alog = A_log[hvn];
      nx_g = 0.f;
      nx_b = 0.f;
      nx_a = 0;
      nx_dtb = 0.f;
      if (tid < en.w) {
        const int64_t idx = (en.z + tid) * kHV + hvn;
        nx_g = gcum_ws[idx];
        nx_b = beta_ws[idx];
        nx_a = a[idx];
        nx_dtb = dt_bias[hvn];
      }
    }
  };

  // ---- TMEM, barriers and the first pair's copies ----
  int p = static_cast<int>(blockIdx.x >> 1);
  bool have = live(p);
  int4 e = have ? chunk_tab[p / kHQK] : make_int4(0, 0, 0, 0);
  if (warp == 0) tmem_alloc(s_base + SM::kTmem, kTcCols);
  if (tid == kBwdTcIssuer) {
    *broken = 0;
    for (int i = 0; i < 8; ++i) mbar_init(bar_qk + 8 * i, 1);
    mbar_init_fence();
    if (have) {
      issue_qk(p % kHQK, e.z);
      issue_rest_a(p / kHQK, 2 * (p % kHQK) + crank, e.z);
      issue_rest_b(p / kHQK, 2 * (p % kHQK) + crank);
      issue_ds(p / kHQK, 2 * (p % kHQK) + crank);
    }
  }
  if (have) fetch_gates(e, 2 * (p % kHQK) + crank);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // both CTAs' barriers are initialised before either signals the other
  cluster_arrive();
  cluster_wait();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + SM::kTmem);
  const int quad = warp & 3, hh = warp >> 2;
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quad) << 16);
  const int kk = 32 * quad + lane;  // k index of this thread's TMEM lane (dots, dq, dk)

  uint32_t par = 0;  // each of the eight barriers completes once per pair
  while (have) {
    const int hqk = p % kHQK, hv = 2 * hqk + crank;
    const int64_t t0 = e.z;
    const int L = e.w;
    GDN_DCHECK(e.x >= 0 && e.x < meta[kMetaN] && L > 0 && t0 + L <= meta[kMetaT]);
    const int pn = p + ncl;
    const bool have_n = live(pn);
    const int4 en = have_n ? chunk_tab[pn / kHQK] : make_int4(0, 0, 0, 0);
    const int hv_n = 2 * (pn % kHQK) + crank;

    // the partner's 32 KB of dq / dk values for this pair land on xfull
    if (tid == kBwdTcIssuer) mbar_arrive_expect_tx(bar_xfull, 32768);
    // ---- gates (inputs fetched a pair ahead) ----
    // token tid's gate terms, kept for the gate gradients at the end: e^{A_log},
    // d softplus / dx at x = a + dt_bias, and gl = -e^{A_log} softplus(x)
    float g_ea = 0.f, g_sig = 0.f, g_gl = 0.f;
    if (tid < 64) {
      const float gg = nx_g, bt = nx_b;
      const float x = bf16_to_f32(nx_a) + nx_dtb;  // a + dt_bias (0 past the end)
      g_ea = expf(nx_alog);
      g_sig = 1.0f / (1.0f + expf(-x));
      g_gl = -g_ea * softplus_stable(x);
      vec(kVG)[tid] = gg;
      vec(kVEG)[tid] = tid < L ? expf(gg) : 0.f;
      vec(kVBT)[tid] = bt;
      vec(kVED)[tid] = tid < L ? expf(nx_gc - gg) : 0.f;
      vec(kVEGL)[tid] = tid < L ? expf(g_gl) : 1.f;
      if (tid == 0) SC[0] = expf(nx_gc);
    }
    __syncthreads();

    // ---- operands written by the threads (bf16, 128-byte swizzle) ----
    // tiles and images landed; rows past the sequence end of the TMA tiles
    // hold the next sequence's tokens: zero them (the images are zero there)
    wait_phase(bar_qk, par, broken);
    wait_phase(bar_rest, par, broken);
    if (L < kChunk) {
      const int nz = kChunk - L;
      for (int idx = tid; idx < 8 * nz * 8; idx += kBwdTcThreads) {
        const int ch = idx & 7, r = L + (idx >> 3) % nz, which = (idx >> 3) / nz;  // 0..7
        const int base = which < 4   ? SM::kQK + (which >> 1) * 16384 + (which & 1) * 8192
                         : which < 6 ? SM::kOX + (which - 4) * 16384
                                     : SM::kDV + (which - 6) * 16384 + 8192;
        *reinterpret_cast<uint4 *>(smem + base + r * 128 + ch * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA batch 1: (a), (b); batch 2: (c), (d), (e) ----
    if (tid == kBwdTcIssuer) {
      const uint32_t id_kk = umma_idesc_bf16(128, 64, false, false);
      const uint32_t id_kk2 = umma_idesc_bf16(128, 128, false, false);
      const uint32_t id_mn = umma_idesc_bf16(128, 64, true, false);
      // one descriptor per layout, advanced by each operand's byte offset
      const uint64_t dk16 = umma_desc_sw128(s_base, 16, 1024);      // K-major
      const uint64_t dmn16k = umma_desc_sw128(s_base, 16384, 1024);  // MN-major, 16 KB between blocks
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        umma_bf16(tmem + kTcA, umma_desc_advance(dk16, SM::kQK + off),
                  umma_desc_advance(dk16, SM::kQK + 8192 + off), id_kk, ks > 0);
        umma_bf16(tmem + kTcB, umma_desc_advance(dk16, SM::kOX + off),
                  umma_desc_advance(dk16, SM::kDV + off), id_kk2, ks > 0);
      }
      umma_commit(bar_m1);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {  // K = v, 16 rows of the MN-major tiles per step
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        const uint64_t s0 = umma_desc_advance(dmn16k, SM::kS0 + ks * 2048);
        umma_bf16(tmem + kTcP1, s0, umma_desc_advance(dk16, SM::kOX + off), id_mn, ks > 0);
        umma_bf16(tmem + kTcP2, s0, umma_desc_advance(dk16, SM::kOX + 8192 + off), id_mn, ks > 0);
      }
      wait_phase(bar_ds, par, broken);  // dS_C (issued after the previous pair's exchange)
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        umma_bf16(tmem + kTcP3, umma_desc_advance(dmn16k, SM::kDS + ks * 2048),
                  umma_desc_advance(dk16, SM::kDV + off), id_mn, ks > 0);
      }
      // S_0^T dS_C into the F / GH columns (free until batch 3): its trace is
      // <dS_C, S_0>
      const uint32_t id_tr = umma_idesc_bf16(128, 128, true, true);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + kTcF, umma_desc_advance(dmn16k, SM::kS0 + ks * 2048),
                  umma_desc_advance(dmn16k, SM::kDS + ks * 2048), id_tr, ks > 0);
      umma_commit(bar_m2);
    }

    // ---- Mq, Ma and their gate terms: row i = TMEM lane, columns 32 hh.. ----
    wait_phase(bar_m1, par, broken);
    tc_fence_after();
    if ((warp & 5) == 4) {
      // warps 4 and 6: rows 0..31, columns 32..63 -- every j > i, so Mq, Ma,
      // their row and column sums and dbA are zero there
      const int i = lane;
      if (warp == 4) {
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4 *>(smem + SM::kMQ + i * 128 + (((4 + cc) ^ i) & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        ROW[(3 + 0) * 64 + i] = 0.f;
        red(0, kRedColWq)[32 + lane] = 0.f;
      } else {
#pragma unroll
        for (int u = 0; u < 32; ++u) MA[i * 65 + 32 + u] = 0.f;
        ROW[(3 + 1) * 64 + i] = 0.f;
        ROW[(3 + 2) * 64 + i] = 0.f;
        red(2, kRedColWa)[32 + lane] = 0.f;
      }
    } else {
      const bool qside = quad < 2;  // lanes 0-63: QK, dO.delta; lanes 64-127: KK, dX.delta
      const int i = 32 * (quad & 1) + lane;
      const float bi = vec(kVBT)[i];
      float rsum = 0.f, dba = 0.f;
      float m[32], w[32];
      __syncwarp();
      tmem_ld32(tl + kTcA + 32 * hh, m);  // QK or KK
      tmem_ld32(tl + kTcB + 32 * hh, w);  // dO.delta or dX.delta
      tmem_wait_ld();
      // e^{G_i - G_j} for the columns j <= i, right to left as a running
      // product of the per-token decays e^{gl_j} (one exponential per row)
      const int jt = 32 * hh + 31;
      float dec = i > jt ? expf(vec(kVG)[i] - vec(kVG)[jt]) : 1.f;
      const float4 *egl4 = reinterpret_cast<const float4 *>(vec(kVEGL) + 32 * hh);
#pragma unroll
      for (int q = 7; q >= 0; --q) {
        const float4 e4 = egl4[q];
        const float egl[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int r = 3; r >= 0; --r) {
          const int u = 4 * q + r, j = 32 * hh + u;
          float x;
          if (qside) {
            x = (i < L && j <= i) ? scale * dec * w[u] : 0.f;  // Mq
          } else {
            const float dA = -w[u];
            x = (i < L && j < i) ? dA * bi * dec : 0.f;  // Ma
            if (i < L && j < i) dba += dA * dec * m[u];
            MA[i * 65 + j] = x;
          }
          w[u] = x;
          m[u] *= x;  // W = M o (QK or KK)
          rsum += m[u];
          if (j <= i) dec *= egl[r];  // column j - 1 next
        }
      }
      if (qside) {  // row i of Mq, columns 32 hh .. 32 hh + 31, as bf16
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4 *>(smem + SM::kMQ + i * 128 + (((4 * hh + cc) ^ i) & 7) * 16) =
              make_uint4(pack_bf16x2(w[8 * cc], w[8 * cc + 1]), pack_bf16x2(w[8 * cc + 2], w[8 * cc + 3]),
                         pack_bf16x2(w[8 * cc + 4], w[8 * cc + 5]),
                         pack_bf16x2(w[8 * cc + 6], w[8 * cc + 7]));
        ROW[(hh * 3 + 0) * 64 + i] = rsum;
      } else {
        ROW[(hh * 3 + 1) * 64 + i] = rsum;
        ROW[(hh * 3 + 2) * 64 + i] = dba;
        if (hh == (quad & 1)) {  // dX_i . v_i sits in this column half
          float x[32];
          tmem_ld32(tl + kTcB + 64 + 32 * hh, x);
          tmem_wait_ld();
          float d = 0.f;
#pragma unroll
          for (int u = 0; u < 32; ++u) d = u == lane ? x[u] : d;
          vec(kVDXv)[i] = i < L ? d : 0.f;
        }
      }
      const float cs = warp_transpose_sum32(m, lane);  // column 32 hh + lane over these 32 rows
      red(quad, qside ? kRedColWq : kRedColWa)[32 * hh + lane] = cs;
    }
    // <dS_C, S_0>: the diagonal of S_0^T dS_C, lanes 32 quad .. of warp 4 + quad
    // (batch 3 overwrites these columns after the next barrier)
    if (hh == 1) {
      wait_phase(bar_m2, par, broken);
      tc_fence_after();
      // batch 2 is done with dS_C: this CTA's exchange area is free
      if (tid == kBwdTcIssuer) mbar_arrive_cluster(dsmem_map(bar_xfree, peer));
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the one-lane branches
      float x[32];
      tmem_ld32(tl + kTcF + 32 * quad, x);
      tmem_wait_ld();
      float d = 0.f;
#pragma unroll
      for (int u = 0; u < 32; ++u) d = u == lane ? x[u] : d;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (lane == 0) SC[4 + quad] = d;  // SC[4..7]
    }
    tc_fence_before();
    __syncthreads();
    {  // Msym = Ma + Ma^T: row i = tid & 63, 16 columns per thread
      const int i = tid & 63, q4 = tid >> 6;
#pragma unroll
      for (int cc = 2 * q4; cc < 2 * q4 + 2; ++cc) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = 8 * cc + u;
          x[u] = MA[i * 65 + j] + MA[j * 65 + i];
        }
        *reinterpret_cast<uint4 *>(smem + SM::kMS + i * 128 + ((cc ^ i) & 7) * 16) =
            make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                       pack_bf16x2(x[6], x[7]));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA batch 3: (f) K^T Mq^T; (g) Q^T Mq, (h) + K^T Msym ----
    if (tid == kBwdTcIssuer) {
      const uint32_t id_f = umma_idesc_bf16(128, 64, true, false);
      const uint32_t id_g = umma_idesc_bf16(128, 64, true, true);
      const uint64_t dk16 = umma_desc_sw128(s_base, 16, 1024);
      const uint64_t dmn16k = umma_desc_sw128(s_base, 16384, 1024);
      const uint64_t dmn8k = umma_desc_sw128(s_base, 8192, 1024);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // K = 64 tokens
        const uint64_t kt = umma_desc_advance(dmn16k, SM::kQK + 8192 + ks * 2048);
        const uint64_t qt = umma_desc_advance(dmn16k, SM::kQK + ks * 2048);
        umma_bf16(tmem + kTcF, kt, umma_desc_advance(dk16, SM::kMQ + ks * 32), id_f, ks > 0);
        umma_bf16(tmem + kTcGH, qt, umma_desc_advance(dmn8k, SM::kMQ + ks * 2048), id_g, ks > 0);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + kTcGH, umma_desc_advance(dmn16k, SM::kQK + 8192 + ks * 2048),
                  umma_desc_advance(dk16, SM::kMS + ks * 32), id_f, 1);
      umma_commit(bar_m3);
    }

    // ---- per-token dot products with q and k: thread = k (TMEM lane), tokens 32 hh.. ----
    wait_phase(bar_m2, par, broken);
    tc_fence_after();
    // batch 2 is done: S_0, [dO;dX] and [delta;V] are no longer read, so the
    // next pair's copies go there now and land while this pair runs (issued
    // by lane 0 of warps 6 and 7, not by the MMA issuer's warp, which has the
    // batch 3 MMAs to issue)
    if (have_n) {
      if (tid == 192) issue_rest_a(pn / kHQK, hv_n, en.z);
      if (tid == 224) issue_rest_b(pn / kHQK, hv_n);
      fetch_gates(en, hv_n);
    }
    __syncwarp();
    {
      const uint8_t *qtile = smem + SM::kQK + (kk >> 6) * 16384;
      const uint8_t *ktile = qtile + 8192;
#pragma unroll 1
      for (int f = 0; f < 3; ++f) {
        const uint32_t col = f == 0 ? kTcP1 : (f == 1 ? kTcP2 : kTcP3);
        const uint8_t *tile = f == 0 ? qtile : ktile;
        float x[32];
        tmem_ld32(tl + col + 32 * hh, x);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) x[u] *= tile_at(tile, 32 * hh + u, kk & 63);
        red(quad, f)[32 * hh + lane] = warp_transpose_sum32(x, lane);
      }
    }

    // ---- dq, dk ----
    // The two v-heads of q/k head hqk (this cluster's two CTAs) both add to
    // its dq and dk rows: rank 0 writes the dq rows and rank 1 the dk rows,
    // each adding the partner's contribution, which arrives by asynchronous
    // stores into the retired dS_C image as [128 k][64 t] fp32 (the
    // 16-byte chunk t / 4 of row k at chunk (t / 4) ^ (k & 7): conflict-free
    // for the 16-byte accesses of consecutive k).  One fp32 sum of two terms
    // per element: the result does not depend on which CTA got there first,
    // and no zeroing pass or read-modify-write of dq / dk in DRAM is needed.
    wait_phase(bar_m3, par, broken);
    tc_fence_after();
    __syncwarp();
    float vq[32], vk[32];
    {
      const float *EG = vec(kVEG), *BT = vec(kVBT), *ED = vec(kVED);
      {
        float pp[32], f[32];
        tmem_ld32(tl + kTcP1 + 32 * hh, pp);
        tmem_ld32(tl + kTcF + 32 * hh, f);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) vq[u] = scale * EG[32 * hh + u] * pp[u] + f[u];
      }
      {
        float pp[32], f[32], p3[32];
        tmem_ld32(tl + kTcP2 + 32 * hh, pp);
        tmem_ld32(tl + kTcGH + 32 * hh, f);
        tmem_ld32(tl + kTcP3 + 32 * hh, p3);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int t = 32 * hh + u;
          vk[u] = f[u] - BT[t] * EG[t] * pp[u] + ED[t] * p3[u];
        }
      }
    }
    // the partner's area is free: send it the half it writes
    wait_phase_cluster(bar_xfree, par, broken);
    {
      const uint32_t rx = dsmem_map(s_base + SM::kDS, peer) + static_cast<uint32_t>(kk) * 256;
      const uint32_t rbar = dsmem_map(bar_xfull, peer);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t chunk = static_cast<uint32_t>(8 * hh + (q ^ (kk & 7)));
        const float4 v = crank ? make_float4(vq[4 * q], vq[4 * q + 1], vq[4 * q + 2], vq[4 * q + 3])
                               : make_float4(vk[4 * q], vk[4 * q + 1], vk[4 * q + 2], vk[4 * q + 3]);
        dsmem_st_async_v4(rx + chunk * 16, v, rbar);
      }
    }

    // ---- gate gradients (tokens t = tid < 64, two warps) ----
    // every warp's dot-product partials (red) are written, and every thread is
    // past the dot products: the Q / K tiles are retired
    __syncthreads();
    if (have_n && tid == kBwdTcIssuer) issue_qk(pn % kHQK, en.z);
    // warps 0 and 1 only, synchronised by a named barrier of their 64 threads,
    // while the other warps go on to their dq / dk rows
    if (warp < 2) {
      const int t = tid;
      float dG = 0.f, dB = 0.f, ez = 0.f;
      float rho = 0.f, xi = 0.f, zeta = 0.f;
      for (int q = 0; q < 4; ++q) {
        rho += red(q, kRedRho)[t];
        xi += red(q, kRedXi)[t];
        zeta += red(q, kRedZeta)[t];
      }
      const float colwq = red(0, kRedColWq)[t] + red(1, kRedColWq)[t];
      const float colwa = red(2, kRedColWa)[t] + red(3, kRedColWa)[t];
      const float rowwq = ROW[0 * 64 + t] + ROW[3 * 64 + t];
      const float rowwa = ROW[1 * 64 + t] + ROW[4 * 64 + t];
      const float dba = ROW[2 * 64 + t] + ROW[5 * 64 + t];
      const float eg = vec(kVEG)[t], bt = vec(kVBT)[t], ed = vec(kVED)[t];
      if (t < L) {
        dB = vec(kVDXv)[t] - eg * xi + dba;
        dG = scale * eg * rho + rowwq - colwq + rowwa - colwa - bt * eg * xi - ed * zeta;
        ez = ed * zeta;  // the chunk-end state depends on G_C through every token
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ez += __shfl_xor_sync(0xffffffffu, ez, o);
      if (lane == 0) SC[12 + warp] = ez;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (t == L - 1) {
        float sds = 0.f;  // <dS_C, S_0>, four warp partials in a fixed order
        for (int w4 = 0; w4 < 4; ++w4) sds += SC[4 + w4];
        dG += SC[0] * sds + SC[12] + SC[13];
      }
      // dg_t = sum_{s >= t} dG_s: suffix scan within each warp, then warp 1's total into warp 0
      float x = dG;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, x, o);
        if (lane + o < 32) x += y;
      }
      if (t == 32) SC[14] = x;  // total of tokens 32..63
      vec(kVDG)[t] = x;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (t < L) {
        const float dg = vec(kVDG)[t] + (t < 32 ? SC[14] : 0.f);
        const int64_t idx = (t0 + t) * kHV + hv;
        da[idx] = -dg * g_ea * g_sig;
        db[idx] = dB * bt * (1.0f - bt);
        dgg_ws[idx] = dg * g_gl;
      }
    }
    // the partner's half has landed: add it to this CTA's own and write the rows
    wait_phase_cluster(bar_xfull, par, broken);
    {
      const float *X = reinterpret_cast<const float *>(smem + SM::kDS) + kk * 64;
      float *dst = crank ? dk : dq;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 x = *reinterpret_cast<const float4 *>(X + 4 * (8 * hh + (q ^ (kk & 7))));
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int u = 4 * q + r, t = 32 * hh + u;
          if (t < L) dst[((t0 + t) * kHQK + hqk) * kD + kk] = (crank ? vk[u] : vq[u]) + xs[r];
        }
      }
    }
    // the next pair overwrites the gate vectors, the partial sums and TMEM
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the exchange is consumed: the next pair's dS_C
    if (have_n && tid == kBwdTcIssuer) issue_ds(pn / kHQK, hv_n);
    p = pn;
    e = en;
    have = have_n;
    par ^= 1u;
  }
  // neither CTA leaves while the other may still signal or store into it
  cluster_arrive();
  cluster_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcCols);
  }
}

// ---------------------------------------------------------------------------
// dA_log and ddt_bias: fixed-order sums over the tokens
// ---------------------------------------------------------------------------
constexpr int kBwdReduceThreads = 256;

// dA_log = sum_t dg_t g_t and ddt_bias = sum_t da_t per v-head, in two fixed-
// order stages (deterministic).  Stage 1: block b sums its contiguous token
// range, thread (token slot ts, head h) reading the [T][8] arrays coalesced;
// the four lanes of a warp that share h are combined by shuffles, the eight
// warps in order.
__global__ void __launch_bounds__(kBwdReduceThreads)
gdn_prefill_bwd_reduce_partial_kernel(const int *__restrict__ meta,
                                      const float *__restrict__ dgg_ws,
                                      const float *__restrict__ da, int64_t T,
                                      float *__restrict__ red) {
  __shared__ float s1[kBwdReduceThreads / 32][kHV], s2[kBwdReduceThreads / 32][kHV];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hv = tid & (kHV - 1), ts = tid / kHV;  // 32 tokens x 8 heads per pass
  const int64_t per = (T + kBwdRedBlocks - 1) / kBwdRedBlocks;
  const int64_t t_begin = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t t_end = t_begin + per < T ? t_begin + per : T;
  float x = 0.f, y = 0.f;
  if (meta[kMetaError] == 0)
    for (int64_t t = t_begin + ts; t < t_end; t += kBwdReduceThreads / kHV) {
      x += dgg_ws[t * kHV + hv];
      y += da[t * kHV + hv];
    }
  // lanes h, h + 8, h + 16, h + 24 hold head h
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  y += __shfl_xor_sync(0xffffffffu, y, 8);
  x += __shfl_xor_sync(0xffffffffu, x, 16);
  y += __shfl_xor_sync(0xffffffffu, y, 16);
  if (lane < kHV) {
    s1[warp][lane] = x;
    s2[warp][lane] = y;
  }
  __syncthreads();
  if (tid < kHV) {
    float a1 = 0.f, a2 = 0.f;
    for (int w = 0; w < kBwdReduceThreads / 32; ++w) {
      a1 += s1[w][tid];
      a2 += s2[w][tid];
    }
    red[(static_cast<int64_t>(blockIdx.x) * kHV + tid) * 2] = a1;
    red[(static_cast<int64_t>(blockIdx.x) * kHV + tid) * 2 + 1] = a2;
  }
}

// Stage 2: one CTA per v-head sums the kBwdRedBlocks partials in a fixed
// order.
static_assert(kBwdRedBlocks == kBwdReduceThreads, "one partial per thread");
__global__ void __launch_bounds__(kBwdReduceThreads)
gdn_prefill_bwd_reduce_kernel(const float *__restrict__ red, float *__restrict__ dA_log,
                              float *__restrict__ ddt_bias) {
  __shared__ float s1[kBwdReduceThreads / 32], s2[kBwdReduceThreads / 32];
  const int hv = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float x = red[(static_cast<int64_t>(tid) * kHV + hv) * 2];
  float y = red[(static_cast<int64_t>(tid) * kHV + hv) * 2 + 1];
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
int prefill_bwd_kernel_launches() { return 7; }

// Clusters of the chunk kernel that are resident at once on this device (one
// CTA per SM, two SMs of a GPC per cluster), queried once per device.
static cudaError_t bwd_chunk_clusters(cudaLaunchConfig_t cfg, int *out) {
  static int cache[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *out = cache[dev];
    return cudaSuccess;
  }
  cfg.gridDim = dim3(2);
  int n = 0;
  err = cudaOccupancyMaxActiveClusters(&n, gdn_prefill_bwd_chunk_kernel, &cfg);
  if (err != cudaSuccess) return err;
  if (n < 1) return cudaErrorInvalidConfiguration;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  *out = n;
  return cudaSuccess;
}

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
  int4 *chunk_tab = reinterpret_cast<int4 *>(ws + f.chunk_tab);
  float *gcum = reinterpret_cast<float *>(ws + f.gcum);
  float *beta = reinterpret_cast<float *>(ws + f.beta);
  uint8_t *m2 = ws + f.m2;
  int4 *items = reinterpret_cast<int4 *>(ws + f.items);
  int *seg_off = reinterpret_cast<int *>(ws + f.seg_off);
  uint8_t *states = ws + w.states;
  uint8_t *dsc = ws + w.dsc;
  uint8_t *delta = ws + w.delta;
  uint8_t *dx = ws + w.dx;
  float *dgg = reinterpret_cast<float *>(ws + w.dgg);

  CUtensorMap tq, tk, tv;
  memset(&tq, 0, sizeof(tq));
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  if (T > 0) {
    if (!make_tmap_2d(&tq, q, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tk, k, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tv, v, kHV * kD, T, 64, 64, true))
      return cudaErrorInvalidValue;
  }
  cudaError_t err;

  // recompute: tables, gates and [P Ainv ; Ainv], then the scan saving S_0 and delta
  gdn_prefill_meta_kernel<<<1, kMetaThreads, 0, stream>>>(
      cu_seqlens, static_cast<int>(N), T, f.nt_max, meta, chunk_off, seq_order, chunk_tab, 0, 0,
      items, seg_off, nullptr, 0);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(gdn_prefill_prep_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPrepSmem);
  if (err != cudaSuccess) return err;
  if (f.nt_max > 0) {
    dim3 grid(static_cast<unsigned>(f.nt_max), kHQK);
    gdn_prefill_prep_kernel<true><<<grid, kPrepThreads, kPrepSmem, stream>>>(
        tq, tk, A_log, static_cast<const uint16_t *>(a), dt_bias,
        static_cast<const uint16_t *>(b), cu_seqlens, meta, chunk_tab, gcum, beta, m2);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  err = cudaFuncSetAttribute(gdn_prefill_scan_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, ScanSmemT<true>::kBytes);
  if (err != cudaSuccess) return err;
  gdn_prefill_scan_kernel<true><<<static_cast<unsigned>(N * kHV), kScanThreads, ScanSmemT<true>::kBytes,
                                  stream>>>(
      tq, tk, tv, tv /* no outputs: the store map is never used */, state, cu_seqlens, meta,
      chunk_off, gcum, beta, m2, scale, nullptr, nullptr,
      items, kMetaPass1, int64_t{1} << 40, seg_off, nullptr, nullptr, nullptr, nullptr, states,
      delta);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  // reverse scan
  CUtensorMap tdo;
  memset(&tdo, 0, sizeof(tdo));
  if (T > 0 && !make_tmap_2d(&tdo, d_out, kHV * kD, T, 64, 64, true)) return cudaErrorInvalidValue;
  err = cudaFuncSetAttribute(gdn_prefill_bwd_scan_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, BwdScanSmem::kBytes);
  if (err != cudaSuccess) return err;
  gdn_prefill_bwd_scan_kernel<<<static_cast<unsigned>(N * kHV), kBwdScanThreads,
                                BwdScanSmem::kBytes, stream>>>(
      tq, tk, tdo, d_final, cu_seqlens, meta, chunk_off, seq_order, gcum, beta, m2, scale, dsc, dx,
      dv, d_state);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  // chunk-parallel gradients: persistent clusters of two CTAs, as many as fit
  if (f.nt_max > 0 && T > 0) {
    const CUtensorMap &tvs = tv;  // V with 128-byte swizzle, 64-wide boxes
    err = cudaFuncSetAttribute(gdn_prefill_bwd_chunk_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, BwdTcSmem::kBytes);
    if (err != cudaSuccess) return err;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kBwdTcThreads);
    cfg.dynamicSmemBytes = BwdTcSmem::kBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    err = bwd_chunk_clusters(cfg, &clusters);
    if (err != cudaSuccess) return err;
    const int npairs = static_cast<int>(f.nt_max * kHQK);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (clusters < npairs ? clusters : npairs)));
    err = cudaLaunchKernelEx(&cfg, gdn_prefill_bwd_chunk_kernel, tq, tk, tdo, tvs, A_log,
                             static_cast<const uint16_t *>(a), dt_bias, cu_seqlens, meta, chunk_tab,
                             gcum, beta, states, dsc, delta, dx, scale, npairs, dq, dk, da, db, dgg);
    if (err != cudaSuccess) return err;
  }
  float *red = reinterpret_cast<float *>(ws + w.red);
  gdn_prefill_bwd_reduce_partial_kernel<<<kBwdRedBlocks, kBwdReduceThreads, 0, stream>>>(
      meta, dgg, da, T, red);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  gdn_prefill_bwd_reduce_kernel<<<kHV, kBwdReduceThreads, 0, stream>>>(red, dA_log, ddt_bias);
  return cudaGetLastError();
}

}  // namespace gdn
