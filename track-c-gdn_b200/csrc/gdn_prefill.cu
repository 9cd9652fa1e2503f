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
//   3. gdn_prefill_scan_kernel   (one CTA per (work item, v-head)) runs the
//      inter-chunk scan with the fp32 state held in registers and a bf16 copy
//      in TMEM as the A operand of the first MMA (the other two MMAs take
//      their A operands, X and V_dec, from TMEM as well);
//   4. gdn_prefill_compose_kernel (segmented evaluation only) joins the
//      segments' affine state maps in fp32.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "gdn_common.cuh"
#include "gdn_wait.cuh"
#include "sm100.cuh"

namespace gdn {
using namespace sm100;

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
// Scan work items (int4 {sequence, segment, mode, 0}).  Without segmentation
// every sequence is one FULL item.  With segmentation (few long sequences),
// sequence n is cut into P_n segments of `seg_chunks` chunks and evaluated
// in three passes, using that the state map of a segment is affine:
//   S_end = S_start Phi + B,
// Phi = the segment's final state from S = I with v = 0, B = its final state
// from S = 0.
//   pass 1 (parallel): HEAD (segment 0 from h0, with outputs; its final state
//          is S_start of segment 1), ZERO (B of segments 1..P-2), IDENT (Phi of
//          segments 1..P-2), FULL (sequences with one segment);
//   compose (sequential per sequence, cheap): S_start(p+1) = S_start(p) Phi(p) + B(p);
//   pass 3 (parallel): MID / TAIL (segments 1..P-1 from S_start(p), with
//          outputs; TAIL writes the final state).
enum ScanItemMode : int { kItemFull = 0, kItemHead, kItemZero, kItemIdent, kItemMid, kItemTail };

// Header written by the metadata kernel: chunk count, error flag, work items
// of pass 1 and pass 3, and the call's sizes (read by the debug-build index
// checks).
enum MetaSlot : int { kMetaChunks = 0, kMetaError, kMetaPass1, kMetaPass3, kMetaN, kMetaT };

// Segmented evaluation is used for at most this many sequences.
constexpr int kSegMaxSeqs = 16;
// Scan CTAs that run at once on a B200 (148 SMs x 2 CTAs).
constexpr int64_t kScanSlots = 296;

struct PrefillWs {
  size_t meta, chunk_off, seq_order, chunk_tab, gcum, beta, m2, items, seg_off, seg_ss, seg_sb,
      seg_phi, total;
  int64_t nt_max;
  int64_t seg_chunks;  // 0: no segmentation
  int64_t seg_max;     // bound on the number of segments (segmented mode)
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr size_t kM2Bytes = 128 * 128;  // [PA ; Ainv] 128 rows x 64 bf16
// The forward's [P ; Ainv] image keeps only what can be nonzero.  P and Ainv
// are lower triangular (column s <= row t), so the 16 columns of K-step ks
// (s = 16 ks .. 16 ks + 15) are nonzero only in rows t >= 16 ks: K-step ks is
// stored as rows 16 ks .. 63 in the no-swizzle K-major operand layout (core
// matrices of 8 rows x 16 bytes; 8-row groups 256 B apart, the two 8-column
// halves 128 B apart) and the scan's MMAs over it have N = 64 - 16 ks.
// One matrix is 5 KiB (5/8 of the full 8 KiB), the image 10 KiB.
constexpr size_t kTriBytes = 5120;
constexpr size_t kImgFwdBytes = 2 * kTriBytes;
constexpr uint32_t kTriSbo = 256, kTriLbo = 128;
// byte offset of K-step ks (0..4) inside one matrix
__host__ __device__ constexpr uint32_t tri_step_off(int ks) {
  return static_cast<uint32_t>(2048 * ks - 256 * ks * (ks - 1));
}
static_assert(tri_step_off(4) == kTriBytes, "K-step offsets");
// byte offset of the 16-byte piece cc (columns 8 cc .. 8 cc + 7) of row t;
// stored only for cc / 2 <= t / 16
__device__ __forceinline__ uint32_t tri_off(int t, int cc) {
  const int ks = cc >> 1, r = t - 16 * ks;
  return tri_step_off(ks) + static_cast<uint32_t>((r >> 3) * kTriSbo + (cc & 1) * kTriLbo + (r & 7) * 16);
}
constexpr size_t kStateBytes = static_cast<size_t>(kHV) * kD * kD * sizeof(float);
// a 128 x 128 state (one v-head) as a bf16 tensor-core operand image
constexpr size_t kStateImgBytes = static_cast<size_t>(kD) * kD * 2;
// 64 tokens x 128 values of one v-head (one chunk of delta or dX) as a bf16
// K-major operand image: 2 v-blocks x 64 token rows x 128 B, 128-byte swizzle
constexpr size_t kTokImgBytes = static_cast<size_t>(kChunk) * kD * 2;

// element (t, v) of a token image
__device__ __forceinline__ void put_tok_img(uint8_t *img, int t, int v, float x) {
  *reinterpret_cast<__nv_bfloat16 *>(img + (v >> 6) * 8192 + t * 128 +
                                     ((((v >> 3) ^ t) & 7) << 4) + (v & 7) * 2) =
      __float2bfloat16_rn(x);
}

// Row `row` (v) of a state image, k = 64 hc .. 64 hc + 63 from x[]: the
// MN-major operand layout (2 k-blocks x 128 v rows x 128 B, 128-byte
// swizzle) that tcgen05 reads with k contiguous.
__device__ __forceinline__ void put_state_img_row(uint8_t *img, int row, int hc, const float *x) {
  uint8_t *r = img + hc * 16384 + row * 128;
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
    *reinterpret_cast<uint4 *>(r + ((cc ^ (row & 7)) << 4)) =
        make_uint4(pack_bf16x2(x[8 * cc], x[8 * cc + 1]), pack_bf16x2(x[8 * cc + 2], x[8 * cc + 3]),
                   pack_bf16x2(x[8 * cc + 4], x[8 * cc + 5]), pack_bf16x2(x[8 * cc + 6], x[8 * cc + 7]));
}

// Segment length (chunks) chosen from T and N alone, so that the workspace
// size is a function of (T, N): segment only when there are fewer scan
// chains (8 per sequence) than SMs and the sequences average at least 12
// chunks; make pass 1 (about two CTAs per segment and v-head) fit one wave.
inline int64_t prefill_segment_chunks(int64_t T, int64_t N) {
  if (N <= 0 || N > kSegMaxSeqs) return 0;
  const int64_t nt = (T + kChunk - 1) / kChunk;
  if (nt < 12 * N) return 0;
  const int64_t lc = (16 * (nt + N) + kScanSlots - 1) / kScanSlots;
  return lc < 4 ? 4 : lc;
}

inline PrefillWs prefill_ws_layout(int64_t T, int64_t N, bool allow_segments = true) {
  PrefillWs w;
  w.nt_max = (T + kChunk - 1) / kChunk + N;
  w.seg_chunks = allow_segments ? prefill_segment_chunks(T, N) : 0;
  w.seg_max = w.seg_chunks ? N + (w.nt_max + w.seg_chunks - 1) / w.seg_chunks : 0;
  const int64_t n_items = w.seg_chunks ? 3 * w.seg_max : N;
  size_t off = 0;
  w.meta = off;  // kMeta* slots
  off = align_up(off + 8 * sizeof(int), 256);
  w.chunk_off = off;
  off = align_up(off + (N + 1) * sizeof(int), 256);
  w.seq_order = off;
  off = align_up(off + N * sizeof(int), 256);
  w.chunk_tab = off;
  off = align_up(off + w.nt_max * sizeof(int4), 256);
  w.items = off;
  off = align_up(off + n_items * sizeof(int4), 256);
  w.seg_off = off;
  off = align_up(off + (N + 1) * sizeof(int), 256);
  w.gcum = off;
  off = align_up(off + T * kHV * sizeof(float), 256);
  w.beta = off;
  off = align_up(off + T * kHV * sizeof(float), 1024);
  w.m2 = off;
  off = align_up(off + static_cast<size_t>(w.nt_max) * kHV * kM2Bytes, 1024);
  w.seg_ss = off;
  off = align_up(off + static_cast<size_t>(w.seg_max) * kStateBytes, 1024);
  w.seg_sb = off;
  off = align_up(off + static_cast<size_t>(w.seg_max) * kStateBytes, 1024);
  w.seg_phi = off;
  off = align_up(off + static_cast<size_t>(w.seg_max) * kStateBytes, 1024);
  w.total = off;
  return w;
}

// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t lmin(int64_t x, int64_t y) { return x < y ? x : y; }

// Aligns the dynamic shared-memory base to A bytes by offsetting the
// __shared__ array itself (not through an integer cast), so the compiler
// still knows every access through the result is a shared-memory access.
template <uint32_t A>
__device__ __forceinline__ uint8_t *smem_align(uint8_t *raw) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(raw));
  return raw + ((A - (a & (A - 1))) & (A - 1));
}

__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ---------------------------------------------------------------------------
// 1. metadata
// ---------------------------------------------------------------------------
constexpr int kMetaThreads = 1024;
constexpr int kLptMaxSeqs = 2048;

__global__ void __launch_bounds__(kMetaThreads)
gdn_prefill_meta_kernel(const int64_t *__restrict__ cu, int N, int64_t T, int64_t nt_max,
                        int *meta, int *chunk_off, int *seq_order, int4 *chunk_tab,
                        int seg_chunks, int seg_max, int4 *items, int *seg_off,
                        const int32_t *__restrict__ slots, int64_t pool_slots) {
  __shared__ int s_wtot[32];
  __shared__ int s_carry;
  __shared__ int s_nc[kLptMaxSeqs];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    meta[kMetaN] = N;
    meta[kMetaT] = static_cast<int>(T < 0x7fffffff ? T : 0x7fffffff);
  }

  // state-pool slots (when given) must lie in the pool
  int bad_slot = 0;
  if (slots != nullptr)
    for (int i = tid; i < N; i += kMetaThreads)
      if (slots[i] < 0 || slots[i] >= pool_slots) bad_slot = 1;
  if (__syncthreads_or(bad_slot)) {
    if (tid == 0) {
      meta[0] = 0;
      meta[1] = 1;
      meta[2] = meta[3] = 0;
      set_device_status(kDevStatusBadSlot);
    }
    return;
  }

  int bad = 0;
  for (int i = tid; i < N; i += kMetaThreads)
    if (cu[i + 1] < cu[i]) bad = 1;
  if (tid == 0 && (cu[0] != 0 || cu[N] != T)) bad = 1;
  if (__syncthreads_or(bad)) {
    if (tid == 0) {
      meta[0] = 0;
      meta[1] = 1;
      meta[2] = meta[3] = 0;
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
    meta[2] = meta[3] = 0;
    if (!ok) set_device_status(kDevStatusBadSeqlens);
  }
  if (nt > nt_max) return;
  __syncthreads();
  // chunk table: (sequence, chunk of it, first token, tokens), so that a
  // chunk's kernels find its place with one load (T < 2^31 tokens)
  for (int i = tid; i < N; i += kMetaThreads) {
    const int off = chunk_off[i], nc = chunk_off[i + 1] - off;
    const int64_t b0 = cu[i], len = cu[i + 1] - b0;
    for (int c = 0; c < nc; ++c)
      chunk_tab[off + c] = make_int4(i, c, static_cast<int>(b0 + static_cast<int64_t>(c) * kChunk),
                                     static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk)));
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
  __syncthreads();

  // Scan work items (see ScanItemMode).  meta[2] = pass-1 items, meta[3] =
  // pass-3 items.
  if (seg_chunks == 0) {
    for (int i = tid; i < N; i += kMetaThreads) items[i] = make_int4(seq_order[i], 0, kItemFull, 0);
    if (tid == 0) {
      meta[2] = N;
      meta[3] = 0;
    }
    return;
  }
  // Segmented (N <= kSegMaxSeqs): thread 0 builds the tables, longest
  // sequences first.  Pass-1 items occupy items[0, 2 seg_max), pass-3 items
  // items[2 seg_max, 3 seg_max).
  if (tid == 0) {
    int so = 0;
    for (int i = 0; i < N; ++i) {
      const int nc = chunk_off[i + 1] - chunk_off[i];
      seg_off[i] = so;
      so += nc > seg_chunks ? (nc + seg_chunks - 1) / seg_chunks : 1;
    }
    seg_off[N] = so;
    if (so > seg_max) {  // cannot happen for a valid cu_seqlens (bound of the layout)
      meta[1] = 1;
      meta[2] = meta[3] = 0;
      set_device_status(kDevStatusBadSeqlens);
      return;
    }
    int n1 = 0, n3 = 0;
    int4 *items3 = items + 2 * seg_max;
    for (int j = 0; j < N; ++j) {
      const int i = seq_order[j];
      const int P = seg_off[i + 1] - seg_off[i];
      if (P == 1) {
        items[n1++] = make_int4(i, 0, kItemFull, 0);
        continue;
      }
      items[n1++] = make_int4(i, 0, kItemHead, 0);
      for (int p = 1; p + 1 < P; ++p) {
        items[n1++] = make_int4(i, p, kItemZero, 0);
        items[n1++] = make_int4(i, p, kItemIdent, 0);
      }
      for (int p = 1; p < P; ++p) items3[n3++] = make_int4(i, p, p + 1 < P ? kItemMid : kItemTail, 0);
    }
    meta[2] = n1;
    meta[3] = n3;
  }
}

// ---------------------------------------------------------------------------
// 2. chunk-parallel preparation
// ---------------------------------------------------------------------------
// One CTA per (chunk, q/k head), 128 threads, both v-heads j = 0, 1 of the
// q/k head.  The [Q;K] tile arrives by TMA; D = [Q;K] K^T on the tensor core
// gives Q K^T (TMEM lanes 0..63) and K K^T (lanes 64..127) at once; each
// thread turns one row into P_j (bf16, parked in its own TMEM lane) or A_j
// (fp32, shared memory); (I + A_j)^-1 is a 2 x 2 block inverse: thread
// (j, c) solves column c of its 32 x 32 diagonal block by fp32 forward
// substitution, and the block products run as warp-level TF32 MMAs; P moves
// into the retired A region and a second MMA forms P_j Ainv_j.  Output per (chunk, v-head): the 16 KiB [P Ainv ; Ainv]
// image in the scan kernel's shared-memory operand layout.  About 51 KB of
// shared memory, 128 TMEM columns and 128 registers per thread: 4 CTAs/SM.
constexpr int kPrepThreads = 128;
// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kPrepQK = 0;          // [Q;K] tile 32 KB; after MMA 1 the fp32 A_0, A_1;
                                    // after the solve [P_0 ; P_1] bf16, K-major 128 x 64
constexpr int kPrepAI = 32768;      // Ainv_0, Ainv_1 bf16, 64 x 64 each (2 x 8 KB)
constexpr int kPrepG = 49152;       // float G[2][64]
constexpr int kPrepB = kPrepG + 512;    // float beta[2][64]
constexpr int kPrepGn = kPrepB + 512;   // float gnext[2][64]: e^{gl_{t+1}} (1 at t = 63)
constexpr int kPrepWt = kPrepGn + 512;  // float warp totals[4]
constexpr int kPrepBar = kPrepWt + 16;  // mbarriers: mma, tma
constexpr int kPrepTmem = kPrepBar + 16;
constexpr int kPrepBroken = kPrepTmem + 4;
constexpr int kPrepSmem = kPrepBroken + 12 + 1024;  // + base alignment slack
constexpr uint32_t kPrepTmemCols = 128;

// (I + A)^-1 for a strictly lower-triangular 64 x 64 fp32 A (given transposed,
// AT[col * 64 + row]) as a 2 x 2 block inverse of 32 x 32 blocks:
//   [L11 0; L21 L22]^-1 = [X11 0; X21 X22],  X11 = L11^-1, X22 = L22^-1,
//   X21 = -X22 (L21 X11).
// Step 1 (this function): thread (h, lane) solves column c = 32 h + lane of
// its diagonal block X_hh by blocked forward substitution in fp32 (16-row
// blocks, A's columns broadcast from shared memory; the coupling of the
// second 16-row block to the first is one warp-level TF32 product), keeps
// the x values in its TMEM lane (columns txs + 32 h ..) and writes them as
// bf16 into the 64 x 64 Ainv image `img` (128-byte rows, 128-byte swizzle),
// with the zeros above the diagonal block for h = 1.  Steps 2 and 3 (the two
// products) run in the kernel, split over all four warps.
__device__ __forceinline__ void img_put(uint8_t *img, int r, int c, float x) {
  *reinterpret_cast<__nv_bfloat16 *>(img + r * 128 + (((c >> 3) ^ (r & 7)) << 4) + (c & 7) * 2) =
      __float2bfloat16_rn(x);
}

// Elements (r, c) and (r, c + 1) of the image, c even: one 32-bit store.
__device__ __forceinline__ void img_put2(uint8_t *img, int r, int c, float x0, float x1) {
  *reinterpret_cast<uint32_t *>(img + r * 128 + (((c >> 3) ^ (r & 7)) << 4) + (c & 7) * 2) =
      pack_bf16x2(x0, x1);
}

// fp32 -> tf32 (round to nearest, ties away from zero), as a 32-bit pattern.
__device__ __forceinline__ uint32_t f32_to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// d[16 x 8] += a[16 x 8] b[8 x 8], one warp, tf32 operands, fp32 accumulator.
// Fragments (g = lane / 4, t = lane % 4): a = {(g, t), (g + 8, t), (g, t + 4),
// (g + 8, t + 4)}, b = {(t, g), (t + 4, g)}, d = {(g, 2t), (g, 2t + 1),
// (g + 8, 2t), (g + 8, 2t + 1)}.
__device__ __forceinline__ void mma_tf32_m16n8k8(float (&d)[4], const uint32_t (&a)[4],
                                                 const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void solve_diag_block_column(const float *AT, float *scr, int lane,
                                                        int h, uint32_t txs, uint8_t *img) {
  const int c = 32 * h + lane;
  if (h == 1) {
    // rows 0..31, columns 32..63 of the image are zero: 16-byte stores
#pragma unroll
    for (int ch = 4; ch < 8; ++ch)
      *reinterpret_cast<uint4 *>(img + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
          make_uint4(0u, 0u, 0u, 0u);
  }
  // The warp's scratch `scr` holds 32 rows n of 16 floats: element k of row n
  // at scr[(n >> 1) * 64 + (n & 1) * 16 + (k ^ 4 ((n >> 1) & 3))], a layout in
  // which the fragment loads, the float4 row accesses and (up to two-way) the
  // accumulator stores below are free of bank conflicts.
  const int g = lane >> 2, t4 = lane & 3, sq = (lane >> 1) & 3;
  float *srow = scr + (lane >> 1) * 64 + (lane & 1) * 16;
#pragma unroll 1
  for (int bb = 0; bb < 2; ++bb) {
    const int r0 = 32 * h + 16 * bb;
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    if (bb == 1) {
      // contribution of the block above, within the diagonal block, for the
      // warp's 32 columns at once: acc = A[r0 .., 32 h ..] X[32 h .., c] as
      // one 16 x 32 x 16 TF32 product (block 0's x values are in `scr`)
      float d[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
        const float *ap = AT + (32 * h + 8 * kt + t4) * 64 + r0 + g;
        const uint32_t af[4] = {f32_to_tf32(ap[0]), f32_to_tf32(ap[8]), f32_to_tf32(ap[4 * 64]),
                                f32_to_tf32(ap[4 * 64 + 8])};
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int n = 8 * nt + g, s = 4 * ((n >> 1) & 3);
          const float *bp = scr + (n >> 1) * 64 + (n & 1) * 16;
          const uint32_t bf[2] = {f32_to_tf32(bp[(8 * kt + t4) ^ s]),
                                  f32_to_tf32(bp[(8 * kt + t4 + 4) ^ s])};
          mma_tf32_m16n8k8(d[nt], af, bf);
        }
      }
      __syncwarp();  // every lane's fragment loads are done: reuse `scr` for D
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int n = 8 * nt + 2 * t4, s = 4 * ((n >> 1) & 3);
        float *p = scr + (n >> 1) * 64;  // rows n (even) and n + 1
        p[g ^ s] = d[nt][0];
        p[16 + (g ^ s)] = d[nt][1];
        p[(g + 8) ^ s] = d[nt][2];
        p[16 + ((g + 8) ^ s)] = d[nt][3];
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = *reinterpret_cast<const float4 *>(srow + 4 * (q ^ sq));
        acc[4 * q] = v.x;
        acc[4 * q + 1] = v.y;
        acc[4 * q + 2] = v.z;
        acc[4 * q + 3] = v.w;
      }
    }
    // inside the 16-row block, right-looking: x_jp is final once the rows
    // above have been applied; column jp of A (float4 reads down the column)
    // then updates the rows below it, so the dependent chain is one FMA per
    // row rather than a dot product per row
    float xb[16];
#pragma unroll
    for (int jp = 0; jp < 16; ++jp) {
      const int r = r0 + jp;
      xb[jp] = (r == c) ? 1.f : (r < c ? 0.f : -acc[jp]);
      const float *colp = AT + (r0 + jp) * 64 + r0;
      const uint64_t xx = f2_pack(xb[jp], xb[jp]);
#pragma unroll
      for (int q = (jp + 1) / 4; q < 4; ++q) {
        const float4 a = *reinterpret_cast<const float4 *>(colp + 4 * q);
        // rows 4q .. 4q+3 below jp: one packed pair (f32x2) where both rows are
        if (4 * q + 0 > jp) {
          const uint64_t r = f2_fma(f2_pack(a.x, a.y), xx, f2_pack(acc[4 * q], acc[4 * q + 1]));
          acc[4 * q] = f2_lo(r);
          acc[4 * q + 1] = f2_hi(r);
        } else if (4 * q + 1 > jp) {
          acc[4 * q + 1] += a.y * xb[jp];
        }
        if (4 * q + 2 > jp) {
          const uint64_t r = f2_fma(f2_pack(a.z, a.w), xx, f2_pack(acc[4 * q + 2], acc[4 * q + 3]));
          acc[4 * q + 2] = f2_lo(r);
          acc[4 * q + 3] = f2_hi(r);
        } else if (4 * q + 3 > jp) {
          acc[4 * q + 3] += a.w * xb[jp];
        }
      }
    }
    if (bb == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4 *>(srow + 4 * (q ^ sq)) =
            make_float4(xb[4 * q], xb[4 * q + 1], xb[4 * q + 2], xb[4 * q + 3]);
      __syncwarp();
    }
    uint32_t u[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(xb[i]);
    tmem_st16(txs + 16 * (2 * h + bb), u);
    tmem_wait_st();
#pragma unroll
    for (int i = 0; i < 16; ++i) img_put(img, r0 + i, c, xb[i]);
  }
}

// kPA: the image is [P Ainv ; Ainv] (the backward's recompute and gradient
// kernels use P Ainv); otherwise [P ; Ainv] (the forward scan forms its
// intra-chunk output from P itself), and the P rows go to the workspace
// straight from the A/P phase, with no P Ainv product.
template <bool kPA>
__global__ void __launch_bounds__(kPrepThreads, 4)
gdn_prefill_prep_kernel(const __grid_constant__ CUtensorMap tmap_q,
                        const __grid_constant__ CUtensorMap tmap_k,
                        const float *__restrict__ A_log, const uint16_t *__restrict__ a,
                        const float *__restrict__ dt_bias, const uint16_t *__restrict__ b,
                        const int64_t *__restrict__ cu, const int *__restrict__ meta,
                        const int4 *__restrict__ chunk_tab, float *__restrict__ gcum_ws,
                        float *__restrict__ beta_ws, uint8_t *__restrict__ m2_ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  const int gchunk = blockIdx.x, hqk = blockIdx.y;
  // the chunk's entry is read alongside the count (the grid covers the
  // table's nt_max entries; one past the count is never used)
  const int4 e = chunk_tab[gchunk];
  if (meta[1] != 0 || gchunk >= meta[0]) return;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  GDN_DCHECK(e.x >= 0 && e.x < meta[kMetaN] && e.y >= 0);
  const int64_t t0 = e.z;
  const int L = e.w;
  GDN_DCHECK(t0 == cu[e.x] + static_cast<int64_t>(e.y) * kChunk && L > 0 && t0 + L <= meta[kMetaT]);

  uint8_t *qk = smem + kPrepQK;
  uint8_t *pp = smem + kPrepQK;  // P image, written only once A is no longer read
  uint8_t *ai = smem + kPrepAI;
  float *Gs = reinterpret_cast<float *>(smem + kPrepG);
  float *Bs = reinterpret_cast<float *>(smem + kPrepB);
  float *Gn = reinterpret_cast<float *>(smem + kPrepGn);
  float *wt = reinterpret_cast<float *>(smem + kPrepWt);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + kPrepBroken);
  const uint32_t bar = smem_u32(smem + kPrepBar), bar_tma = bar + 8;

  if (warp == 0) tmem_alloc(smem_u32(smem + kPrepTmem), kPrepTmemCols);
  if (tid == 0) {
    *broken = 0;
    mbar_init(bar, 1);
    mbar_init_fence();
    mbar_init(bar_tma, 1);
    mbar_init_fence();
    // [Q;K] tile: Q rows 0..63 and K rows 64..127 of each 64-wide d-block
    mbar_arrive_expect_tx(bar_tma, 32768);
    const uint32_t base = smem_u32(qk);
    for (int blk = 0; blk < 2; ++blk) {
      tma_load_2d(base + blk * 16384, &tmap_q, hqk * kD + 64 * blk, static_cast<int>(t0), bar_tma);
      tma_load_2d(base + blk * 16384 + 8192, &tmap_k, hqk * kD + 64 * blk, static_cast<int>(t0),
                  bar_tma);
    }
  }

  // Gate inputs of token t = tid % 64 for v-head 2 hqk + tid / 64 (zero past
  // the chunk's end): loaded now, turned into the gates while MMA 1 runs.
  const int gj = tid >> 6, gt = tid & 63, ghv = 2 * hqk + gj;
  const bool gvalid = gt < L;
  uint16_t g_a = 0, g_b = 0;
  const float g_alog = A_log[ghv], g_dtb = dt_bias[ghv];
  if (gvalid) {
    const int64_t idx = (t0 + gt) * kHV + ghv;
    g_a = a[idx];
    g_b = b[idx];
  }
  // thread 0's mbarrier initialisation (and *broken = 0) before any thread
  // polls the barrier
  __syncthreads();

  wait_phase(bar_tma, 0, broken);
  if (L < kChunk) {
    // rows past the sequence end hold the next sequence's tokens: zero them
    for (int idx = tid; idx < 4 * (kChunk - L) * 8; idx += kPrepThreads) {
      const int ch = idx & 7, rr = (idx >> 3) % (kChunk - L), blk = (idx >> 3) / (kChunk - L);
      *reinterpret_cast<uint4 *>(qk + (blk >> 1) * 16384 + (blk & 1) * 8192 + (L + rr) * 128 +
                                 ch * 16) = make_uint4(0u, 0u, 0u, 0u);
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
    const uint64_t dqk = umma_desc_sw128(smem_u32(qk), 16, 1024);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
      umma_bf16(tmem, umma_desc_advance(dqk, off), umma_desc_advance(dqk, 8192 + off), idesc, ks > 0);
    }
    umma_commit(bar);
  }
  // Gates for v-heads 2*hqk + j (j = tid / 64), token t = tid % 64, while the
  // MMA runs.
  {
    const int j = gj, t = gt;
    const bool valid = gvalid;
    float gl = 0.f, bt = 0.f;
    if (valid) {
      gl = -expf(g_alog) * softplus_stable(bf16_to_f32(g_a) + g_dtb);
      bt = 1.0f / (1.0f + expf(-bf16_to_f32(g_b)));
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
    // per-token decay e^{gl_t} (1 past the end), stored one slot down so that
    // gnext[c] = e^{gl_{c+1}}: the factor that extends a row's running decay
    // product from column c+1 to column c
    Gn[j * 64 + (t == 0 ? 63 : t - 1)] = t == 0 ? 1.f : expf(gl);
    if (valid) {
      const int64_t idx = (t0 + t) * kHV + ghv;
      gcum_ws[idx] = x;
      beta_ws[idx] = bt;
    }
  }
  // the gates (Gs, Bs, Gn) are read by the A/P rows after the barrier below
  __syncthreads();
  wait_phase(bar, 0, broken);
  tc_fence_after();

  // A_j^T (fp32, into the retired [Q;K] region: AT[j][col][row], so a warp's
  // stores for one column are 32 consecutive floats) from the K K^T rows
  // (warps 2,3) and P_j (bf16 operand rows) from the Q K^T rows (warps 0,1),
  // eight accumulator columns at a time, right to left: the decay factor
  // e^{G_i - G_c} = prod_{k=c+1..i} e^{gl_k} of row i is a running product
  // (no per-entry exponential; exact to fp32 rounding, never overflows).
  float *AT = reinterpret_cast<float *>(smem + kPrepQK);
  {
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    // Rows 0..31 (warps 0 and 2) have no nonzero entry right of column 31:
    // their P rows are zero there and their A rows are not stored there (that
    // block of A is never read; the solve uses it as scratch).
    auto rows = [&](auto upper_tag) {
      constexpr bool kUpper = decltype(upper_tag)::value;
      constexpr int kGroups = kUpper ? 4 : 8;  // 8-column groups that can be nonzero
      // row i of this thread, as an expression the compiler can bound: the
      // lower rows' column tests in groups 0..3 (columns 0..31 < 32 <= i)
      // then fold to true
      const int i = kUpper ? lane : 32 + lane;
      const bool rv = i < L;
      float acc[8 * kGroups];  // row i of Q K^T (warps 0,1) or K K^T (warps 2,3)
      tmem_ld32(trow, *reinterpret_cast<float(*)[32]>(acc));
      if constexpr (!kUpper) tmem_ld32(trow + 32, *reinterpret_cast<float(*)[32]>(acc + 32));
      tmem_wait_ld();
      // a row past the sequence end (tail chunks only) is zero in A and P:
      // zero its products once here (0 times a finite, non-negative decay
      // factor is +0, the value the masks below would have written)
      if (!rv) {
#pragma unroll
        for (int u = 0; u < 8 * kGroups; ++u) acc[u] = 0.f;
      }
#pragma unroll 1
      for (int j = 0; j < 2; ++j) {
        // e^{G_i - G_c} for the current column c (1 for c >= i), times beta_i
        // for the A rows (warps 2, 3)
        float dec = warp >= 2 ? Bs[j * 64 + i] : 1.f;
        uint32_t prow[32];  // row i of P_j as bf16 pairs (warps 0,1)
#pragma unroll
        for (int cc = kGroups - 1; cc >= 0; --cc) {
          const float4 g0 = *reinterpret_cast<const float4 *>(Gn + j * 64 + 8 * cc);
          const float4 g1 = *reinterpret_cast<const float4 *>(Gn + j * 64 + 8 * cc + 4);
          const float gn[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          float dc[8];
#pragma unroll
          for (int u = 7; u >= 0; --u) {
            if (8 * cc + u < i) dec *= gn[u];
            dc[u] = dec;
          }
          const float *a8 = acc + 8 * cc;
          float prod[8];  // a8 * dc on packed pairs
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            const uint64_t r = f2_mul(f2_pack(a8[u], a8[u + 1]), f2_pack(dc[u], dc[u + 1]));
            prod[u] = f2_lo(r);
            prod[u + 1] = f2_hi(r);
          }
          if (warp >= 2) {
            // only the strictly lower triangle: nothing reads A at col >= i
            // (the solve masks the entries it loads there)
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int col = 8 * cc + u;
              if (col < i) AT[(j * 64 + col) * 64 + i] = prod[u];
            }
          } else {
            float vals[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int col = 8 * cc + u;
              vals[u] = col <= i ? prod[u] : 0.f;
            }
            prow[4 * cc + 0] = pack_bf16x2(vals[0], vals[1]);
            prow[4 * cc + 1] = pack_bf16x2(vals[2], vals[3]);
            prow[4 * cc + 2] = pack_bf16x2(vals[4], vals[5]);
            prow[4 * cc + 3] = pack_bf16x2(vals[6], vals[7]);
          }
        }
        if constexpr (kUpper) {
#pragma unroll
          for (int k = 16; k < 32; ++k) prow[k] = 0u;
        }
        // D's columns 0..63 were read above; lanes 0..63 now keep P_0 | P_1
        if (warp < 2) {
          if constexpr (kPA) {
            tmem_st32(trow + 32 * j, prow);
          } else {
            // row i of P_j -> row i of the compact image of v-head 2 hqk + j
            // (the K-steps ks <= i / 16)
            uint8_t *img = m2_ws + ((static_cast<size_t>(gchunk) * kHV + 2 * hqk + j) * kImgFwdBytes);
#pragma unroll
            for (int cc = 0; cc < kGroups; ++cc)
              if ((cc >> 1) <= (i >> 4))
                *reinterpret_cast<uint4 *>(img + tri_off(i, cc)) =
                    make_uint4(prow[4 * cc], prow[4 * cc + 1], prow[4 * cc + 2], prow[4 * cc + 3]);
          }
        }
      }
    };
    if (warp & 1)
      rows(std::false_type{});
    else
      rows(std::true_type{});
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // (I + A_j)^-1 as a 2 x 2 block inverse (see solve_diag_block_column).
  // Thread (j = tid / 64, h = warp & 1, lane) owns column 32 h + lane of v-head j.
  {
    const int j = tid >> 6, h = warp & 1;
    float *ATj = AT + j * 4096;
    uint8_t *img = ai + j * 8192;
    const uint32_t txs = tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64;
    // step 1: diagonal blocks X11 (h = 0) and X22 (h = 1), in parallel
    // scratch of step 1: rows 0..31 of columns 32 + 16 h .. 47 + 16 h of A_j,
    // the zero block above L22, which is neither written nor read
    solve_diag_block_column(ATj, ATj + (32 + 16 * h) * 64, lane, h, txs, img);
    tc_fence_before();
    __syncthreads();  // every diagonal block solved: L11 and L22 are no longer read
    tc_fence_after();
    // Steps 2 and 3 are 32 x 32 x 32 products: warp-level TF32 MMAs
    // (m16n8k8, fp32 accumulation) -- the reference merges its blocks in TF32
    // too (kernel.py:718-737), and the result is rounded to bf16 below.
    // Operands are laid out so that every fragment load below is free of
    // bank conflicts:
    //   X11^T in the retired L22 columns, rows padded to 36 floats:
    //         X11T[n * 36 + k] = X11[k][n] (later T^T in the same place);
    //   X22   row-major in the retired L11 area with an XOR-swizzled column:
    //         X22[m][c] at ATj[m * 64 + (c ^ 4 (m & 7))].
    float *X11T = ATj + 32 * 64;
    {
      float x[32];
      tmem_ld32(txs + 32 * h, x);  // x[k] = X_hh[k][lane]
      tmem_wait_ld();
      if (h == 0) {
        float4 *dst = reinterpret_cast<float4 *>(X11T + lane * 36);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) ATj[k * 64 + (lane ^ (4 * (k & 7)))] = x[k];
      }
    }
    __syncthreads();
    // fragment coordinates (PTX m16n8k8 .tf32 layout): g = lane / 4, t = lane % 4
    const int g = lane >> 2, t4 = lane & 3;
    // step 2: T = L21 X11, rows 16 h .. 16 h + 15 (this warp), all 32 columns;
    // L21[r][k] = ATj[k * 64 + 32 + r]
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    {
      const float *l21 = ATj + 32 + 16 * h + g;
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        const int k0 = 8 * kt;
        const uint32_t af[4] = {f32_to_tf32(l21[(k0 + t4) * 64]), f32_to_tf32(l21[(k0 + t4) * 64 + 8]),
                                f32_to_tf32(l21[(k0 + t4 + 4) * 64]),
                                f32_to_tf32(l21[(k0 + t4 + 4) * 64 + 8])};
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const float *bp = X11T + (8 * nt + g) * 36 + k0 + t4;
          const uint32_t bf[2] = {f32_to_tf32(bp[0]), f32_to_tf32(bp[4])};
          mma_tf32_m16n8k8(acc[nt], af, bf);
        }
      }
    }
    __syncthreads();  // X11 fully read: T^T replaces it
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int n = 8 * nt + 2 * t4, m = 16 * h + g;
      X11T[n * 36 + m] = acc[nt][0];
      X11T[(n + 1) * 36 + m] = acc[nt][1];
      X11T[n * 36 + m + 8] = acc[nt][2];
      X11T[(n + 1) * 36 + m + 8] = acc[nt][3];
    }
    __syncthreads();
    // step 3: X21 = -X22 T, rows 16 h .. 16 h + 15 -> image rows 32 .. 63,
    // columns 0 .. 31 (rows m and m + 8 share the swizzle: (m & 7) = g)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    {
      const int m = 16 * h + g;
      const float *x22a = ATj + m * 64, *x22b = ATj + (m + 8) * 64;
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        const int c0 = (8 * kt + t4) ^ (4 * g), c1 = (8 * kt + t4 + 4) ^ (4 * g);
        const uint32_t af[4] = {f32_to_tf32(x22a[c0]), f32_to_tf32(x22b[c0]), f32_to_tf32(x22a[c1]),
                                f32_to_tf32(x22b[c1])};
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const float *bp = X11T + (8 * nt + g) * 36 + 8 * kt + t4;
          const uint32_t bf[2] = {f32_to_tf32(bp[0]), f32_to_tf32(bp[4])};
          mma_tf32_m16n8k8(acc[nt], af, bf);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int c = 8 * nt + 2 * t4;
        img_put2(img, 32 + m, c, -acc[nt][0], -acc[nt][1]);
        img_put2(img, 40 + m, c, -acc[nt][2], -acc[nt][3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();  // every column solved: the A region is free
  tc_fence_after();
  if constexpr (!kPA) {
    // [P ; Ainv]: the P rows are already out; the stored K-steps of Ainv_j
    // (128-byte-swizzled rows in shared memory) -> the compact image's second
    // matrix, one 16-byte piece per iteration, consecutive in global memory
    uint8_t *img0 = m2_ws + (static_cast<size_t>(gchunk) * kHV + 2 * hqk) * kImgFwdBytes + kTriBytes;
    // K-step by K-step (compile-time bounds): step ks holds rows 16 ks .. 63,
    // (64 - 16 ks) x 2 pieces per matrix
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int n = (64 - 16 * ks) * 2, base = static_cast<int>(tri_step_off(ks) >> 4);
      for (int idx = tid; idx < 2 * n; idx += kPrepThreads) {
        const int j = idx >= n, qb = idx - j * n;
        const int t = 16 * ks + (qb >> 4) * 8 + (qb & 7), cc = 2 * ks + ((qb >> 3) & 1);
        reinterpret_cast<uint4 *>(img0 + j * kImgFwdBytes)[base + qb] =
            *reinterpret_cast<const uint4 *>(ai + j * 8192 + sw128(t, cc));
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tmem, kPrepTmemCols);
    }
    return;
  }
  uint8_t *img0 = m2_ws + (static_cast<size_t>(gchunk) * kHV + 2 * hqk) * kM2Bytes;
  if (warp < 2) {
    const int i = warp * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * warp) << 16);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float prow[32];  // bf16 pairs, as raw 32-bit words
      tmem_ld32(trow + 32 * j, prow);
      tmem_wait_ld();
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
        *reinterpret_cast<uint4 *>(pp + sw128(j * 64 + i, cc)) =
            make_uint4(__float_as_uint(prow[4 * cc]), __float_as_uint(prow[4 * cc + 1]),
                       __float_as_uint(prow[4 * cc + 2]), __float_as_uint(prow[4 * cc + 3]));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // D_j[128 x 64] = [P_0 ; P_1] Ainv_j  (B = Ainv_j, MN-major: rows = K index),
  // reusing TMEM columns 64 j .. 64 j + 63.
  if (tid == 0) {
    const uint32_t idesc = umma_idesc_bf16(128, 64, false, true);
    const uint64_t dp = umma_desc_sw128(smem_u32(pp), 16, 1024);
    const uint64_t dai = umma_desc_sw128(smem_u32(ai), 8192, 1024);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + 64 * j, umma_desc_advance(dp, ks * 32),
                  umma_desc_advance(dai, j * 8192 + ks * 2048), idesc, ks > 0);
    }
    umma_commit(bar);
  }
  // Ainv halves -> rows 64..127 of the workspace images while the MMA runs.
  for (int idx = tid; idx < 2 * 512; idx += kPrepThreads) {
    const int j = idx >> 9, o = idx & 511;
    reinterpret_cast<uint4 *>(img0 + j * kM2Bytes + 8192)[o] =
        reinterpret_cast<const uint4 *>(ai + j * 8192)[o];
  }
  wait_phase(bar, 1, broken);
  tc_fence_after();
  {
    // warps 0,1: rows 0..63 of D_0 = P_0 Ainv_0; warps 2,3: rows 64..127 of
    // D_1 = P_1 Ainv_1.  Row i of P_j Ainv_j -> row i of image j.
    const int j = warp >> 1, i = (warp & 1) * 32 + lane;
    float acc[64];
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * warp) << 16) + 64 * j;
    tmem_ld32(trow, *reinterpret_cast<float(*)[32]>(acc));
    tmem_ld32(trow + 32, *reinterpret_cast<float(*)[32]>(acc + 32));
    tmem_wait_ld();
    uint8_t *img = img0 + j * kM2Bytes;
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
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kPrepTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 3. sequential inter-chunk scan
// ---------------------------------------------------------------------------
// One CTA per (sequence, v-head), 256 threads, two CTAs per SM.  The 128
// v-rows of the state sit on the 128 TMEM lanes: thread (quad q = warp % 4,
// lane l, half h = warp / 4) owns row v = 32 q + l and column half h of every
// [v x 64] tile (k-half h of the state, or token half h of a chunk).
//   S      fp32 S[v][k] in registers (64 k per thread)
//   TMEM   cols [0, 64)    bf16(S): A operand of MMA 1; then V_new, then
//                          bf16 V_dec (A operand of MMA 3)
//          cols [64, 128)  O: e^G Yq = S Q~^T (MMA 1), + bf16(V_new) P^T
//          cols [128, 256) Yk (MMA 1), then bf16 X (A operand of MMA 2) and
//                          bf16 V_new (A operand of the output MMA); then dS
// Every A operand is read from TMEM (the TS form); B operands (Q~ and K, the
// [P ; Ainv] image) are in shared memory.  Per chunk (t = token of the
// chunk, L valid tokens, G the within-chunk cumulative gate):
//   MMA 1   [e^G Yq | Yk] = S [Q~ ; K]^T, Q~ = e^G Q   M=128, N=128, K=128
//           X[v][t] = beta_t (V[t][v] - e^{G_t} Yk[v][t])
//   MMA 2   V_new = X Ainv^T                          M=128, N=64..16, K=64
//           V_dec[v][t] = e^{G_last - G_t} V_new[v][t]
//   output  O += bf16(V_new) P^T;  out[t][v] = scale O[v][t]
//   MMA 3   dS = V_dec K                               M=128, N=128,   K=64
//           S = e^{G_last} S + dS,  bf16(S) -> TMEM
// Thread 0 issues the MMAs; lane 0 of warp 1 the copies; warps 2 and 3 turn
// the gates into per-token factors.  Operands arrive by TMA (Q and K tiles,
// 128-byte swizzle, double buffered and loaded two chunks ahead, on one
// mbarrier per buffer; the V tile plain) and a bulk copy (the image), each
// issued as soon as its buffer is free.  Q~ of chunk c + 1 is formed in
// place while MMA 3 of chunk c runs, so that MMA 1 finds it ready.
constexpr int kScanThreads = 256;
constexpr int kCopyThread = 32;  // lane 0 of warp 1

template <bool kSave>
struct ScanSmemT {
  // Q and K tiles of a chunk, double buffered: [Q.d0 | K.d0 | Q.d1 | K.d1],
  // each 64 t rows x 128 B (64 bf16 of d), 128-byte swizzle.  Rows 0..63 of
  // [Q.db ; K.db] are the 128 N rows of MMA 1's B operand for d-block db.
  static constexpr int kQK0 = 0;
  static constexpr int kQK1 = 32768;
  // [P ; Ainv] image: the forward's compact 10 KiB; the backward's recompute
  // (no outputs) only the Ainv half of its [PA ; Ainv] image, 8 KiB
  static constexpr int kM2 = 65536;
  static constexpr int kM2Size = kSave ? 8192 : 10240;
  // V tile: 2 v-blocks x 64 t rows x 128 B, 128-byte swizzle (the MN-major
  // A operand of the V MMA)
  static constexpr int kV = kM2 + kM2Size;
  // bf16 output tile of a full chunk, [64 t][128 v] (256-byte rows), for one
  // TMA store (the forward only)
  static constexpr int kOst = kV + 16384;
  static constexpr int kOstSize = kSave ? 0 : 16384;
  // per-token gate factors of the current / next chunk, computed once per
  // chunk: e^{G_t}, beta_t, e^{G_last - G_t} (0 past the end), e^{G_last}
  // (three chunks' worth: the current one, and the next two, whose factors
  // are stored a chunk ahead so that Q~ of the next chunk can be formed at
  // the start of this one)
  static constexpr int kG = kOst + kOstSize;  // float eG[3][64]
  static constexpr int kB = kG + 768;  // float beta[3][64]
  static constexpr int kDec = kB + 768;  // float eDec[3][64]
  static constexpr int kEn = kDec + 768;  // float -eG[3][64] (the X phase's fused multiply-add)
  static constexpr int kGl = kEn + 768;  // float eGlast[3]
  // 16 x 16 bf16 identity, no-swizzle K-major (B operand of the V MMA)
  static constexpr int kI = kGl + 16;
  static constexpr int kBar = kI + 512;
  static constexpr int kBarMma = kBar, kBarV = kBar + 8, kBarM2 = kBar + 16,
                       kBarK0 = kBar + 24,  // K tile of buffer b: kBarK0 + 8 b
                       kBarQ0 = kBar + 40;  // Q tile of buffer b: kBarQ0 + 8 b
  static constexpr int kBarO = kBar + 56;   // the output MMA (O += bf16(V_new) P^T)
  static constexpr int kTmem = kBar + 64;
  static constexpr int kBroken = kBar + 68;
  static constexpr int kBytes = kBar + 72 + 1024;  // + base alignment slack
  static constexpr uint32_t kTmemCols = 256;
  // kColO: e^G Yq = S Q~^T (MMA 1), then + bf16(V_new) P^T (the output MMA):
  // scale * that is the output.  kColY: Yk (MMA 1, the 64 columns right after
  // kColO, as MMA 1's N = 128 result), then dS (MMA 3, 128 columns).
  static constexpr uint32_t kColSb = 0, kColO = 64, kColY = 128, kColYk = kColY;
  // bf16 operand images read from TMEM: X over the Yk columns (thread half
  // hc: columns kColX + 32 hc .. + 15, two tokens per column; MMA 2), then
  // bf16(V_new) in the same columns (the output MMA); V_new and then V_dec
  // (MMA 3) over the bf16(S) columns
  static constexpr uint32_t kColX = kColYk, kColVnb = kColX, kColVn = kColSb;
  // V[t][v] in fp32 (the V MMA), read by the X phase; free until MMA 3's dS
  static constexpr uint32_t kColV = 192;
};
using ScanSmem = ScanSmemT<false>;
// the epilogue stages one 64 KB (n, hv) state over the two Q/K tile buffers
static_assert(ScanSmem::kQK0 == 0 && ScanSmem::kQK1 + 32768 <= ScanSmem::kM2, "state staging region");
static_assert(ScanSmem::kColO + 64 == ScanSmem::kColYk, "MMA 1 writes [e^G Yq | Yk] in one pass");
static_assert(ScanSmem::kV % 1024 == 0 && ScanSmemT<true>::kV % 1024 == 0, "swizzled V tile alignment");
// two CTAs per SM: 228 KB per SM, 1 KB of it reserved per CTA
static_assert(2 * (ScanSmem::kBytes + 1024) <= 228 * 1024 &&
              2 * (ScanSmemT<true>::kBytes + 1024) <= 228 * 1024, "two CTAs per SM");

// kSave = true is the backward pass's recompute: FULL items only, no outputs
// and no final state; instead the state at the start of every chunk goes to
// save_states + ((global chunk) * 8 + hv) * kStateImgBytes as a bf16 operand
// image (put_state_img_row) and each chunk's delta (V_new, the v-vectors the
// WY system solves for; 0 past the sequence end) to save_delta +
// ((global chunk) * 8 + hv) * kTokImgBytes as a token image (put_tok_img).
template <bool kSave>
__global__ void __launch_bounds__(kScanThreads, 2)
gdn_prefill_scan_kernel(const __grid_constant__ CUtensorMap tmap_q,
                        const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v,
                        const __grid_constant__ CUtensorMap tmap_o, const float *h0,
                        const int64_t *__restrict__ cu, const int *__restrict__ meta,
                        const int *__restrict__ chunk_off,
                        const float *__restrict__ gcum_ws, const float *__restrict__ beta_ws,
                        const uint8_t *__restrict__ m2_ws, float scale,
                        uint16_t *__restrict__ out, float *final_state,
                        const int4 *__restrict__ items, int count_slot, int64_t seg_tokens,
                        const int *__restrict__ seg_off, float *seg_ss, float *seg_sb,
                        float *seg_phi, const int32_t *__restrict__ slots,
                        uint8_t *__restrict__ save_states, uint8_t *__restrict__ save_delta) {
  using SM = ScanSmemT<kSave>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  if (meta[1] != 0) return;
  const int item = blockIdx.x / kHV;
  if (item >= meta[count_slot]) return;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, hc = warp >> 2;
  const int vrow = 32 * quad + lane;  // state row (v) owned by this thread
  const int hv = blockIdx.x % kHV;
  const int hqk = hv >> 1;
  const int4 it = items[item];
  const int n = it.x, seg = it.y, mode = it.z;
  // this item's token range: segment `seg` of sequence n (the whole sequence
  // when not segmented: seg = 0 and seg_tokens exceeds any length)
  const int64_t seg_begin = static_cast<int64_t>(seg) * seg_tokens;
  const int64_t bos = cu[n] + seg_begin;
  const int64_t len = lmin(cu[n + 1] - bos, seg_tokens);
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);
  const int gbase = chunk_off[n] + static_cast<int>(seg_begin / kChunk);
  GDN_DCHECK(n >= 0 && n < meta[kMetaN] && mode >= kItemFull && mode <= kItemTail);
  GDN_DCHECK(len >= 0 && bos + len <= meta[kMetaT]);
  GDN_DCHECK(gbase >= 0 && gbase + nchunks <= chunk_off[n + 1] && chunk_off[n + 1] <= meta[kMetaChunks]);
  GDN_DCHECK(mode == kItemFull || (seg_off != nullptr && seg_off[n] + seg < seg_off[n + 1]));
  const bool ident = mode == kItemIdent;
  const bool write_out = mode == kItemFull || mode == kItemHead || mode == kItemMid ||
                         mode == kItemTail;
  // where the state starts from and where the final state goes
  const int64_t srow = static_cast<int64_t>(vrow) * kD + 64 * hc;  // within one (., hv) state
  const int64_t hv_off = static_cast<int64_t>(hv) * kD * kD;
  auto seg_state = [&](float *buf, int p) {
    return buf + (static_cast<int64_t>(seg_off[n] + p) * kHV) * kD * kD + hv_off;
  };
  // initial / final state of sequence n: dense (index n) or a state-pool slot
  const int64_t sidx = slots != nullptr ? static_cast<int64_t>(slots[n]) : n;
  const float *init = nullptr;
  if (mode == kItemFull || mode == kItemHead)
    init = h0 != nullptr ? h0 + sidx * kHV * kD * kD + hv_off : nullptr;
  else if (mode == kItemMid || mode == kItemTail)
    init = seg_state(seg_ss, seg);
  float *fin = nullptr;
  if (kSave)
    fin = nullptr;
  else if (mode == kItemFull || mode == kItemTail)
    fin = final_state + sidx * kHV * kD * kD + hv_off;
  else if (mode == kItemHead)
    fin = seg_state(seg_ss, 1);
  else if (mode == kItemZero)
    fin = seg_state(seg_sb, seg);
  else if (mode == kItemIdent)
    fin = seg_state(seg_phi, seg);

  float *Eg = reinterpret_cast<float *>(smem + SM::kG);
  float *Bs = reinterpret_cast<float *>(smem + SM::kB);
  float *Ed = reinterpret_cast<float *>(smem + SM::kDec);
  float *En = reinterpret_cast<float *>(smem + SM::kEn);
  float *Egl = reinterpret_cast<float *>(smem + SM::kGl);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + SM::kBroken);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_mma = s_base + SM::kBarMma, bar_v = s_base + SM::kBarV,
                 bar_m2 = s_base + SM::kBarM2, bar_k0 = s_base + SM::kBarK0,
                 bar_q0 = s_base + SM::kBarQ0, bar_o = s_base + SM::kBarO;

  // Items without outputs (ZERO, IDENT) need neither Q nor the Q-side MMAs;
  // IDENT treats V as zero and needs no V either.
  const bool need_q = write_out && !kSave;
  const bool need_v = !ident;

  // Chunk operand loads: the first ones by thread 0 at the start, then each
  // next one by lane 0 of warp 1 (kCopyThread) as soon as its buffer is free,
  // so that thread 0, which issues every MMA, has no copies to issue.  Each
  // barrier still has one re-arming thread, and only the waits that happen
  // before its re-arm poll it.
  // The Q (where outputs are formed) or the K tile of chunk c into tile
  // buffer b, each on its own barrier: a buffer's Q half is free once MMA 1
  // has run, its K half only after MMA 3.
  auto issue_tile = [&](bool is_k, int c, int b) {
    const int y = static_cast<int>(bos + static_cast<int64_t>(c) * kChunk);
    const uint32_t dst = s_base + (b ? SM::kQK1 : SM::kQK0) + (is_k ? 8192 : 0);
    const uint32_t bar = (is_k ? bar_k0 : bar_q0) + 8 * b;
    const void *tm = is_k ? static_cast<const void *>(&tmap_k) : static_cast<const void *>(&tmap_q);
    mbar_arrive_expect_tx(bar, 16384u);
    tma_load_2d(dst, tm, hqk * kD, y, bar);
    tma_load_2d(dst + 16384, tm, hqk * kD + 64, y, bar);
  };
  auto issue_v = [&](int c) {
    const int y = static_cast<int>(bos + static_cast<int64_t>(c) * kChunk);
    mbar_arrive_expect_tx(bar_v, 16384);
    tma_load_2d(s_base + SM::kV, &tmap_v, hv * kD, y, bar_v);
    tma_load_2d(s_base + SM::kV + 8192, &tmap_v, hv * kD + 64, y, bar_v);
  };
  // the forward reads the compact [P ; Ainv] image; the backward's recompute,
  // which forms no outputs, only the Ainv half (its second 8 KiB) of the
  // [PA ; Ainv] image that the reverse scan reads whole
  constexpr uint32_t kImgStride = static_cast<uint32_t>(kSave ? kM2Bytes : kImgFwdBytes);
  constexpr uint32_t kImgOff = kSave ? 8192u : 0u;
  constexpr uint32_t kImgLoad = kSave ? 8192u : static_cast<uint32_t>(kImgFwdBytes);
  auto issue_m2 = [&](int c) {
    mbar_arrive_expect_tx(bar_m2, kImgLoad);
    bulk_load(s_base + SM::kM2,
              m2_ws + (static_cast<int64_t>(gbase + c) * kHV + hv) * kImgStride + kImgOff,
              kImgLoad, bar_m2);
  };
  // Gates of chunk c for token gt = tid - 64 (threads 64..127, warps 2 and 3:
  // thread 0, which issues the MMAs and copies, has no part in them): fetched
  // into registers a chunk ahead, turned into the per-token factors when the
  // buffer is free.
  const int gt = tid - 64;
  const bool gate_thread = static_cast<unsigned>(gt) < 64u;
  struct GateRegs {
    float g, g_last, beta;
    bool valid;
  };
  // Only predicated loads here (no use of the loaded values), so the thread
  // does not wait for them until store_gates, a chunk later.
  auto fetch_gates = [&](int c) {
    const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk));
    GateRegs r;
    r.valid = gt < L;
    r.g_last = gcum_ws[(t0 + L - 1) * kHV + hv];
    r.g = 0.f;
    r.beta = 0.f;
    if (r.valid) {
      r.g = gcum_ws[(t0 + gt) * kHV + hv];
      r.beta = beta_ws[(t0 + gt) * kHV + hv];
    }
    return r;
  };
  auto store_gates = [&](const GateRegs &r, int buf) {
    const float g = r.valid ? r.g : r.g_last;
    const float eg = expf(g);
    Eg[buf * 64 + gt] = eg;
    En[buf * 64 + gt] = -eg;
    Bs[buf * 64 + gt] = r.beta;
    Ed[buf * 64 + gt] = r.valid ? expf(r.g_last - g) : 0.f;
    if (gt == 0) Egl[buf] = expf(r.g_last);
  };
  // Q~ = e^{G_t} Q in place in tile buffer b with the factors of gate buffer
  // gb: row t of both d-blocks times e^{G_t}, the tile's 1,024 16-byte pieces
  // spread over nt threads (this one is number ti; a piece lies in one row,
  // the swizzle only permutes pieces within a row), on packed pairs.  The
  // caller waits for the tile first and fences (async proxy) and
  // synchronises before MMA 1 reads it.
  auto scale_q = [&](int b, int gb, int ti, int nt) {
    uint8_t *qt = smem + (b ? SM::kQK1 : SM::kQK0);
#pragma unroll
    for (int m = 0; m < 5; ++m) {  // nt >= 224 threads: at most 5 pieces each
      const int piece = ti + nt * m;
      if (piece >= 1024) break;
      const int db = piece >> 9, t = (piece >> 3) & 63;
      uint4 *ptr = reinterpret_cast<uint4 *>(qt + db * 16384 + t * 128 + (piece & 7) * 16);
      const uint4 w = *ptr;
      const float e = Eg[gb * 64 + t];
      const uint64_t ee = f2_pack(e, e);
      const uint32_t in[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t r = f2_mul(f2_pack(bf16_lo(in[h]), bf16_hi(in[h])), ee);
        o[h] = pack_bf16x2(f2_lo(r), f2_hi(r));
      }
      *ptr = make_uint4(o[0], o[1], o[2], o[3]);
    }
  };

  // Barriers first, then the first chunk's operand loads and gates, so their
  // latency overlaps the initial-state load below.
  if (warp == 0) tmem_alloc(s_base + SM::kTmem, SM::kTmemCols);
  if (tid == 0) {
    *broken = 0;
    for (int i = 0; i < 8; ++i) mbar_init(bar_mma + 8 * i, 1);  // mma, v, m2, k0/1, q0/1, o
    mbar_init_fence();
    if (nchunks > 0) {
      if (need_q) issue_tile(false, 0, 0);
      issue_tile(true, 0, 0);
      if (nchunks > 1) {
        if (need_q) issue_tile(false, 1, 1);
        issue_tile(true, 1, 1);
      }
      if (need_v) issue_v(0);
      issue_m2(0);
    }
  }
  GateRegs gates0, gates1;
  if (gate_thread && nchunks > 0) gates0 = fetch_gates(0);
  if (gate_thread && nchunks > 1) gates1 = fetch_gates(1);

  // fp32 state row slice S[v][64 hc .. 64 hc + 63].
  float s[64];
  if (init != nullptr) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 x = *reinterpret_cast<const float4 *>(init + srow + 4 * i);
      s[4 * i] = x.x;
      s[4 * i + 1] = x.y;
      s[4 * i + 2] = x.z;
      s[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) s[i] = (ident && vrow == 64 * hc + i) ? 1.f : 0.f;
  }
  if (tid < 32) {
    // the 16 x 16 identity: row r, K half kh (columns 8 kh .. 8 kh + 7) is
    // the core-matrix row at (r / 8) * 256 + kh * 128 + (r % 8) * 16
    const int r = tid >> 1, kh = tid & 1, wi = (r >> 3) == kh ? (r & 7) >> 1 : -1;
    const uint32_t one = (r & 1) ? 0x3F800000u : 0x00003F80u;  // bf16 1.0 in word wi
    *reinterpret_cast<uint4 *>(smem + SM::kI + (r >> 3) * 256 + kh * 128 + (r & 7) * 16) =
        make_uint4(wi == 0 ? one : 0u, wi == 1 ? one : 0u, wi == 2 ? one : 0u, wi == 3 ? one : 0u);
    fence_async_smem();
  }
  __syncthreads();  // barriers initialised, TMEM address published, identity written
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + SM::kTmem);
  const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * quad) << 16);
  {
    uint32_t pk[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pk[j] = pack_bf16x2(s[2 * j], s[2 * j + 1]);
    tmem_st32(tlane + SM::kColSb + 32 * hc, pk);
  }
  if (gate_thread && nchunks > 0) store_gates(gates0, 0);
  if (gate_thread && nchunks > 1) store_gates(gates1, 1);
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Q~ of the first chunk (every later one is formed a chunk ahead)
  uint32_t ph_q = 0;  // bit b = parity of Q barrier b
  if (need_q && nchunks > 0) {
    wait_phase(bar_q0, 0, broken);
    ph_q ^= 1u;
    scale_q(0, 0, tid, kScanThreads);
    fence_async_smem();
    __syncthreads();
  }

  const uint32_t idesc_n64 = umma_idesc_bf16(128, 64, false, false);
  const uint32_t idesc_n128 = umma_idesc_bf16(128, 128, false, false);
  const uint32_t idesc_v = umma_idesc_bf16(128, 16, true, false);  // A MN-major
  const uint32_t idesc_ds = umma_idesc_bf16(128, 128, false, true);
  uint32_t ph_mma = 0, ph_v = 0, ph_m2 = 0, ph_o = 0;
  uint32_t ph_k = 0;  // bit b = parity of tile buffer b

  // The chunk loop, instantiated twice: with outputs (FULL, HEAD, MID, TAIL)
  // and state only (ZERO, IDENT).  Compile-time flags keep the loop free of
  // per-chunk mode branches.
  auto chunk_loop = [&](auto out_tag) {
    constexpr bool kOut = decltype(out_tag)::value;
    for (int c = 0; c < nchunks; ++c) {
      const int cb = c & 1, gs = c % 3;
      const int64_t t0 = bos + static_cast<int64_t>(c) * kChunk;
      const int L = static_cast<int>(lmin(kChunk, len - static_cast<int64_t>(c) * kChunk));
      const uint32_t kbuf = s_base + (cb ? SM::kQK1 : SM::kQK0);
      const uint32_t bar_k = bar_k0 + 8 * cb;
      // gate buffers rotate over three chunks: gs (this chunk), gs1 (next),
      // gs2 (the one after, fetched now and stored before the V barrier)
      const int gs1 = gs == 2 ? 0 : gs + 1, gs2 = gs1 == 2 ? 0 : gs1 + 1;
      GateRegs next_gates;
      if (gate_thread && c + 2 < nchunks) next_gates = fetch_gates(c + 2);
      if constexpr (kSave)
        put_state_img_row(save_states + (static_cast<int64_t>(gbase + c) * kHV + hv) * kStateImgBytes,
                          vrow, hc, s);

      // The tiles and the image are read only by the tensor core, so only the
      // MMA thread waits for them here: the copy thread re-arms each barrier
      // for a later chunk right after the MMA that consumed it, and a thread
      // still polling the old phase could otherwise see two completions and
      // wait forever.  (Every thread already waited for this buffer's tiles
      // before forming Q~, a chunk earlier, long before that re-arm.)  The
      // tail chunk (always the last, so never re-armed) is the exception:
      // every thread must see its tiles landed before zeroing rows.
      const bool tail = L < kChunk;
      if (tid == 0 || tail) wait_phase(bar_k, (ph_k >> cb) & 1, broken);
      if (tail && (kOut || need_v)) wait_phase(bar_v, ph_v, broken);
      ph_k ^= 1u << cb;
      if (tail) {
        // tail chunk: zero the rows past the sequence end (TMA brought in the
        // next sequence's tokens there; Q~ rows included), and the V rows, so
        // that nothing of the next sequence reaches this one's state (a row
        // of the swizzled tiles keeps its 8 pieces: zero them all)
        for (int idx = tid; idx < 2 * 2 * (kChunk - L) * 8; idx += kScanThreads) {
          const int ch = idx & 7, r = L + ((idx >> 3) % (kChunk - L)), blk = (idx >> 3) / (kChunk - L);
          const int which = blk >> 1, dblk = blk & 1;  // which: 0 Q, 1 K
          *reinterpret_cast<uint4 *>(smem + (cb ? SM::kQK1 : SM::kQK0) + dblk * 16384 + which * 8192 +
                                     r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
        }
        if (kOut || need_v) {
          for (int idx = tid; idx < 2 * (kChunk - L) * 8; idx += kScanThreads) {
            const int ch = idx & 7, r = L + ((idx >> 3) % (kChunk - L)), vb = (idx >> 3) / (kChunk - L);
            *reinterpret_cast<uint4 *>(smem + SM::kV + vb * 8192 + r * 128 + ch * 16) =
                make_uint4(0, 0, 0, 0);
          }
        }
        fence_async_smem();
        __syncthreads();
      }

      // ---- MMA 1: [e^G Yq | Yk] = S [Q~ ; K]^T with outputs (B = the two
      // 64-row tiles of d-block db, adjacent: N = 128), Yk = S K^T without ----
      if (tid == 0) {
        tc_fence_after();
        if constexpr (kOut) {
          const uint64_t dqk = umma_desc_sw128(kbuf, 16, 1024);
  #pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t boff = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma_bf16_ts(tmem + SM::kColO, tmem + SM::kColSb + 8 * ks, umma_desc_advance(dqk, boff),
                         idesc_n128, ks > 0);
          }
        } else {
          const uint64_t dk = umma_desc_sw128(kbuf + 8192, 16, 1024);
  #pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t boff = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma_bf16_ts(tmem + SM::kColYk, tmem + SM::kColSb + 8 * ks, umma_desc_advance(dk, boff),
                         idesc_n64, ks > 0);
          }
        }
        if (kOut || need_v) {
          // ---- V MMA: V[t][v] in fp32 (exact) into kColV, for the X phase:
          // A = the V tile (MN-major, v = M), B = the 16 x 16 identity;
          // K-step ks gives tokens 16 ks .. 16 ks + 15 (N = 16) ----
          wait_phase(bar_v, ph_v, broken);
          tc_fence_after();
          const uint64_t dv = umma_desc_sw128(s_base + SM::kV, 8192, 1024);
          const uint64_t di = umma_desc_noswz(s_base + SM::kI, 128, 256);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + SM::kColV + 16 * ks, umma_desc_advance(dv, ks * 2048), di, idesc_v, 0);
        }
        umma_commit(bar_mma);
      }
      if constexpr (kOut) {
        // ---- Q~ of the next chunk, in the other tile buffer, by warps 1..7
        // while thread 0 issues MMA 1 (the factors were stored a chunk ago;
        // the X barrier below orders the writes before MMA 1 of the next
        // chunk) ----
        if (c + 1 < nchunks) {
          if (warp != 0) {
            wait_phase(bar_q0 + 8 * (cb ^ 1), (ph_q >> (cb ^ 1)) & 1, broken);
            scale_q(cb ^ 1, gs1, tid - 32, kScanThreads - 32);
            fence_async_smem();
          }
          ph_q ^= 1u << (cb ^ 1);
        }
      }
      wait_phase(bar_mma, ph_mma, broken);
      ph_mma ^= 1;
      tc_fence_after();
      // MMA 1 has read Q~ of this chunk: the Q tile two chunks ahead can come
      if (kOut && tid == kCopyThread && c + 2 < nchunks) issue_tile(false, c + 2, cb);
      if (kOut || need_v) ph_v ^= 1;

      // ---- X = beta (V - e^G Yk) -> TMEM ----
  #pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int tb = 32 * hc + 16 * p;
        float yk[16], vv[16];
        tmem_ld16(tlane + SM::kColYk + tb, yk);
        if (kOut || need_v) {
          tmem_ld16(tlane + SM::kColV + tb, vv);
        } else {
  #pragma unroll
          for (int j = 0; j < 16; ++j) vv[j] = 0.f;  // IDENT: V is zero
        }
        tmem_wait_ld();
  #pragma unroll
        for (int g = 0; g < 4; ++g) {
          // packed pairs (f32x2): x = beta * fma(-e^G, y, v), as the scalar
          // form; past the sequence end beta = 0 (and the V rows are zero)
          const float4 en4 = *reinterpret_cast<const float4 *>(En + gs * 64 + tb + 4 * g);
          const float4 bt4 = *reinterpret_cast<const float4 *>(Bs + gs * 64 + tb + 4 * g);
          const uint64_t en2[2] = {f2_pack(en4.x, en4.y), f2_pack(en4.z, en4.w)};
          const uint64_t bt2[2] = {f2_pack(bt4.x, bt4.y), f2_pack(bt4.z, bt4.w)};
  #pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int j = 4 * g + 2 * h;
            const uint64_t x =
                f2_mul(bt2[h], f2_fma(en2[h], f2_pack(yk[j], yk[j + 1]), f2_pack(vv[j], vv[j + 1])));
            yk[j] = f2_lo(x);
            yk[j + 1] = f2_hi(x);
          }
        }
        // bf16 X into the Yk columns this thread has read (MMA 2's A operand)
        uint32_t pk[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) pk[j] = pack_bf16x2(yk[2 * j], yk[2 * j + 1]);
        tmem_st8(tlane + SM::kColX + 32 * hc + 8 * p, pk);
      }
      // the previous chunk's output store has read its tile before this
      // barrier, so the output phase below may overwrite it
      if constexpr (kOut) {
        if (tid == kCopyThread) bulk_wait_read_all();
      }
      tmem_wait_st();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == kCopyThread && (kOut || need_v) && c + 1 < nchunks) issue_v(c + 1);

      // ---- MMA 2: V_new = X Ainv^T ----
      const uint32_t m2buf = s_base + SM::kM2;
      if (tid == 0) {
        wait_phase(bar_m2, ph_m2, broken);
        tc_fence_after();
        if constexpr (kSave) {
          const uint64_t da = umma_desc_sw128(m2buf, 16, 1024);  // Ainv (swizzled, 1024-aligned)
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_ts(tmem + SM::kColVn, tmem + SM::kColX + 32 * (ks >> 1) + 8 * (ks & 1),
                         umma_desc_advance(da, ks * 32), idesc_n64, ks > 0);
        } else {
          // K-step ks only reaches tokens t >= 16 ks (N = 64 - 16 ks)
          const uint64_t da = umma_desc_noswz(m2buf + kTriBytes, kTriLbo, kTriSbo);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_ts(tmem + SM::kColVn + 16 * ks,
                         tmem + SM::kColX + 32 * (ks >> 1) + 8 * (ks & 1),
                         umma_desc_advance(da, tri_step_off(ks)),
                         umma_idesc_bf16(128, 64 - 16 * ks, false, false), ks > 0);
        }
        umma_commit(bar_mma);
      }
      ph_m2 ^= 1;
      wait_phase(bar_mma, ph_mma, broken);
      ph_mma ^= 1;
      tc_fence_after();
      // the output MMA still reads this chunk's P rows: with outputs the next
      // image is issued once that MMA has completed
      if (!kOut && tid == kCopyThread && c + 1 < nchunks) issue_m2(c + 1);

      // ---- V_dec (the outputs wait until MMA 3 runs) ----
  #pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int tb = 32 * hc + 16 * p;
        float zv[16];
        tmem_ld16(tlane + SM::kColVn + tb, zv);
        tmem_wait_ld();
        if constexpr (kSave) {
          // thread (vrow, hc) holds V_new[vrow][tb .. tb+15]; a warp's store
          // for one token covers 32 consecutive v (64 B)
          uint8_t *img = save_delta + (static_cast<int64_t>(gbase + c) * kHV + hv) * kTokImgBytes;
#pragma unroll
          for (int j = 0; j < 16; ++j) put_tok_img(img, tb + j, vrow, tb + j < L ? zv[j] : 0.f);
        }
        // V_dec = e^{G_last - G_t} V_new (0 past the end), on packed pairs, then
        // bf16 into the V_new columns this thread has read (MMA 3's A operand)
        uint32_t pk[8];
        if constexpr (kOut) {
          // bf16(V_new) into the X columns (MMA 2 has read them): the output
          // MMA's A operand
  #pragma unroll
          for (int j = 0; j < 8; ++j) pk[j] = pack_bf16x2(zv[2 * j], zv[2 * j + 1]);
          tmem_st8(tlane + SM::kColVnb + 32 * hc + 8 * p, pk);
        }
  #pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float4 ed4 = *reinterpret_cast<const float4 *>(Ed + gs * 64 + tb + 4 * g);
          const uint64_t a = f2_mul(f2_pack(zv[4 * g], zv[4 * g + 1]), f2_pack(ed4.x, ed4.y));
          const uint64_t b = f2_mul(f2_pack(zv[4 * g + 2], zv[4 * g + 3]), f2_pack(ed4.z, ed4.w));
          pk[2 * g] = pack_bf16x2(f2_lo(a), f2_hi(a));
          pk[2 * g + 1] = pack_bf16x2(f2_lo(b), f2_hi(b));
        }
        tmem_st8(tlane + SM::kColVn + 32 * hc + 8 * p, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();

      // ---- output MMA: O += bf16(V_new) P^T (onto e^G Yq; before MMA 3, which
      // overwrites its A operand), then MMA 3: dS = V_dec K ----
      if (tid == 0) {
        if constexpr (kOut) {
          const uint64_t dp = umma_desc_noswz(m2buf, kTriLbo, kTriSbo);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_ts(tmem + SM::kColO + 16 * ks,
                         tmem + SM::kColVnb + 32 * (ks >> 1) + 8 * (ks & 1),
                         umma_desc_advance(dp, tri_step_off(ks)),
                         umma_idesc_bf16(128, 64 - 16 * ks, false, false), 1);
          umma_commit(bar_o);
        }
        // B = K MN-major (rows = K index t): the two 64-wide k blocks K.d0,
        // K.d1 are 16 KB apart
        const uint64_t dkm = umma_desc_sw128(kbuf + 8192, 16384, 1024);
  #pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16_ts(tmem + SM::kColY, tmem + SM::kColVn + 32 * (ks >> 1) + 8 * (ks & 1),
                       umma_desc_advance(dkm, ks * 2048), idesc_ds, ks > 0);
        umma_commit(bar_mma);
      }
      if constexpr (kOut) {
        // ---- outputs O = scale (e^G Yq + bf16(V_new) P^T), while MMA 3 runs
        // (it writes columns kColY.., these are kColO..); then this chunk's
        // image is no longer read and the next one can come in ----
        wait_phase(bar_o, ph_o, broken);
        ph_o ^= 1;
        tc_fence_after();
        if (tid == kCopyThread && c + 1 < nchunks) issue_m2(c + 1);
        // Lanes 2m and 2m + 1 (rows v, v + 1) swap one value per token pair
        // so that each stores a bf16 pair of adjacent v: the even lane token
        // t, the odd lane token t + 1 -- half the store instructions.
        const uint64_t sc2 = f2_pack(scale, scale);
        if (L == kChunk) {
          // a full chunk: the bf16 tile [t][v] in shared memory (a warp's
          // stores for one token cover 64 contiguous bytes), sent by one TMA
          // store after the barrier that ends the chunk
          uint16_t *ost = reinterpret_cast<uint16_t *>(smem + SM::kOst) + vrow;
  #pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int tb = 32 * hc + 16 * p;
            float zo[16];
            tmem_ld16(tlane + SM::kColO + tb, zo);
            tmem_wait_ld();
  #pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const uint64_t o = f2_mul(sc2, f2_pack(zo[j], zo[j + 1]));
              ost[(tb + j) * kD] = __bfloat16_as_ushort(__float2bfloat16_rn(f2_lo(o)));
              ost[(tb + j + 1) * kD] = __bfloat16_as_ushort(__float2bfloat16_rn(f2_hi(o)));
            }
          }
          fence_async_smem();
        } else {
          // the tail chunk: direct stores of the first L tokens only
          const bool odd = lane & 1;
          uint32_t *orow = reinterpret_cast<uint32_t *>(
              out + ((t0 + 32 * hc + (odd ? 1 : 0)) * kHV + hv) * kD + (vrow & ~1));
  #pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int tb = 32 * hc + 16 * p;
            float zo[16];
            tmem_ld16(tlane + SM::kColO + tb, zo);
            tmem_wait_ld();
  #pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const uint64_t o = f2_mul(sc2, f2_pack(zo[j], zo[j + 1]));
              const float oe = f2_lo(o), oo = f2_hi(o);  // tokens tb + j, tb + j + 1
              const float got = __shfl_xor_sync(0xffffffffu, odd ? oe : oo, 1);
              const uint32_t pair = odd ? pack_bf16x2(got, oo) : pack_bf16x2(oe, got);
              if (tb + j + (odd ? 1 : 0) < L) orow[(16 * p + j) * (kHV * kD / 2)] = pair;
            }
          }
        }
        // the gate factors of chunk c + 2, while MMA 3 runs (their buffer's
        // last reader was the previous chunk; the barrier ending this chunk
        // makes them visible before Q~ of chunk c + 2 is formed)
        if (gate_thread && c + 2 < nchunks) store_gates(next_gates, gs2);
      } else {
        if (gate_thread && c + 2 < nchunks) store_gates(next_gates, gs2);
      }
      wait_phase(bar_mma, ph_mma, broken);
      ph_mma ^= 1;
      tc_fence_after();
      // MMA 3 is done with this chunk's K tile
      if (tid == kCopyThread && c + 2 < nchunks) issue_tile(true, c + 2, cb);

      // ---- S = e^{G_last} S + dS ;  bf16(S) -> TMEM ----
      {
        const float eg_last = Egl[gs];
  #pragma unroll
        for (int p = 0; p < 2; ++p) {
          float ds[32];
          tmem_ld32(tlane + SM::kColY + 64 * hc + 32 * p, ds);
          tmem_wait_ld();
          const uint64_t gl2 = f2_pack(eg_last, eg_last);
  #pragma unroll
          for (int j = 0; j < 32; j += 2) {  // e^{G_last} S + dS on packed pairs
            const uint64_t x =
                f2_fma(gl2, f2_pack(s[32 * p + j], s[32 * p + j + 1]), f2_pack(ds[j], ds[j + 1]));
            s[32 * p + j] = f2_lo(x);
            s[32 * p + j + 1] = f2_hi(x);
          }
        }
        uint32_t pk[32];
  #pragma unroll
        for (int j = 0; j < 32; ++j) pk[j] = pack_bf16x2(s[2 * j], s[2 * j + 1]);
        tmem_st32(tlane + SM::kColSb + 32 * hc, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      // every thread's part of a full chunk's output tile is written (and
      // fenced for the async proxy): one TMA store (x = v-head column,
      // 256-byte aligned; y = the chunk's first token)
      if constexpr (kOut) {
        if (L == kChunk && tid == kCopyThread) {
          tma_store_2d(&tmap_o, hv * kD, static_cast<int>(t0), s_base + SM::kOst);
          bulk_commit_group();
        }
      }
    }
  };
  // (the recompute has no outputs: its kernel has no output loop at all)
  if constexpr (!kSave) {
    if (write_out)
      chunk_loop(std::true_type{});
    else
      chunk_loop(std::false_type{});
  } else {
    chunk_loop(std::false_type{});
  }

  if (fin != nullptr) {
    // The (n, hv) state is one contiguous 64 KB block.  It goes out through
    // shared memory so that each warp store covers 512 contiguous bytes (one
    // state row) rather than 16 bytes of 32 rows: the same bytes, but whole
    // lines, which is what matters when `fin` is another GPU's memory and
    // every store crosses NVLink as its own request.  The two Q/K tile
    // buffers (first 64 KB) are free: every MMA and TMA load has completed.  Chunk c
    // of row r is kept at c ^ (r & 7), conflict-free on both sides.
    float4 *stage = reinterpret_cast<float4 *>(smem + SM::kQK0);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = 16 * hc + i;
      stage[vrow * 32 + (c ^ (vrow & 7))] =
          make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
    }
    __syncthreads();
    float4 *dst = reinterpret_cast<float4 *>(fin);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = kScanThreads * i + tid, r = j >> 5, c = j & 31;
      dst[j] = stage[r * 32 + (c ^ (r & 7))];
    }
  }

  if (tid == kCopyThread) bulk_wait_all();  // the last output store has completed
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, SM::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 4. segment composition (segmented mode only)
// ---------------------------------------------------------------------------
// S_start(p+1) = S_start(p) Phi(p) + B(p) for p = 1 .. P-2, in fp32.  Rows of
// S are independent, so one CTA per (sequence, v-head, 8-row block); Phi(p)
// (64 KiB) arrives by one bulk copy, double buffered one segment ahead, and
// B(p+1) is read into registers during step p; the 8 rows of S_start(p)
// stay in shared memory (double buffered) between steps, so a step needs one
// CTA barrier.  Thread (col, rh) produces S[r0 + 4 rh + i][col] for i < 4;
// the fully unrolled k loop lets the loads run ahead of the FMAs.
constexpr int kComposeThreads = 256;
constexpr int kComposeRows = 8;
constexpr int kCmpPhi = 0;                                   // 2 x 64 KiB
constexpr int kCmpX = 2 * 65536;                             // 2 x (8 x 128 fp32)
constexpr int kCmpXBytes = kComposeRows * kD * 4;
constexpr int kCmpBar = kCmpX + 2 * kCmpXBytes;
constexpr int kCmpBroken = kCmpBar + 16;
constexpr int kCmpSmem = kCmpBroken + 16 + 128;  // + base alignment slack

__global__ void __launch_bounds__(kComposeThreads, 1)
gdn_prefill_compose_kernel(const int *__restrict__ meta, const int *__restrict__ seg_off,
                           float *seg_ss, const float *__restrict__ seg_sb,
                           const float *__restrict__ seg_phi) {
  if (meta[1] != 0) return;
  const int n = blockIdx.x, hv = blockIdx.y, r0 = blockIdx.z * kComposeRows;
  const int P = seg_off[n + 1] - seg_off[n];
  if (P < 3) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<128>(smem_raw);
  volatile int *broken = reinterpret_cast<volatile int *>(smem + kCmpBroken);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar0 = s_base + kCmpBar;
  const int tid = threadIdx.x, col = tid & 127, rh = tid >> 7;
  const int64_t per_seg = static_cast<int64_t>(kHV) * kD * kD;
  const int64_t base = static_cast<int64_t>(seg_off[n]) * per_seg + static_cast<int64_t>(hv) * kD * kD;
  const int64_t my_rows = static_cast<int64_t>(r0 + 4 * rh) * kD + col;

  if (tid == 0) {
    *broken = 0;
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    mbar_init_fence();
  }
  {
    const float4 *src = reinterpret_cast<const float4 *>(seg_ss + base + per_seg + r0 * kD);
    float4 *dst = reinterpret_cast<float4 *>(smem + kCmpX);
    for (int i = tid; i < kComposeRows * kD / 4; i += kComposeThreads) dst[i] = src[i];
  }
  float bnext[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) bnext[i] = seg_sb[base + per_seg + my_rows + i * kD];
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar0, 65536);
    bulk_load(s_base + kCmpPhi, seg_phi + base + per_seg, 65536, bar0);
  }
  uint32_t ph0 = 0, ph1 = 0;
  for (int p = 1; p + 1 < P; ++p) {
    const int b = (p - 1) & 1;
    // the other Phi buffer was last read in step p-1, which every thread has left
    if (tid == 0 && p + 2 < P) {
      mbar_arrive_expect_tx(bar0 + 8 * (b ^ 1), 65536);
      bulk_load(s_base + kCmpPhi + 65536 * (b ^ 1), seg_phi + base + (p + 1) * per_seg, 65536,
                bar0 + 8 * (b ^ 1));
    }
    float acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = bnext[i];
    if (p + 2 < P) {
#pragma unroll
      for (int i = 0; i < 4; ++i) bnext[i] = seg_sb[base + (p + 1) * per_seg + my_rows + i * kD];
    }
    if (b == 0) {
      wait_phase(bar0, ph0, broken);
      ph0 ^= 1;
    } else {
      wait_phase(bar0 + 8, ph1, broken);
      ph1 ^= 1;
    }
    const float *Phi = reinterpret_cast<const float *>(smem + kCmpPhi + 65536 * b) + col;
    const float4 *X4 =
        reinterpret_cast<const float4 *>(smem + kCmpX + kCmpXBytes * b) + (4 * rh) * (kD / 4);
#pragma unroll 4
    for (int kk = 0; kk < kD; kk += 4) {
      const float f0 = Phi[(kk + 0) * kD], f1 = Phi[(kk + 1) * kD], f2 = Phi[(kk + 2) * kD],
                  f3 = Phi[(kk + 3) * kD];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 x = X4[i * (kD / 4) + kk / 4];
        acc[i] = fmaf(x.x, f0, acc[i]);
        acc[i] = fmaf(x.y, f1, acc[i]);
        acc[i] = fmaf(x.z, f2, acc[i]);
        acc[i] = fmaf(x.w, f3, acc[i]);
      }
    }
    // next step reads the other X buffer, whose last readers (step p-1) are done
    float *xo = reinterpret_cast<float *>(smem + kCmpX + kCmpXBytes * (b ^ 1)) + (4 * rh) * kD + col;
    float *dst = seg_ss + base + (p + 1) * per_seg + my_rows;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xo[i * kD] = acc[i];
      dst[i * kD] = acc[i];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
size_t prefill_workspace_bytes(int64_t T, int64_t N, bool allow_segments) {
  return prefill_ws_layout(T, N, allow_segments).total;
}

int prefill_kernel_launches(int64_t T, int64_t N, bool allow_segments) {
  if (N == 0) return 0;
  const PrefillWs w = prefill_ws_layout(T, N, allow_segments);
  return (w.nt_max > 0 ? 3 : 2) + (w.seg_chunks ? 2 : 0);
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D bf16 tensor map over a [rows, row_elems] row-major tensor.
static bool make_tmap_2d(CUtensorMap *m, const void *base, uint64_t row_elems, uint64_t rows,
                         uint32_t box_x, uint32_t box_y, bool swizzle128) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {row_elems, rows};
  const cuuint64_t strides[1] = {row_elems * 2};
  const cuuint32_t box[2] = {box_x, box_y};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_prefill(const void *q, const void *k, const void *v, const float *state,
                           const float *A_log, const void *a, const float *dt_bias, const void *b,
                           const int64_t *cu_seqlens, int64_t N, int64_t T, float scale,
                           void *out, float *final_state, void *workspace, bool allow_segments,
                           const int32_t *slots, int64_t pool_slots, cudaStream_t stream,
                           const cudaEvent_t *events, int num_events) {
  if (N == 0) return cudaSuccess;
  // events[i] (when given) is recorded on the stream right after the i-th
  // kernel launch, for per-kernel timing with CUDA events
  int launched = 0;
  auto mark = [&]() -> cudaError_t {
    const int i = launched++;
    return (events != nullptr && i < num_events) ? cudaEventRecord(events[i], stream) : cudaSuccess;
  };
  const PrefillWs w = prefill_ws_layout(T, N, allow_segments);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int *meta = reinterpret_cast<int *>(ws + w.meta);
  int *chunk_off = reinterpret_cast<int *>(ws + w.chunk_off);
  int *seq_order = reinterpret_cast<int *>(ws + w.seq_order);
  int4 *chunk_tab = reinterpret_cast<int4 *>(ws + w.chunk_tab);
  float *gcum = reinterpret_cast<float *>(ws + w.gcum);
  float *beta = reinterpret_cast<float *>(ws + w.beta);
  uint8_t *m2 = ws + w.m2;
  int4 *items = reinterpret_cast<int4 *>(ws + w.items);
  int *seg_off = reinterpret_cast<int *>(ws + w.seg_off);
  float *seg_ss = reinterpret_cast<float *>(ws + w.seg_ss);
  float *seg_sb = reinterpret_cast<float *>(ws + w.seg_sb);
  float *seg_phi = reinterpret_cast<float *>(ws + w.seg_phi);
  const int64_t seg_tokens = w.seg_chunks ? w.seg_chunks * kChunk : (int64_t{1} << 40);

  CUtensorMap tq, tk, tv, to;
  memset(&tq, 0, sizeof(tq));
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  memset(&to, 0, sizeof(to));
  if (T > 0) {
    // to: the output as [T][8 * 128] bf16, one (64 token x 128 v) box per
    // full chunk and v-head (the scan's TMA store)
    if (!make_tmap_2d(&tq, q, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tk, k, kHQK * kD, T, 64, 64, true) ||
        !make_tmap_2d(&tv, v, kHV * kD, T, 64, 64, true) ||
        !make_tmap_2d(&to, out, kHV * kD, T, kD, 64, false))
      return cudaErrorInvalidValue;
  }

  gdn_prefill_meta_kernel<<<1, kMetaThreads, 0, stream>>>(
      cu_seqlens, static_cast<int>(N), T, w.nt_max, meta, chunk_off, seq_order, chunk_tab,
      static_cast<int>(w.seg_chunks), static_cast<int>(w.seg_max), items, seg_off, slots,
      pool_slots);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = mark();
  if (err != cudaSuccess) return err;

  err = cudaFuncSetAttribute(gdn_prefill_prep_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem);
  if (err != cudaSuccess) return err;
  if (w.nt_max > 0) {
    dim3 grid(static_cast<unsigned>(w.nt_max), kHQK);
    gdn_prefill_prep_kernel<false><<<grid, kPrepThreads, kPrepSmem, stream>>>(
        tq, tk, A_log, static_cast<const uint16_t *>(a), dt_bias,
        static_cast<const uint16_t *>(b), cu_seqlens, meta, chunk_tab, gcum, beta, m2);
    err = cudaGetLastError();
    if (err == cudaSuccess) err = mark();
    if (err != cudaSuccess) return err;
  }
  err = cudaFuncSetAttribute(gdn_prefill_scan_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, ScanSmem::kBytes);
  if (err != cudaSuccess) return err;
  // pass 1 (the only pass without segmentation)
  const int64_t n1 = w.seg_chunks ? 2 * w.seg_max : N;
  gdn_prefill_scan_kernel<false><<<static_cast<unsigned>(n1 * kHV), kScanThreads,
                                   ScanSmem::kBytes, stream>>>(
      tq, tk, tv, to, state, cu_seqlens, meta, chunk_off, gcum, beta, m2, scale,
      static_cast<uint16_t *>(out), final_state, items, 2, seg_tokens, seg_off, seg_ss, seg_sb,
      seg_phi, slots, nullptr, nullptr);
  err = cudaGetLastError();
  if (err == cudaSuccess) err = mark();
  if (err != cudaSuccess || w.seg_chunks == 0) return err;

  err = cudaFuncSetAttribute(gdn_prefill_compose_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kCmpSmem);
  if (err != cudaSuccess) return err;
  dim3 cgrid(static_cast<unsigned>(N), kHV, kD / kComposeRows);
  gdn_prefill_compose_kernel<<<cgrid, kComposeThreads, kCmpSmem, stream>>>(meta, seg_off, seg_ss,
                                                                           seg_sb, seg_phi);
  err = cudaGetLastError();
  if (err == cudaSuccess) err = mark();
  if (err != cudaSuccess) return err;
  // pass 3
  gdn_prefill_scan_kernel<false><<<static_cast<unsigned>(w.seg_max * kHV), kScanThreads,
                                   ScanSmem::kBytes, stream>>>(
      tq, tk, tv, to, state, cu_seqlens, meta, chunk_off, gcum, beta, m2, scale,
      static_cast<uint16_t *>(out), final_state, items + 2 * w.seg_max, 3, seg_tokens, seg_off,
      seg_ss, seg_sb, seg_phi, slots, nullptr, nullptr);
  err = cudaGetLastError();
  if (err == cudaSuccess) err = mark();
  return err;
}

}  // namespace gdn
