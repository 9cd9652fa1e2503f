/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet kernel pair for the
 * fixed geometry qk4_v8_d128_k_last:
 *   4 q/k heads, 8 v heads (v-head h reads q/k head h/2), head dim 128,
 *   recurrent state k-last fp32 [N, 8, 128 (v), 128 (k)].
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream (cudaStream_t passed as void*, NULL = legacy default stream).  Calls
 * are asynchronous on that stream, never synchronise the host, never
 * allocate device memory (outputs and workspaces are the caller's; the
 * Python mirror in track-c-gdn_b200/ is what allocates them for its
 * value-returning `run`s), and return a gdn_status_t.  Tensors are dense
 * row-major (contiguous); bf16 tensors are passed as raw 16-bit storage.
 *
 * The library is built from track-c-gdn_b200/csrc/ by __graft_entry__.build()
 * into track-c-gdn_b200/libgdn_b200.so.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GDN_OK = 0,
  GDN_ERR_NULL_POINTER = 1,   /* a required pointer is NULL */
  GDN_ERR_BAD_SIZE = 2,       /* negative / inconsistent sizes */
  GDN_ERR_MISALIGNED = 3,     /* a pointer violates the documented alignment */
  GDN_ERR_WORKSPACE = 4,      /* workspace missing or smaller than required */
  GDN_ERR_LAUNCH = 5,         /* the CUDA launch itself failed */
  GDN_ERR_DEVICE = 6,         /* no sm_100 device / wrong device */
  GDN_ERR_ALIASING = 7,       /* outputs overlap inputs where not allowed */
  GDN_ERR_TOO_LARGE = 8       /* problem exceeds the no-allocation scratch */
} gdn_status_t;

/* ABI version of this header (bumped on any signature change). */
int gdn_b200_abi_version(void);

/* Human-readable text for a gdn_status_t. */
const char *gdn_b200_status_string(int status);

/*
 * Device-side status word.  Kernels never trap: when one meets an
 * inconsistency it cannot report synchronously (cu_seqlens that do not match
 * total_tokens, a bounded wait that ran out) it records a nonzero code in a
 * per-device word and skips the work.  This call copies the word for the
 * current device into *code (stream-ordered, then synchronises `stream`) and
 * clears it.  Codes: 0 none, 1 bad cu_seqlens, 2 wait timeout, 3 a state-pool
 * slot index outside [0, pool_slots) (that request / call is skipped), 4 a
 * device-side index check failed (debug build libgdn_b200_debug.so only).
 */
int gdn_b200_read_device_status(int *code, void *stream);

/*
 * Decode step.  Replaces the reference entry point
 *   run(q, k, v, state, A_log, a, dt_bias, b, scale)
 *   gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:100-146
 * q, k      [B,1,4,128] bf16 (8-byte aligned)
 * v         [B,1,8,128] bf16 (8-byte aligned)
 * state     [B,8,128,128] fp32 (16-byte aligned) or NULL for a zero state
 *           (kernel.py:86-94)
 * A_log     [8] fp32;  dt_bias [8] fp32
 * a, b      [B,1,8] bf16
 * scale     0.0f selects 1/sqrt(128) (kernel.py:112-115)
 * out       [B,1,8,128] bf16 (8-byte aligned)
 * new_state [B,8,128,128] fp32 (16-byte aligned).  May equal `state` (update
 *           in place); must not partially overlap it.
 * Per (request, v-head) it computes g = exp(-exp(A_log) softplus(a+dt_bias))
 * (softplus threshold 20), beta = sigmoid(b), S <- g S,
 * S <- S + beta (v - S k) k^T, out = S (scale q)   (kernel.py:26-79).
 */
int gdn_decode_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                  const float *state, const float *A_log,
                                  const void *a, const float *dt_bias,
                                  const void *b, float scale, int64_t batch,
                                  void *out, float *new_state, void *stream);

/*
 * Multi-token decode (speculative verify / multi-token prediction): T tokens
 * per request, applied in order -- the same result as T calls of
 * gdn_decode_qk4_v8_d128_k_last (bit for bit), with each head's 64 KiB state
 * streamed through HBM once instead of T times.  No counterpart in the
 * reference (its decode definition takes one token per request).
 * q, k      [B,T,4,128] bf16 (8-byte aligned)
 * v         [B,T,8,128] bf16 (8-byte aligned)
 * state     [B,8,128,128] fp32 (16-byte aligned) or NULL for a zero state
 * a, b      [B,T,8] bf16;  A_log, dt_bias [8] fp32;  scale 0.0f -> 1/sqrt(128)
 * out       [B,T,8,128] bf16 (8-byte aligned)
 * new_state [B,8,128,128] fp32, the state after the last token; may equal
 *           `state`
 * intermediate_states  NULL, or [B,T,8,128,128] fp32 (16-byte aligned,
 *           overlapping neither state buffer): the state after each token,
 *           for rolling back rejected speculative tokens
 * 1 <= T <= GDN_DECODE_MTP_MAX_TOKENS.
 */
#define GDN_DECODE_MTP_MAX_TOKENS 64
int gdn_decode_mtp_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                      const float *state, const float *A_log,
                                      const void *a, const float *dt_bias,
                                      const void *b, float scale, int64_t batch,
                                      int64_t num_tokens, void *out, float *new_state,
                                      float *intermediate_states, void *stream);

/*
 * Decode against a paged state pool: the state of request i lives at
 * state_pool[slots[i]] ([pool_slots,8,128,128] fp32, 16-byte aligned) and is
 * updated there in place, so a serving engine keeps its GDN cache as one pool
 * and never gathers or scatters states around the call.  num_tokens = 1 is
 * gdn_decode_qk4_v8_d128_k_last, > 1 gdn_decode_mtp_qk4_v8_d128_k_last (same
 * results bit for bit).  slots: [B] int32 on the device, distinct within a
 * call (requests sharing a slot race); a slot outside [0, pool_slots) sets
 * device status 3 and that request is skipped.  No counterpart in the
 * reference (its definitions take dense [B,...] states).
 */
int gdn_decode_pool_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                       float *state_pool, int64_t pool_slots,
                                       const int32_t *slots, const float *A_log,
                                       const void *a, const float *dt_bias, const void *b,
                                       float scale, int64_t batch, int64_t num_tokens,
                                       void *out, void *stream);

/*
 * Decode with the recurrent state stored in bf16 (half the state bytes, so
 * about twice the decode throughput on the HBM roofline): the state is
 * widened to fp32, the step computed in fp32 exactly as
 * gdn_decode_qk4_v8_d128_k_last does (the output uses the unrounded update),
 * and the new state rounded to nearest even and stored back in place; with
 * T > 1 tokens the state is rounded after every token, as T separate calls
 * would.  state_bf16: [B,8,128,128] bf16 when slots is NULL, else a pool
 * [pool_slots,8,128,128] bf16 addressed by slots ([B] int32, distinct; a slot
 * outside the pool sets device status 3).  16-byte aligned.  The reference
 * keeps its state in fp32 only; this is an opt-in storage format.
 */
int gdn_decode_bf16_state_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                             void *state_bf16, int64_t pool_slots,
                                             const int32_t *slots, const float *A_log,
                                             const void *a, const float *dt_bias, const void *b,
                                             float scale, int64_t batch, int64_t num_tokens,
                                             void *out, void *stream);

/*
 * Workspace (bytes) the prefill needs for `total_tokens` tokens packed into
 * `num_seqs` sequences.  Independent of the sequence lengths.
 */
size_t gdn_prefill_workspace_bytes(int64_t total_tokens, int64_t num_seqs);

/*
 * Number of kernels one gdn_prefill_qk4_v8_d128_k_last call launches for
 * (total_tokens, num_seqs): 3, or 5 when the call uses the segmented
 * evaluation (see below); 0 for num_seqs = 0.  For launch accounting; no
 * counterpart in the reference.
 */
int gdn_prefill_kernel_launches(int64_t total_tokens, int64_t num_seqs);

/*
 * Chunked (64-token) prefill over ragged sequences.  Replaces the reference
 * entry point
 *   run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
 *   solution/triton/kernel.py:1762-1802
 * q, k        [T,4,128] bf16 (16-byte aligned)
 * v           [T,8,128] bf16 (16-byte aligned)
 * state       [N,8,128,128] fp32 initial states (16-byte aligned), or NULL
 *             for zeros
 * A_log, dt_bias [8] fp32;  a, b [T,8] bf16
 * cu_seqlens  [N+1] int64 on the device, cu_seqlens[0] = 0,
 *             non-decreasing, cu_seqlens[N] = T (checked on the device; a
 *             violation sets device status 1 and leaves outputs unwritten)
 * scale       0.0f selects 1/sqrt(128)
 * out         [T,8,128] bf16 (16-byte aligned)
 * final_state [N,8,128,128] fp32 (16-byte aligned); may equal `state`
 * workspace   >= gdn_prefill_workspace_bytes(T, N) bytes, 1024-byte aligned
 * No host synchronisation: unlike the reference (kernel.py:1665, :181-184)
 * the chunk metadata is built on the device.
 * Few long sequences (num_seqs <= 16 averaging >= 12 chunks, decided from T
 * and N alone) are evaluated in segments run in parallel and then joined
 * through the segments' affine state maps; results agree with the
 * single-pass evaluation within the stated tolerances, not bit for bit.
 */
int gdn_prefill_qk4_v8_d128_k_last(
    const void *q, const void *k, const void *v, const float *state,
    const float *A_log, const void *a, const float *dt_bias, const void *b,
    const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
    float scale, void *out, float *final_state, void *workspace,
    size_t workspace_bytes, void *stream);

/*
 * gdn_prefill_qk4_v8_d128_k_last, recording CUDA events for per-kernel
 * timing: events[i] (a cudaEvent_t passed as void*) is recorded on `stream`
 * right after the i-th kernel this call launches, for i < num_events.  The
 * call launches gdn_prefill_kernel_launches(T, N) kernels, in this order:
 * metadata, chunk preparation, scan (pass 1), and with the segmented
 * evaluation also the segment composition and the scan's pass 3.  Results
 * are those of gdn_prefill_qk4_v8_d128_k_last bit for bit.  No counterpart
 * in the reference (its timing is the harness's, around the whole call).
 */
int gdn_prefill_qk4_v8_d128_k_last_events(
    const void *q, const void *k, const void *v, const float *state,
    const float *A_log, const void *a, const float *dt_bias, const void *b,
    const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
    float scale, void *out, float *final_state, void *workspace,
    size_t workspace_bytes, void *const *events, int num_events, void *stream);

/*
 * Prefill against a paged state pool: sequence n starts from
 * state_pool[slots[n]] and its final state is written back there (a new
 * sequence's slot must hold zeros or its initial state).  Otherwise as
 * gdn_prefill_qk4_v8_d128_k_last (same workspace size).  slots: [N] int32 on
 * the device, distinct; any slot outside [0, pool_slots) sets device status 3
 * and the call writes nothing.  No counterpart in the reference.
 */
int gdn_prefill_pool_qk4_v8_d128_k_last(
    const void *q, const void *k, const void *v, float *state_pool, int64_t pool_slots,
    const int32_t *slots, const float *A_log, const void *a, const float *dt_bias,
    const void *b, const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
    float scale, void *out, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Prefill that allocates nothing -- no counterpart in the reference.
 * Same arguments and results as gdn_prefill_qk4_v8_d128_k_last minus the
 * workspace: for callers that may not allocate device memory while a step
 * runs (e.g. a plugin whose host framework owns all device memory, or a
 * serving loop that cannot afford cudaMalloc's implicit synchronisation).
 * The scratch is a 32 MiB buffer compiled into the library
 * (GDN_PREFILL_NOALLOC_SCRATCH_BYTES), held on every GPU that loads it until
 * exit.  When gdn_prefill_workspace_bytes(T, N) exceeds it, the call runs the
 * single-pass evaluation (smaller workspace) if that fits, and otherwise is
 * rejected with GDN_ERR_TOO_LARGE before anything is launched; a problem
 * always fits when T + 64 N <= 15,872 (e.g. T <= 15,808 for one sequence).
 * All calls on a device share the buffer: calls whose kernels overlap on
 * that GPU race and must be serialised by the caller.  The first call on
 * each device looks up the buffer's device address (cudaGetSymbolAddress,
 * with that device current); make it before any stream capture begins.
 */
#define GDN_PREFILL_NOALLOC_SCRATCH_BYTES (32u << 20)
int gdn_prefill_qk4_v8_d128_k_last_noalloc(
    const void *q, const void *k, const void *v, const float *state,
    const float *A_log, const void *a, const float *dt_bias, const void *b,
    const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
    float scale, void *out, float *final_state, void *stream);

/*
 * Backward of the prefill -- no counterpart in the reference, whose prefill
 * is forward-only (solution/triton/kernel.py:1: "Forward-only").
 * Gradients of (out, final_state) = gdn_prefill_qk4_v8_d128_k_last(q, k, v,
 * state, A_log, a, dt_bias, b, cu_seqlens, scale) given
 *   d_out          [T,8,128] bf16 (16-byte aligned),
 *   d_final_state  [N,8,128,128] fp32 or NULL (zero),
 * written as fp32:
 *   dq, dk [T,4,128]   dv [T,8,128]   da, db [T,8]   dA_log, ddt_bias [8]
 *   d_state [N,8,128,128] (the initial state's gradient; NULL: not computed).
 * The inputs are the forward's (state NULL: zero initial state); the call
 * recomputes the forward's chunk states itself.  dq/dk/dv/d_state/d_final
 * 16-byte aligned, da/db/dA_log/ddt_bias 4-byte aligned.  The workspace
 * (1024-byte aligned, gdn_prefill_backward_workspace_bytes(T, N) bytes) holds
 * the recomputed chunk-start states and their gradients (bf16): about
 * 2 x 256 KiB per 64-token chunk, plus 8 KiB per token.  No host
 * synchronisation; bad cu_seqlens are reported through the device status
 * (code 1) as in the forward.  Deterministic: identical inputs give
 * identical gradients bit for bit.
 */
size_t gdn_prefill_backward_workspace_bytes(int64_t total_tokens, int64_t num_seqs);
int gdn_prefill_backward_kernel_launches(void);
int gdn_prefill_backward_qk4_v8_d128_k_last(
    const void *q, const void *k, const void *v, const float *state,
    const float *A_log, const void *a, const float *dt_bias, const void *b,
    const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
    float scale, const void *d_out, const float *d_final_state,
    float *dq, float *dk, float *dv, float *da, float *db,
    float *dA_log, float *ddt_bias, float *d_state,
    void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
