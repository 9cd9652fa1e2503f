/*
 * gdn_oracle.c -- CPU restatement of the Gated DeltaNet (GDN) decode step and
 * prefill recurrence for the fixed geometry qk4_v8_d128_k_last.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against (tests/, __graft_entry__.smoke()) and the CPU baseline that
 * bench.py times (its `cpu_baseline` leg and `--impl reference` arm).  The
 * product path never links, loads or calls it.
 *
 * Semantics follow the reference solution files (paths inside the reference
 * project sanghamitrajohri/track-c-gdn):
 *   decode : gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py
 *            gates :21-23 (softplus with threshold 20), :59-65;
 *            per-row update and readout :67-79; q pre-scaled :56.
 *   prefill: solution/triton/kernel.py
 *            gates :1712-1722 (stable softplus, sigmoid beta);
 *            the chunked kernels :473-1542 are an exact re-association of the
 *            token-by-token recurrence implemented here:
 *              S <- g_t S ; S <- S + beta_t (v_t - S k_t) k_t^T ; o_t = scale S q_t
 *            starting from h0 (or zeros), returning the final S.
 * Layouts (all row-major, contiguous):
 *   q, k  : [T, 4, 128] bf16 (passed as raw uint16 bit patterns)
 *   v     : [T, 8, 128] bf16
 *   a, b  : [T, 8]      bf16
 *   A_log, dt_bias : [8] fp32
 *   state : [N, 8, 128(v), 128(k)] fp32  ("k-last")
 *   out   : [T, 8, 128] fp32 (unrounded; tests round to bf16 as needed)
 * v-head hv reads q/k head hv/2 (decode kernel.py:47, prefill kernel.py:495).
 *
 * Arithmetic is IEEE fp32 throughout (expf/logf from libm), matching the
 * "fp32 recurrence" the reference kernels approximate.  Work is split across
 * (sequence, v-head) pairs with OpenMP; each pair is independent.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define HQK 4
#define HV 8
#define D 128

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

/* decode kernel.py:21-23 -- softplus with a threshold of 20 */
static inline float softplus_thr20(float x) {
  return x <= 20.0f ? logf(1.0f + expf(x)) : x;
}

/* prefill kernel.py:1714-1720 -- overflow-safe softplus */
static inline float softplus_stable(float x) {
  return x > 0.0f ? x + logf(1.0f + expf(-x)) : logf(1.0f + expf(x));
}

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

int gdn_oracle_abi_version(void) { return 1; }

/*
 * One decode step for B requests (decode kernel.py:26-79).
 * state may be NULL (zero state, kernel.py:86-94).  new_state may alias state.
 */
void gdn_oracle_decode(int B, const uint16_t *q, const uint16_t *k,
                       const uint16_t *v, const float *state,
                       const float *A_log, const uint16_t *a,
                       const float *dt_bias, const uint16_t *b, float scale,
                       float *out, float *new_state, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int bh = 0; bh < B * HV; ++bh) {
    const int bb = bh / HV, hv = bh % HV, h = hv / 2;
    float qv[D], kv[D], row[D];
    for (int i = 0; i < D; ++i) {
      qv[i] = bf16_to_f32(q[((size_t)bb * HQK + h) * D + i]) * scale;
      kv[i] = bf16_to_f32(k[((size_t)bb * HQK + h) * D + i]);
    }
    const float a_val = bf16_to_f32(a[(size_t)bb * HV + hv]);
    const float b_val = bf16_to_f32(b[(size_t)bb * HV + hv]);
    const float log_g = -expf(A_log[hv]) * softplus_thr20(a_val + dt_bias[hv]);
    const float g = expf(log_g);
    const float beta = 1.0f / (1.0f + expf(-b_val));
    const size_t sbase = (size_t)bh * D * D;
    for (int vv = 0; vv < D; ++vv) {
      const float vval = bf16_to_f32(v[(size_t)bh * D + vv]);
      float old = 0.0f;
      for (int i = 0; i < D; ++i) {
        row[i] = (state ? state[sbase + (size_t)vv * D + i] : 0.0f) * g;
        old += row[i] * kv[i];
      }
      const float delta = beta * (vval - old);
      float o = 0.0f;
      for (int i = 0; i < D; ++i) {
        row[i] = row[i] + kv[i] * delta;
        o += row[i] * qv[i];
      }
      out[(size_t)bh * D + vv] = o;
      memcpy(new_state + sbase + (size_t)vv * D, row, sizeof(row));
    }
  }
}

/*
 * Prefill over N ragged sequences described by cu_seqlens[N+1] (int64 token
 * offsets, cu_seqlens[N] == T).  h0 may be NULL (zero initial state).
 * out: [T, 8, 128] fp32; final_state: [N, 8, 128, 128] fp32.
 */
void gdn_oracle_prefill(int N, const int64_t *cu_seqlens, const uint16_t *q,
                        const uint16_t *k, const uint16_t *v, const float *h0,
                        const float *A_log, const uint16_t *a,
                        const float *dt_bias, const uint16_t *b, float scale,
                        float *out, float *final_state, int nthreads) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int nh = 0; nh < N * HV; ++nh) {
    const int n = nh / HV, hv = nh % HV, h = hv / 2;
    float *S = (float *)malloc(sizeof(float) * D * D);
    if (h0) memcpy(S, h0 + (size_t)nh * D * D, sizeof(float) * D * D);
    else memset(S, 0, sizeof(float) * D * D);
    const float decay = expf(A_log[hv]);
    float kv[D], qv[D];
    for (int64_t t = cu_seqlens[n]; t < cu_seqlens[n + 1]; ++t) {
      const float x = bf16_to_f32(a[(size_t)t * HV + hv]) + dt_bias[hv];
      const float g = expf(-decay * softplus_stable(x));
      const float beta = sigmoidf_(bf16_to_f32(b[(size_t)t * HV + hv]));
      for (int i = 0; i < D; ++i) {
        kv[i] = bf16_to_f32(k[((size_t)t * HQK + h) * D + i]);
        qv[i] = bf16_to_f32(q[((size_t)t * HQK + h) * D + i]);
      }
      for (int vv = 0; vv < D; ++vv) {
        float *row = S + (size_t)vv * D;
        float old = 0.0f;
        for (int i = 0; i < D; ++i) {
          row[i] *= g;
          old += row[i] * kv[i];
        }
        const float delta =
            beta * (bf16_to_f32(v[((size_t)t * HV + hv) * D + vv]) - old);
        float o = 0.0f;
        for (int i = 0; i < D; ++i) {
          row[i] += delta * kv[i];
          o += row[i] * qv[i];
        }
        out[((size_t)t * HV + hv) * D + vv] = o * scale;
      }
    }
    memcpy(final_state + (size_t)nh * D * D, S, sizeof(float) * D * D);
    free(S);
  }
}
