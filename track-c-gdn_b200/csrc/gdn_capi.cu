// gdn_capi.cu -- extern "C" entry points declared in include/gdn_b200.h.
//
// Host-side checks mirror the reference's own asserts (decode kernel.py:117-120,
// prefill kernel.py:1635-1667) as far as they can be made without touching
// device memory; the one check that needs device data (cu_seqlens[-1] == T,
// kernel.py:1665) runs on the device (device status 1) so no call ever
// synchronises the host.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../../include/gdn_b200.h"
#include "gdn_common.cuh"

namespace gdn {
cudaError_t launch_decode(const void *q, const void *k, const void *v, const float *state,
                          const float *A_log, const void *a, const float *dt_bias,
                          const void *b, float scale, int64_t batch, void *out,
                          float *new_state, const int32_t *slots, int64_t pool_slots,
                          cudaStream_t stream);
cudaError_t launch_decode_mtp(const void *q, const void *k, const void *v, const float *state,
                              const float *A_log, const void *a, const float *dt_bias,
                              const void *b, float scale, int64_t batch, int num_tokens,
                              void *out, float *new_state, float *inter, const int32_t *slots,
                              int64_t pool_slots, cudaStream_t stream);
cudaError_t launch_decode_bf16_state(const void *q, const void *k, const void *v, void *state,
                                     const float *A_log, const void *a, const float *dt_bias,
                                     const void *b, float scale, int64_t batch, int num_tokens,
                                     void *out, const int32_t *slots, int64_t pool_slots,
                                     cudaStream_t stream);
size_t prefill_workspace_bytes(int64_t T, int64_t N, bool allow_segments);
int prefill_kernel_launches(int64_t T, int64_t N, bool allow_segments);
size_t prefill_bwd_workspace_bytes(int64_t T, int64_t N);
int prefill_bwd_kernel_launches();
cudaError_t launch_prefill_bwd(const void *q, const void *k, const void *v, const float *state,
                               const float *A_log, const void *a, const float *dt_bias,
                               const void *b, const int64_t *cu_seqlens, int64_t N, int64_t T,
                               float scale, const void *d_out, const float *d_final, float *dq,
                               float *dk, float *dv, float *da, float *db, float *dA_log,
                               float *ddt_bias, float *d_state, void *workspace,
                               cudaStream_t stream);
cudaError_t launch_prefill(const void *q, const void *k, const void *v, const float *state,
                           const float *A_log, const void *a, const float *dt_bias, const void *b,
                           const int64_t *cu_seqlens, int64_t N, int64_t T, float scale,
                           void *out, float *final_state, void *workspace, bool allow_segments,
                           const int32_t *slots, int64_t pool_slots, cudaStream_t stream,
                           const cudaEvent_t *events, int num_events);
}  // namespace gdn

namespace {

constexpr float kDefaultScale = 0.08838834764831845f;  // 1/sqrt(128)

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool overlap(const void *a, size_t na, const void *b, size_t nb) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + nb && y < x + na;
}

// Current device must be sm_100 (B200 family); cached per device ordinal.
int check_device(int *num_sms) {
  static int cached_dev = -1, cached_ok = 0, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_DEVICE;
  if (dev != cached_dev) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return GDN_ERR_DEVICE;
    cached_ok = prop.major == 10 && prop.minor == 0;
    cached_sms = prop.multiProcessorCount;
    cached_dev = dev;
  }
  if (num_sms) *num_sms = cached_sms;
  return cached_ok ? GDN_OK : GDN_ERR_DEVICE;
}


// Argument checks of the dense prefill entry points, then the launches.
int prefill_checked(const void *q, const void *k, const void *v, const float *state,
                    const float *A_log, const void *a, const float *dt_bias, const void *b,
                    const int64_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                    float scale, void *out, float *final_state, void *workspace,
                    size_t workspace_bytes, void *stream, const cudaEvent_t *events,
                    int num_events) {
  if (num_seqs < 0 || total_tokens < 0 || total_tokens > (int64_t{1} << 31) ||
      num_seqs > (int64_t{1} << 24))
    return GDN_ERR_BAD_SIZE;
  if (num_seqs == 0) return total_tokens == 0 ? GDN_OK : GDN_ERR_BAD_SIZE;
  if (!cu_seqlens || !A_log || !dt_bias || !final_state || !workspace) return GDN_ERR_NULL_POINTER;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_NULL_POINTER;
  if ((q && !aligned(q, 16)) || (k && !aligned(k, 16)) || (v && !aligned(v, 16)) ||
      (out && !aligned(out, 16)) || !aligned(final_state, 16) || (state && !aligned(state, 16)) ||
      !aligned(cu_seqlens, 8))
    return GDN_ERR_MISALIGNED;
  if (!aligned(workspace, 1024) ||
      workspace_bytes < gdn::prefill_workspace_bytes(total_tokens, num_seqs, true))
    return GDN_ERR_WORKSPACE;
  const size_t state_bytes = static_cast<size_t>(num_seqs) * gdn::kHV * gdn::kD * gdn::kD * 4;
  if (state && state != final_state && overlap(state, state_bytes, final_state, state_bytes))
    return GDN_ERR_ALIASING;
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs,
                                        total_tokens, scale, out, final_state, workspace, true,
                                        nullptr, 0, static_cast<cudaStream_t>(stream), events,
                                        num_events);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int gdn_b200_abi_version(void) { return 1; }

const char *gdn_b200_status_string(int status) {
  switch (status) {
    case GDN_OK: return "ok";
    case GDN_ERR_NULL_POINTER: return "a required pointer is NULL";
    case GDN_ERR_BAD_SIZE: return "negative or inconsistent sizes";
    case GDN_ERR_MISALIGNED: return "a pointer violates the documented alignment";
    case GDN_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case GDN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GDN_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case GDN_ERR_ALIASING: return "an output partially overlaps an input";
    case GDN_ERR_TOO_LARGE: return "problem exceeds the no-allocation entry point's built-in scratch";
    default: return "unknown status";
  }
}

int gdn_b200_read_device_status(int *code, void *stream) {
  if (code == nullptr) return GDN_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int zero = 0;
  if (cudaMemcpyFromSymbolAsync(code, gdn::g_device_status, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (cudaMemcpyToSymbolAsync(gdn::g_device_status, &zero, sizeof(int), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return GDN_ERR_LAUNCH;
  return GDN_OK;
}

int gdn_decode_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                  const float *state, const float *A_log, const void *a,
                                  const float *dt_bias, const void *b, float scale,
                                  int64_t batch, void *out, float *new_state, void *stream) {
  if (batch < 0 || batch > (int64_t{1} << 26)) return GDN_ERR_BAD_SIZE;
  if (batch == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
    return GDN_ERR_NULL_POINTER;
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(out, 8) ||
      !aligned(new_state, 16) || (state && !aligned(state, 16)) || !aligned(a, 2) ||
      !aligned(b, 2) || !aligned(A_log, 4) || !aligned(dt_bias, 4))
    return GDN_ERR_MISALIGNED;
  const size_t state_bytes = static_cast<size_t>(batch) * gdn::kHV * gdn::kD * gdn::kD * 4;
  if (state && state != new_state && overlap(state, state_bytes, new_state, state_bytes))
    return GDN_ERR_ALIASING;
  int sms = 0;
  if (int st = check_device(&sms)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_decode(q, k, v, state, A_log, a, dt_bias, b, scale, batch, out,
                                       new_state, nullptr, 0, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_decode_mtp_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                      const float *state, const float *A_log, const void *a,
                                      const float *dt_bias, const void *b, float scale,
                                      int64_t batch, int64_t num_tokens, void *out,
                                      float *new_state, float *intermediate_states, void *stream) {
  if (batch < 0 || num_tokens < 1 || num_tokens > GDN_DECODE_MTP_MAX_TOKENS ||
      batch > (int64_t{1} << 26) / num_tokens)
    return GDN_ERR_BAD_SIZE;
  if (batch == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
    return GDN_ERR_NULL_POINTER;
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(out, 8) ||
      !aligned(new_state, 16) || (state && !aligned(state, 16)) ||
      (intermediate_states && !aligned(intermediate_states, 16)) || !aligned(a, 2) ||
      !aligned(b, 2) || !aligned(A_log, 4) || !aligned(dt_bias, 4))
    return GDN_ERR_MISALIGNED;
  const size_t state_bytes = static_cast<size_t>(batch) * gdn::kHV * gdn::kD * gdn::kD * 4;
  if (state && state != new_state && overlap(state, state_bytes, new_state, state_bytes))
    return GDN_ERR_ALIASING;
  if (intermediate_states) {
    const size_t inter_bytes = state_bytes * static_cast<size_t>(num_tokens);
    if ((state && overlap(state, state_bytes, intermediate_states, inter_bytes)) ||
        overlap(new_state, state_bytes, intermediate_states, inter_bytes))
      return GDN_ERR_ALIASING;
  }
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_decode_mtp(q, k, v, state, A_log, a, dt_bias, b, scale, batch,
                                           static_cast<int>(num_tokens), out, new_state,
                                           intermediate_states, nullptr, 0,
                                           static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

size_t gdn_prefill_workspace_bytes(int64_t total_tokens, int64_t num_seqs) {
  if (total_tokens < 0 || num_seqs < 0) return 0;
  return gdn::prefill_workspace_bytes(total_tokens, num_seqs, true);
}

int gdn_prefill_kernel_launches(int64_t total_tokens, int64_t num_seqs) {
  if (total_tokens < 0 || num_seqs < 0) return 0;
  return gdn::prefill_kernel_launches(total_tokens, num_seqs, true);
}

size_t gdn_prefill_backward_workspace_bytes(int64_t total_tokens, int64_t num_seqs) {
  if (total_tokens < 0 || num_seqs < 0) return 0;
  return gdn::prefill_bwd_workspace_bytes(total_tokens, num_seqs);
}

int gdn_prefill_backward_kernel_launches(void) { return gdn::prefill_bwd_kernel_launches(); }

int gdn_prefill_backward_qk4_v8_d128_k_last(
    const void *q, const void *k, const void *v, const float *state, const float *A_log,
    const void *a, const float *dt_bias, const void *b, const int64_t *cu_seqlens,
    int64_t num_seqs, int64_t total_tokens, float scale, const void *d_out,
    const float *d_final_state, float *dq, float *dk, float *dv, float *da, float *db,
    float *dA_log, float *ddt_bias, float *d_state, void *workspace, size_t workspace_bytes,
    void *stream) {
  if (num_seqs < 0 || total_tokens < 0 || total_tokens > (int64_t{1} << 31) ||
      num_seqs > (int64_t{1} << 24))
    return GDN_ERR_BAD_SIZE;
  if (num_seqs == 0) return total_tokens == 0 ? GDN_OK : GDN_ERR_BAD_SIZE;
  if (!cu_seqlens || !A_log || !dt_bias || !dA_log || !ddt_bias || !workspace)
    return GDN_ERR_NULL_POINTER;
  if (total_tokens > 0 &&
      (!q || !k || !v || !a || !b || !d_out || !dq || !dk || !dv || !da || !db))
    return GDN_ERR_NULL_POINTER;
  const void *a16[] = {q, k, v, d_out, dq, dk, dv, state, d_final_state, d_state};
  for (const void *p : a16)
    if (p && !aligned(p, 16)) return GDN_ERR_MISALIGNED;
  if ((da && !aligned(da, 4)) || (db && !aligned(db, 4)) || !aligned(dA_log, 4) ||
      !aligned(ddt_bias, 4) || !aligned(cu_seqlens, 8))
    return GDN_ERR_MISALIGNED;
  if (!aligned(workspace, 1024) ||
      workspace_bytes < gdn::prefill_bwd_workspace_bytes(total_tokens, num_seqs))
    return GDN_ERR_WORKSPACE;
  const size_t state_bytes = static_cast<size_t>(num_seqs) * gdn::kHV * gdn::kD * gdn::kD * 4;
  if (d_state && ((state && overlap(state, state_bytes, d_state, state_bytes)) ||
                  (d_final_state && overlap(d_final_state, state_bytes, d_state, state_bytes))))
    return GDN_ERR_ALIASING;
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_prefill_bwd(
      q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens, scale, d_out,
      d_final_state, dq, dk, dv, da, db, dA_log, ddt_bias, d_state, workspace,
      static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_prefill_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                   const float *state, const float *A_log, const void *a,
                                   const float *dt_bias, const void *b,
                                   const int64_t *cu_seqlens, int64_t num_seqs,
                                   int64_t total_tokens, float scale, void *out,
                                   float *final_state, void *workspace, size_t workspace_bytes,
                                   void *stream) {
  return prefill_checked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                         scale, out, final_state, workspace, workspace_bytes, stream, nullptr, 0);
}

int gdn_prefill_qk4_v8_d128_k_last_events(const void *q, const void *k, const void *v,
                                          const float *state, const float *A_log, const void *a,
                                          const float *dt_bias, const void *b,
                                          const int64_t *cu_seqlens, int64_t num_seqs,
                                          int64_t total_tokens, float scale, void *out,
                                          float *final_state, void *workspace,
                                          size_t workspace_bytes, void *const *events,
                                          int num_events, void *stream) {
  if (num_events < 0 || (num_events > 0 && events == nullptr)) return GDN_ERR_NULL_POINTER;
  return prefill_checked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                         scale, out, final_state, workspace, workspace_bytes, stream,
                         reinterpret_cast<const cudaEvent_t *>(events), num_events);
}

int gdn_decode_pool_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                       float *state_pool, int64_t pool_slots,
                                       const int32_t *slots, const float *A_log, const void *a,
                                       const float *dt_bias, const void *b, float scale,
                                       int64_t batch, int64_t num_tokens, void *out,
                                       void *stream) {
  if (batch < 0 || pool_slots < 0 || num_tokens < 1 || num_tokens > GDN_DECODE_MTP_MAX_TOKENS ||
      batch > (int64_t{1} << 26) / num_tokens || pool_slots > (int64_t{1} << 26))
    return GDN_ERR_BAD_SIZE;
  if (batch == 0) return GDN_OK;
  if (pool_slots == 0) return GDN_ERR_BAD_SIZE;
  if (!q || !k || !v || !state_pool || !slots || !A_log || !a || !dt_bias || !b || !out)
    return GDN_ERR_NULL_POINTER;
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(out, 8) ||
      !aligned(state_pool, 16) || !aligned(slots, 4) || !aligned(a, 2) || !aligned(b, 2) ||
      !aligned(A_log, 4) || !aligned(dt_bias, 4))
    return GDN_ERR_MISALIGNED;
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err =
      num_tokens == 1
          ? gdn::launch_decode(q, k, v, state_pool, A_log, a, dt_bias, b, scale, batch, out,
                               state_pool, slots, pool_slots, static_cast<cudaStream_t>(stream))
          : gdn::launch_decode_mtp(q, k, v, state_pool, A_log, a, dt_bias, b, scale, batch,
                                   static_cast<int>(num_tokens), out, state_pool, nullptr, slots,
                                   pool_slots, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_decode_bf16_state_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                             void *state_bf16, int64_t pool_slots,
                                             const int32_t *slots, const float *A_log,
                                             const void *a, const float *dt_bias, const void *b,
                                             float scale, int64_t batch, int64_t num_tokens,
                                             void *out, void *stream) {
  if (batch < 0 || num_tokens < 1 || num_tokens > GDN_DECODE_MTP_MAX_TOKENS ||
      batch > (int64_t{1} << 26) / num_tokens || pool_slots < 0 || pool_slots > (int64_t{1} << 26))
    return GDN_ERR_BAD_SIZE;
  if (batch == 0) return GDN_OK;
  if (slots && pool_slots == 0) return GDN_ERR_BAD_SIZE;
  if (!q || !k || !v || !state_bf16 || !A_log || !a || !dt_bias || !b || !out)
    return GDN_ERR_NULL_POINTER;
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(v, 8) || !aligned(out, 8) ||
      !aligned(state_bf16, 16) || (slots && !aligned(slots, 4)) || !aligned(a, 2) ||
      !aligned(b, 2) || !aligned(A_log, 4) || !aligned(dt_bias, 4))
    return GDN_ERR_MISALIGNED;
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_decode_bf16_state(
      q, k, v, state_bf16, A_log, a, dt_bias, b, scale, batch, static_cast<int>(num_tokens), out,
      slots, slots ? pool_slots : 0, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_prefill_pool_qk4_v8_d128_k_last(const void *q, const void *k, const void *v,
                                        float *state_pool, int64_t pool_slots,
                                        const int32_t *slots, const float *A_log, const void *a,
                                        const float *dt_bias, const void *b,
                                        const int64_t *cu_seqlens, int64_t num_seqs,
                                        int64_t total_tokens, float scale, void *out,
                                        void *workspace, size_t workspace_bytes, void *stream) {
  if (num_seqs < 0 || total_tokens < 0 || total_tokens > (int64_t{1} << 31) ||
      num_seqs > (int64_t{1} << 24) || pool_slots < 0 || pool_slots > (int64_t{1} << 26))
    return GDN_ERR_BAD_SIZE;
  if (num_seqs == 0) return total_tokens == 0 ? GDN_OK : GDN_ERR_BAD_SIZE;
  if (pool_slots == 0) return GDN_ERR_BAD_SIZE;
  if (!cu_seqlens || !A_log || !dt_bias || !state_pool || !slots || !workspace)
    return GDN_ERR_NULL_POINTER;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_NULL_POINTER;
  if ((q && !aligned(q, 16)) || (k && !aligned(k, 16)) || (v && !aligned(v, 16)) ||
      (out && !aligned(out, 16)) || !aligned(state_pool, 16) || !aligned(slots, 4) ||
      !aligned(cu_seqlens, 8))
    return GDN_ERR_MISALIGNED;
  if (!aligned(workspace, 1024) ||
      workspace_bytes < gdn::prefill_workspace_bytes(total_tokens, num_seqs, true))
    return GDN_ERR_WORKSPACE;
  if (int st = check_device(nullptr)) return st;
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_prefill(q, k, v, state_pool, A_log, a, dt_bias, b, cu_seqlens,
                                        num_seqs, total_tokens, scale, out, state_pool, workspace,
                                        true, slots, pool_slots, static_cast<cudaStream_t>(stream),
                                        nullptr, 0);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // extern "C"
