// gdn_prefill_noalloc.cu -- the chunked prefill with no allocation anywhere on
// the call path.
//
// Who needs it: callers that are not allowed to allocate device memory while
// they run a step -- for example a plugin inside a host framework that owns
// all device memory and forbids cudaMalloc inside its execute callback, or a
// serving loop that cannot take cudaMalloc's implicit device-wide
// synchronisation.  The regular entry point asks for a caller-provided
// workspace; this one uses a scratch buffer compiled into the library.
//
// The scratch is a file-scope device array of kNoallocScratchBytes (32 MiB).
// Every GPU that loads this library holds it until the process exits.  All
// calls on a device share it: two calls whose kernels overlap on that GPU
// (different streams, or another thread) race on it and must be serialised by
// the caller.  Nothing in it needs to start at zero -- each call's metadata
// kernel rewrites the header (chunk count, status flag, tables) that the
// later kernels read, and those kernels only read entries this call wrote --
// so the contents left by the previous call are harmless.
//
// Host code never hands the array's name to a kernel (on the host it is a
// stand-in symbol, not a device address).  The first call on each device,
// with that device current, looks the device address up once with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture begins.
#include <mutex>

namespace gdn {

constexpr size_t kNoallocScratchBytes = size_t{32} << 20;

// +1024 so the workspace can start on a 1024-byte boundary inside the array.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes + 1024];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void *g_noalloc_addr[kMaxDevices] = {};

// Device address of this device's copy of g_noalloc_scratch, looked up once.
int noalloc_scratch_address(void **addr) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return GDN_ERR_DEVICE;
    g_noalloc_addr[dev] = p;
  }
  *addr = g_noalloc_addr[dev];
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_prefill_qk4_v8_d128_k_last_noalloc(
    const void *q, const void *k, const void *v, const float *state, const float *A_log,
    const void *a, const float *dt_bias, const void *b, const int64_t *cu_seqlens,
    int64_t num_seqs, int64_t total_tokens, float scale, void *out, float *final_state,
    void *stream) {
  if (num_seqs < 0 || total_tokens < 0 || total_tokens > (int64_t{1} << 31) ||
      num_seqs > (int64_t{1} << 24))
    return GDN_ERR_BAD_SIZE;
  if (num_seqs == 0) return total_tokens == 0 ? GDN_OK : GDN_ERR_BAD_SIZE;
  // the segmented evaluation when its larger workspace fits the scratch,
  // else the single-pass one
  const bool segments =
      gdn::prefill_workspace_bytes(total_tokens, num_seqs, true) <= gdn::kNoallocScratchBytes;
  if (!segments &&
      gdn::prefill_workspace_bytes(total_tokens, num_seqs, false) > gdn::kNoallocScratchBytes)
    return GDN_ERR_TOO_LARGE;
  if (!cu_seqlens || !A_log || !dt_bias || !final_state) return GDN_ERR_NULL_POINTER;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_NULL_POINTER;
  if ((q && !aligned(q, 16)) || (k && !aligned(k, 16)) || (v && !aligned(v, 16)) ||
      (out && !aligned(out, 16)) || !aligned(final_state, 16) || (state && !aligned(state, 16)) ||
      !aligned(cu_seqlens, 8))
    return GDN_ERR_MISALIGNED;
  const size_t state_bytes = static_cast<size_t>(num_seqs) * gdn::kHV * gdn::kD * gdn::kD * 4;
  if (state && state != final_state && overlap(state, state_bytes, final_state, state_bytes))
    return GDN_ERR_ALIASING;
  if (int st = check_device(nullptr)) return st;
  void *scratch = nullptr;
  if (int st = gdn::noalloc_scratch_address(&scratch)) return st;
  const uintptr_t base = reinterpret_cast<uintptr_t>(scratch);
  void *ws = reinterpret_cast<void *>((base + 1023) & ~uintptr_t{1023});
  if (scale == 0.0f) scale = kDefaultScale;
  cudaError_t err = gdn::launch_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs,
                                        total_tokens, scale, out, final_state, ws, segments,
                                        nullptr, 0, static_cast<cudaStream_t>(stream), nullptr, 0);
  return err == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
