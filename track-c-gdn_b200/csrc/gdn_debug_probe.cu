// gdn_debug_probe.cu -- debug build only (-DGDN_DEBUG_CHECKS): a probe that
// makes the bounded mbarrier wait of the prefill kernels run out, so that
// the give-up path (device status 2, the CTA frees its TMEM and returns, the
// context stays usable) is exercised by a test without faulting or hanging
// anything.  The barrier it waits on has no copy or MMA attached, so giving
// up leaves nothing in flight.
#ifdef GDN_DEBUG_CHECKS

#include "../../include/gdn_b200_debug.h"

namespace gdn {

__device__ int g_probe_result[4];

constexpr int kProbeThreads = 128;
constexpr uint32_t kProbeTmemCols = 32;

__global__ void __launch_bounds__(kProbeThreads, 1) gdn_wait_timeout_probe_kernel() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int broken;
  __shared__ int gave_up;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) tmem_alloc(smem_u32(&tmem_base), kProbeTmemCols);
  if (tid == 0) {
    broken = 0;
    gave_up = 0;
    mbar_init(smem_u32(&bar), 1);  // one arrival expected; none ever comes
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool ok = wait_phase(smem_u32(&bar), 0, reinterpret_cast<volatile int *>(&broken));
  if (!ok) atomicAdd(&gave_up, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kProbeTmemCols);
  }
  __syncthreads();
  if (tid == 0) {
    g_probe_result[0] = ok ? 1 : 0;
    g_probe_result[1] = broken;
    g_probe_result[2] = 1;
    g_probe_result[3] = gave_up;
  }
}

}  // namespace gdn

extern "C" int gdn_b200_debug_wait_timeout_probe(int64_t limit_cycles, int *result, void *stream) {
  if (result == nullptr) return GDN_ERR_NULL_POINTER;
  if (limit_cycles < 1 || limit_cycles > (int64_t{1} << 33)) return GDN_ERR_BAD_SIZE;
  if (int st = check_device(nullptr)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long limit = limit_cycles, restore = 1ll << 33;
  const int zeros[4] = {0, 0, 0, 0};
  if (cudaMemcpyToSymbolAsync(gdn::g_probe_result, zeros, sizeof(zeros), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(gdn::g_wait_limit_cycles, &limit, sizeof(limit), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  gdn::gdn_wait_timeout_probe_kernel<<<1, gdn::kProbeThreads, 0, s>>>();
  const cudaError_t launch = cudaGetLastError();
  // restore the budget whatever happened, then read the result
  if (cudaMemcpyToSymbolAsync(gdn::g_wait_limit_cycles, &restore, sizeof(restore), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess ||
      launch != cudaSuccess ||
      cudaMemcpyFromSymbolAsync(result, gdn::g_probe_result, sizeof(zeros), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  return GDN_OK;
}

#endif  // GDN_DEBUG_CHECKS
