// sm100.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a) features
// the GDN kernels use: tcgen05 MMA with TMEM accumulators, TMEM allocation
// and loads, mbarriers with bounded waits, and UMMA shared-memory /
// instruction descriptors.
//
// Shared-memory operand format used throughout (the canonical "128-byte
// swizzle" UMMA layout): an operand tile is a set of 1024-byte atoms, each
// atom 8 rows x 128 bytes, 1024-byte aligned; inside an atom the 16-byte
// chunk index c of row r is stored at chunk position (c ^ (r & 7)).  One
// physical tile of rows x 64 bf16 can be described to the tensor core either
//   K-major : rows = M/N index, the 64 bf16 of a row = K index;
//             SBO = 1024 (next 8 rows), LBO unused; a K=16 step is +32 bytes
//   MN-major: rows = K index, the 64 bf16 of a row = M/N index;
//             SBO = byte distance between 8-row (K) groups,
//             LBO = byte distance between 64-wide M/N groups.
#pragma once
#include <cstdint>

namespace gdn {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- UMMA descriptors -----------------------------------------------------

// Shared-memory matrix descriptor (64 bit):
//   [0,14)  start address >> 4      [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4 [46,48) version = 1 (sm_100)
//   [49,52) base offset = 0 (atoms are 1024-byte aligned)
//   [61,64) layout: 2 = 128-byte swizzle
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Shared-memory matrix descriptor for the canonical no-swizzle K-major
// layout: the operand is a grid of core matrices of 8 rows x 16 bytes (8
// bf16 of K), each 128 contiguous bytes; lbo_bytes = distance between core
// matrices adjacent in K, sbo_bytes = between core matrices adjacent in M/N.
// [61,64) layout = 0 (no swizzle).
__device__ __forceinline__ uint64_t umma_desc_noswz(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

// The descriptor of the operand `bytes` further on in shared memory (bytes a
// multiple of 16): shared-memory addresses stay below 2^18, so the 14-bit
// start-address field (address >> 4) never carries and the offset adds
// directly -- one add per MMA instead of rebuilding the descriptor.
__device__ __forceinline__ uint64_t umma_desc_advance(uint64_t desc, uint32_t bytes) {
  return desc + (bytes >> 4);
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation:
//   [4,6) D format = 1 (f32)   [7,10) A format = 1 (bf16)  [10,13) B format = 1
//   [15] A major (1 = MN)      [16] B major (1 = MN)
//   [17,23) N >> 3             [24,29) M >> 4
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((static_cast<uint32_t>(N) >> 3) << 17) |
         ((static_cast<uint32_t>(M) >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T-in-UMMA-convention, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with the A operand in TMEM (M rows on lanes, two bf16 per 32-bit
// column: a K=16 step spans 8 columns).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :
      : "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `mbar` when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint32_t mbar_saddr) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      :
      : "r"(mbar_saddr)
      : "memory");
}

// ---- fences ---------------------------------------------------------------

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor core operand reads).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMEM -----------------------------------------------------------------

// Warp-collective: allocate `ncols` (power of two >= 32) TMEM columns and
// write the base address to shared memory at `dst_saddr`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_saddr, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :
               : "r"(dst_saddr), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Warp-collective.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               :
               : "r"(taddr), "r"(ncols)
               : "memory");
}

// Warp-collective: lane l of this warp receives 32 consecutive fp32 columns
// of TMEM lane (lane base of taddr) + l.  Call tmem_wait_ld() before use.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]),
        "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]),
        "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]),
        "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]),
        "=r"(u[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Warp-collective: lane l writes 32 consecutive 32-bit columns of TMEM lane
// (lane base of taddr) + l.  Call tmem_wait_st() before the data is consumed.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&u)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      :
      : "r"(taddr), "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]),
        "r"(u[6]), "r"(u[7]), "r"(u[8]), "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]),
        "r"(u[13]), "r"(u[14]), "r"(u[15]), "r"(u[16]), "r"(u[17]), "r"(u[18]), "r"(u[19]),
        "r"(u[20]), "r"(u[21]), "r"(u[22]), "r"(u[23]), "r"(u[24]), "r"(u[25]), "r"(u[26]),
        "r"(u[27]), "r"(u[28]), "r"(u[29]), "r"(u[30]), "r"(u[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      :
      : "r"(taddr), "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]),
        "r"(u[6]), "r"(u[7]), "r"(u[8]), "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]),
        "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&u)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
               :
               : "r"(taddr), "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]),
                 "r"(u[6]), "r"(u[7])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Warp-collective: lane l receives 8 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&r)[8]) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]),
                 "=r"(u[6]), "=r"(u[7])
               : "r"(taddr));
}

// Warp-collective: lane l receives 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]),
        "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(taddr));
}

// ---- TMA / bulk copies (no multicast) ---------------------------------------

// Expect `bytes` of asynchronous transactions on `mbar` and arrive once.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :
               : "r"(mbar), "r"(bytes)
               : "memory");
}

// 2D tiled TMA load of one box at coordinates (x = inner, y = outer).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int x, int y,
                                            uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];"
      :
      : "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// 2D tiled TMA store of one box from shared memory to this GPU's global
// memory, tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_store_2d(const void *tmap, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               :
               : "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until this thread's committed bulk stores have read their shared-memory
// source (the buffer may be rewritten) ...
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// ... or have completed (their writes are done).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---- thread-block clusters: rank, distributed shared memory, barrier ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of shared::cta address `saddr` in CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Asynchronous 16-byte store into the shared memory of a CTA of the cluster
// (`caddr`); its completion counts 16 transaction bytes on that CTA's
// mbarrier `cmbar` (both shared::cluster addresses in the same CTA).
__device__ __forceinline__ void dsmem_st_async_v4(uint32_t caddr, float4 v, uint32_t cmbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(caddr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cmbar)
      : "memory");
}
// Arrive (release at cluster scope) on the mbarrier at shared::cluster address
// `caddr`, which may belong to another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}
// Every thread of every CTA of the cluster arrives (release) / waits for all
// of them (acquire); warp-uniform.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Contiguous global -> shared bulk copy (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :
      : "r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(mbar)
      : "memory");
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t saddr, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" : : "r"(saddr), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t saddr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with acquire at cluster scope: for phases completed by another CTA
// of the cluster (a remote arrive or remote asynchronous stores).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t saddr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false if it did not complete within `max_iters` polls (each poll may
// itself suspend for a hardware-defined interval).
__device__ __forceinline__ bool mbar_wait(uint32_t saddr, uint32_t parity,
                                          uint32_t max_iters = (1u << 24)) {
  for (uint32_t i = 0; i < max_iters; ++i) {
    if (mbar_try_wait(saddr, parity)) return true;
  }
  return false;
}

}  // namespace sm100
}  // namespace gdn
