// Thin inline-PTX wrappers for the sm_100a features the tensor-core matmul
// uses: mbarriers, 1-D bulk copies (TMA engine, no tensor map), tensor memory
// (allocation, scale-factor copies, loads) and tcgen05 block-scaled MMA.
// Encodings follow the PTX ISA for sm_100a; bitfield layouts of the shared
// memory and instruction descriptors are those the hardware defines (the
// same fields CUTLASS's cute/arch/mma_sm100_desc.hpp names).
#pragma once

#include <cstdint>

namespace msb {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// The bound of every wait, in SM cycles (clock64: monotonic on the SM the
// thread runs on) for a limit given in nanoseconds: 2 cycles per ns, at
// least the limit at SM clocks up to 2 GHz (B200 peaks at 1.965 GHz). The
// global timer is not used: read with an unsigned difference, a timer that
// steps back once ends a wait at once, and a wait must only give up once
// the limit has really passed.
__device__ __forceinline__ long long wait_cycles(long long limit_ns) { return 2 * limit_ns; }

// Waits for the phase of `parity` for at most `limit_ns` nanoseconds (the
// library's wait limit, one second unless msb_set_option changed it); false
// if it gave up. try_wait suspends the thread in hardware between checks, so
// waiting warps take no issue slots.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  long long limit_ns) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long c0 = clock64(), lim = wait_cycles(limit_ns);
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - c0 > lim) return false;
  }
  return true;
}

// Makes this thread's ordinary shared-memory stores visible to the async
// proxy (TMA, tcgen05.cp and the MMA's operand reads) that reads them next.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- bulk copy global -> shared (completes transaction bytes on `bar`) -----
// src and dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- tiled TMA copy global -> shared through a 3-D tensor map ---------------
// Coordinates innermost first. The innermost coordinate counts 8-byte
// elements and is always even here (2 per 16-byte row), so every copy
// starts on a 16-byte boundary.
__device__ __forceinline__ void tma_3d(void *dst, const void *tmap, int c0, int c1, int c2,
                                       uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// ---- tensor memory ------------------------------------------------------------
// Allocation is warp-wide; the TMEM address is written to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Copies 32 rows x 16 bytes of shared memory (described by `desc`) into 4
// TMEM columns of all four 32-lane sub-partitions.
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc)
               : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued before it
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[128 x N] (+)= A[128 x 64] * B[N x 64]^T with e2m1 operands and one e8m0
// scale per 32 elements of K, read from TMEM at sfa / sfb.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// D[128 x N] (+)= A[128 x 16] * B[N x 16]^T with f16 operands from shared
// memory and f32 accumulation in TMEM (kind::f16).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Each thread of a warp reads 32 consecutive columns of its lane
// (lanes 32*(warp%4) .. +31).
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- descriptors ----------------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle: 8-row core matrices
// of 16-byte rows; `sbo` = bytes between 8-row groups, `lbo` = bytes between
// the two 16-byte halves of K. Version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor of kind::mxf4 block-scaled MMA: A and B e2m1
// (format 1), both K-major, e8m0 scales (bit 23), M = 128, given N, dense
// K = 64; the scale-factor byte selectors of A (bits 29-30) and B (4-5).
__host__ __device__ constexpr uint32_t idesc_mxf4(uint32_t n, uint32_t sfa_id, uint32_t sfb_id) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (sfa_id << 29) | (sfb_id << 4);
}

// Instruction descriptor of kind::f16: A and B f16 (format 0), both
// K-major, f32 accumulator (bits 4-5 = 1), M = 128, given N (multiple of 16).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

}  // namespace sm100
}  // namespace msb
