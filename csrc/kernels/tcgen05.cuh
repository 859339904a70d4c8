// Blackwell (sm_100a) 5th-generation tensor-core helpers: TMEM allocation,
// UMMA shared-memory / instruction descriptors, block-scaled MMA issue,
// scale-factor copies into TMEM, accumulator loads, mbarrier helpers.
//
// Descriptor bit layouts follow the PTX ISA for tcgen05 (matching CUTLASS's
// cute::UMMA::SmemDescriptor / InstrDescriptorBlockScaled):
//   SMEM descriptor: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4,
//                    [46,48) version (1 on sm_100), [61,64) layout (0 = no swizzle).
//   K-major, no swizzle: core matrices of 8 rows x 16 bytes (128 B contiguous);
//   LBO = byte distance between the two 16-byte K halves of one MMA-K (32 B),
//   SBO = byte distance between consecutive 8-row groups.
//   Block-scaled instruction descriptor: [4,6) B scale-factor id, [7,10) A fmt,
//   [10,13) B fmt, [15] A major, [16] B major, [17,23) N>>3, [23] scale fmt
//   (1 = UE8M0), [24,29) M>>4, [29,31) A scale-factor id.
//   Scale factors (UE8M0, one per 32 K) live in TMEM: a 512-byte SMEM atom holds
//   128 rows x 4 k-blocks at byte (m % 32) * 16 + (m / 32) * 4 + kb and is copied
//   with tcgen05.cp 32x128b.warpx4 into 4 TMEM columns; the MMA's scale-factor id
//   selects the k-block byte.
#pragma once
#include "common.cuh"

namespace moet {
namespace tc {

MOET_DEVICE uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MOET_DEVICE uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;            // version 1 (sm_100)
  return d;                          // base offset 0, lbo mode 0, layout 0 (no swizzle)
}

// kind::mxf8f6f4 block-scaled, e4m3 x e4m3, UE8M0 scales, K-major A and B.
MOET_DEVICE uint32_t idesc_mxf8(int M, int N, int a_sf_id, int b_sf_id) {
  uint32_t d = 0;
  d |= (uint32_t)(b_sf_id & 3) << 4;
  d |= 0u << 7;                      // A = E4M3
  d |= 0u << 10;                     // B = E4M3
  d |= (uint32_t)((N >> 3) & 0x3F) << 17;
  d |= 1u << 23;                     // scale format UE8M0
  d |= (uint32_t)((M >> 4) & 0x1F) << 24;
  d |= (uint32_t)(a_sf_id & 3) << 29;
  return d;
}

MOET_DEVICE void mma_mxf8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate,
                          uint32_t tsfa, uint32_t tsfb) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

MOET_DEVICE void cp_sf_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc));
}

MOET_DEVICE void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_addr(mbar)) : "memory");
}

MOET_DEVICE void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOET_DEVICE void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
MOET_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Whole warp: allocate ncols TMEM columns (power of two >= 32); address written to *dst (smem).
MOET_DEVICE void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols));
}
MOET_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
MOET_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// Warp loads 8 consecutive 32-bit columns of its 32 TMEM lanes (lane quarter = warp % 4).
MOET_DEVICE void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
MOET_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

MOET_DEVICE void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
MOET_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait (about a second at most); false on timeout.
MOET_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t it = 0; it < (1u << 22); it++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Byte offset of element (r, k) in a K-major no-swizzle operand tile whose
// rows are `kbytes` long: 8-row groups of core matrices, 16-byte K slices.
MOET_DEVICE uint32_t kmajor_off(int r, int k, int kbytes) {
  return (uint32_t)((r >> 3) * (kbytes / 16) * 128 + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}
// Byte offset of scale factor (row r < 128, k-block kb) inside 512-byte atoms (one per 4 k-blocks).
MOET_DEVICE uint32_t sf_off(int r, int kb) {
  return (uint32_t)((kb >> 2) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (kb & 3));
}

}  // namespace tc
}  // namespace moet
