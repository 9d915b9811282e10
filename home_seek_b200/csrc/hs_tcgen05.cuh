// tcgen05 / TMEM helpers (inline PTX, sm_100a): TMEM allocation, UMMA shared
// memory and instruction descriptors, block-scaled MMA, scale-factor copies
// into TMEM, commits and TMEM loads. Descriptor bit layouts follow the PTX ISA
// for tcgen05 (matrix descriptors with version 1, block-scaled instruction
// descriptor) as restated in CUTLASS's cute/arch/mma_sm100_desc.hpp.
#pragma once

#include "hs_common.cuh"

namespace hs {
namespace tc5 {

HS_DI void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
HS_DI void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole warp: allocate ncols TMEM columns, address written to *slot (shared).
HS_DI void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HS_DI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// K-major operand in a 128B-swizzled layout: rows of 128 bytes, 8-row atoms
// 1024 bytes apart (SBO), the tile 1024-byte aligned. Advancing K by 32 bytes
// inside the swizzle atom is a +2 on the start-address field.
HS_DI uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;             // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // stride byte offset: next 8-row atom
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// Source of a 32x128b scale-factor copy: 32 rows of 16 bytes, contiguous
// (no swizzle, 8-row core matrices 128 bytes apart).
HS_DI uint64_t sdesc_sf(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 16;
  d |= static_cast<uint64_t>(128u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled, K-major A and B,
// f32 accumulate implied, UE8M0 scales. a_fmt: 5 = E2M1, 0 = E4M3; b = E4M3.
HS_DI uint32_t idesc_mxf8f6f4(uint32_t a_fmt, uint32_t n, uint32_t a_sf_id, uint32_t b_sf_id) {
  uint32_t d = 0;
  d |= (b_sf_id & 3u) << 4;
  d |= (a_fmt & 7u) << 7;
  d |= 0u << 10;                 // B = E4M3
  d |= ((n >> 3) & 0x3Fu) << 17;
  d |= 1u << 23;                 // scale format UE8M0
  d |= ((128u >> 4) & 0x1Fu) << 24;  // M = 128
  d |= (a_sf_id & 3u) << 29;
  return d;
}

// The same descriptor with the B format given (bits 10-12): 5 = E2M1, 0 = E4M3.
HS_DI uint32_t idesc_mxf8f6f4_ab(uint32_t a_fmt, uint32_t b_fmt, uint32_t n, uint32_t a_sf_id, uint32_t b_sf_id) {
  return idesc_mxf8f6f4(a_fmt, n, a_sf_id, b_sf_id) | ((b_fmt & 7u) << 10);
}

HS_DI void mma_mxf8f6f4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate,
                        uint32_t tsfa, uint32_t tsfb) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// 32 lanes x 128 bits from shared memory, broadcast to the four lane quadrants.
HS_DI void cp_sf_32x128b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Arrive on an mbarrier when every previously issued tcgen05 op of this thread completes.
HS_DI void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Warp loads 32 lanes x 16 consecutive 32-bit columns.
HS_DI void ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
HS_DI void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc5
}  // namespace hs
