// tcgen05 (5th-generation tensor core) helpers for sm_100a, hand-written PTX.
//
// Conventions validated on B200 by a known-answer test of
// tcgen05.mma.kind::mxf8f6f4.block_scale (A = e2m1 weights, B = e4m3,
// ue8m0 block scales, f32 accumulate):
//   * operands in shared memory, K-major, 128-byte swizzle: 8-row atoms of
//     1024 B, rows of 128 B; descriptor LBO = 16 B (unused), SBO = 1024 B,
//     version 1, layout type 2; a K step of 32 elements advances the start
//     address by 32 B inside the atom;
//   * FP4 operands are fetched with TMA data type 16U4_ALIGN16B (16 codes
//     occupy 16 bytes of shared memory: 8 bytes of codes, 8-byte gap); the
//     mbarrier transaction count is the number of PACKED bytes;
//   * scale factors live in tensor memory in the 128-row x 4-block "atom":
//     lane 32w + r, column 4a + j holds the four ue8m0 bytes (blocks 4a..4a+3)
//     of row r + 32j; the instruction descriptor's sf_id selects the block
//     inside the 32-bit word;
//   * the accumulator of an M = 128 MMA: row m in lane m, column n in column n.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace ds {
namespace tc5 {

using ds::ptx::smem_u32;

// Shared-memory matrix descriptor: K-major, 128-byte swizzle.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;   // leading byte offset (16 B units; unused when swizzled)
  d |= (uint64_t)64 << 32;  // stride byte offset: 1024 B between 8-row atoms
  d |= (uint64_t)1 << 46;   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;   // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled, M = 128, A = E2M1,
// B = E4M3, ue8m0 scales, K = 32; sf_id picks the scale byte for this K step.
__device__ __forceinline__ uint32_t idesc_e2m1_e4m3(int n, uint32_t sf_id) {
  return (sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | (8u << 24) |
         (sf_id << 29);
}

// Same, A = B = E4M3 (MXFP8).
__device__ __forceinline__ uint32_t idesc_e4m3_e4m3(int n, uint32_t sf_id) {
  return (sf_id << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | (8u << 24) |
         (sf_id << 29);
}

__device__ __forceinline__ void mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Instruction descriptor, kind::mxf4 block-scaled (scale_vec::2X), M = 128,
// A = B = E2M1, ue8m0 scales, K = 64; sf_id (0 or 2) picks the byte pair of
// the 4-block scale word that this K step uses.
__device__ __forceinline__ uint32_t idesc_mxf4(int n, uint32_t sf_id) {
  return (sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | (8u << 24) | (sf_id << 29);
}

// D (+)= A * B, both packed e2m1 (two codes per byte, K-major, 128-byte swizzle), K = 64.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// f32 pair -> e2m1 pair (round to nearest even, saturating to +-6): lo in
// bits 0..3, hi in bits 4..7.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.u32.u8 %0, t; }" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ue8m0 byte of the block scale that maps a block maximum `amax` into
// (3, 6], the top of the e2m1 range: 2^(E-2) when the maximum's mantissa is
// <= 1.5, else 2^(E-1) (E its exponent); zero blocks get scale 1.
__device__ __forceinline__ int e2m1_block_scale(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int ef = (int)(b >> 23);
  if (ef == 0) return 127;
  const int s = (b & 0x7FFFFFu) <= 0x400000u ? ef - 2 : ef - 1;
  return min(max(s, 1), 253);
}

// e2m1 pair (bits 0..7) -> two f32 (exact).
__device__ __forceinline__ void e2m1x2_to_f32x2(uint32_t b, float& lo, float& hi) {
  uint32_t h2;
  asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(h2) : "r"(b));
  lo = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
  hi = __half2float(__ushort_as_half((uint16_t)(h2 >> 16)));
}

// Instruction descriptor, kind::f16 with bf16 A and B, f32 accumulate, M = 128.
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (8u << 24);
}

// D (+)= A * B, bf16 operands in shared memory (K = 16 per instruction).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole-warp tensor-memory allocation; the base address is written to *dst.
__device__ __forceinline__ void alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// Lane-quarter address: warp w may only touch lanes 32*(w % 4) .. +31.
__device__ __forceinline__ uint32_t lane_quarter(uint32_t taddr, int warp) {
  return taddr + ((uint32_t)((warp & 3) * 32) << 16);
}

__device__ __forceinline__ void st_x4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void ld_x4(uint32_t taddr, float (&v)[4]) {
  uint32_t r0, r1, r2, r3;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}

// 16 consecutive accumulator columns of this warp's 32 lanes (no wait).
__device__ __forceinline__ void ld_x16_nowait(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Offset of byte k of row r (0..7) inside a K-major SW128 operand tile whose
// 128-byte K chunks are 8-row atoms of 1024 B.
__device__ __forceinline__ uint32_t b_tile_off(int r, int k) {
  return (uint32_t)((k >> 7) * 1024 + r * 128 + ((((k >> 4) & 7) ^ r) << 4) + (k & 15));
}

// f32 -> e4m3 (round to nearest even, saturating to +-448).
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return (uint8_t)(r & 0xFFu);
}

// Two f32 -> two e4m3 bytes: lo in bits 0..7, hi in bits 8..15.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two e4m3 bytes (bits 0..15) -> two f32 (exact).
__device__ __forceinline__ void e4m3x2_to_f32x2(uint32_t b, float& lo, float& hi) {
  uint32_t h2;
  asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(h2) : "r"(b));
  lo = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
  hi = __half2float(__ushort_as_half((uint16_t)(h2 >> 16)));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  uint32_t h2;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(h2) : "h"((uint16_t)b));
  return __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
}

}  // namespace tc5
}  // namespace ds
