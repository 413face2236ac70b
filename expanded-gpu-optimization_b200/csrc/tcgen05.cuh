// Thin inline-PTX wrappers for the sm_100a tensor-core path: TMEM allocation, tcgen05.mma
// issue (kind::f16 and kind::tf32, A from tensor or shared memory, B from shared memory),
// commits, TMEM loads/stores, fences and the shared-memory matrix / instruction descriptors.
//
// Descriptor encodings follow the PTX ISA's tcgen05 "shared memory descriptor" and
// "instruction descriptor" tables (the same bit positions CUTLASS's
// cute/arch/mma_sm100_desc.hpp spells out).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace fhb {
namespace tc {

// ---- TMEM allocation (one full warp) ----
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}

// ---- ordering between tcgen05 operations and thread synchronisation ----
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- MMA issue: one elected lane of a converged warp issues the MMAs ----
// The 12 MMAs of one 3xFP16 chunk (K = 16), issued by one elected lane of a converged warp in
// one block: for each jet component c, D_c (+)= A_hi B_hi, then += A_lo B_hi and A_hi B_lo,
// with D_c at TMEM column d0 + 64c, A_hi at a0 + 16c and A_lo 8 columns on. The first MMA of
// each component accumulates only if `accumulate`; the others always do. The components are
// interleaved (the A_hi B_hi of all four, then A_lo B_hi, then A_hi B_lo), so consecutive
// MMAs write different accumulators; each D_c still takes its three products in the same
// order.
__device__ __forceinline__ void mma_f16_ts_chunk_warp(uint32_t d0, uint32_t a0, uint64_t b_hi,
                                                      uint64_t b_lo, uint32_t idesc,
                                                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, pa, pt;\n\t"
      ".reg .b32 d1, d2, d3, h1, h2, h3, l0, l1, l2, l3;\n\t"
      "setp.ne.b32 pa, %5, 0;\n\t"
      "setp.ne.b32 pt, %6, 0;\n\t"
      "add.u32 d1, %0, 64;\n\tadd.u32 d2, %0, 128;\n\tadd.u32 d3, %0, 192;\n\t"
      "add.u32 h1, %1, 16;\n\tadd.u32 h2, %1, 32;\n\tadd.u32 h3, %1, 48;\n\t"
      "add.u32 l0, %1, 8;\n\tadd.u32 l1, %1, 24;\n\tadd.u32 l2, %1, 40;\n\t"
      "add.u32 l3, %1, 56;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [h1], %2, %4, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d2], [h2], %2, %4, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d3], [h3], %2, %4, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [l0], %2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [l1], %2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d2], [l2], %2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d3], [l3], %2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [h1], %3, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d2], [h2], %3, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [d3], [h3], %3, %4, pt;\n\t}"
      ::"r"(d0), "r"(a0), "l"(b_hi), "l"(b_lo), "r"(idesc), "r"(accumulate), "r"(1u)
      : "memory");
}

// The 24 MMAs of one 3xTF32 chunk (two K steps of 8), issued the same way: K step kk uses
// B descriptors b_hi[kk], b_lo[kk]; component c's A_hi block of step kk at a0 + 32c + 8kk and
// its A_lo block 16 columns on; D_c at d0 + 64c. The first MMA of each component in K step 0
// accumulates only if `accumulate`. Components interleaved as in the f16 chunk.
__device__ __forceinline__ void mma_tf32_ts_chunk_warp(uint32_t d0, uint32_t a0, uint64_t bh0,
                                                       uint64_t bl0, uint64_t bh1, uint64_t bl1,
                                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, pa, pt;\n\t"
      ".reg .b32 d1, d2, d3, x0, x1, x2, x3, x4, x5, x6, x7, y0, y1, y2, y3, y4, y5, y6, y7;\n\t"
      "setp.ne.b32 pa, %7, 0;\n\t"
      "setp.ne.b32 pt, %8, 0;\n\t"
      "add.u32 d1, %0, 64;\n\tadd.u32 d2, %0, 128;\n\tadd.u32 d3, %0, 192;\n\t"
      // x: A_hi blocks (c, kk) at 32c + 8kk; y: A_lo blocks 16 columns on
      "add.u32 x0, %1, 0;\n\tadd.u32 x1, %1, 8;\n\tadd.u32 x2, %1, 32;\n\tadd.u32 x3, %1, 40;\n\t"
      "add.u32 x4, %1, 64;\n\tadd.u32 x5, %1, 72;\n\tadd.u32 x6, %1, 96;\n\tadd.u32 x7, %1, 104;\n\t"
      "add.u32 y0, %1, 16;\n\tadd.u32 y1, %1, 24;\n\tadd.u32 y2, %1, 48;\n\tadd.u32 y3, %1, 56;\n\t"
      "add.u32 y4, %1, 80;\n\tadd.u32 y5, %1, 88;\n\tadd.u32 y6, %1, 112;\n\tadd.u32 y7, %1, 120;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [x0], %2, %6, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [x2], %2, %6, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [x4], %2, %6, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [x6], %2, %6, pa;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [y0], %2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [y2], %2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [y4], %2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [y6], %2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [x0], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [x2], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [x4], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [x6], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [x1], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [x3], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [x5], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [x7], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [y1], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [y3], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [y5], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [y7], %4, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [x1], %5, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d1], [x3], %5, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d2], [x5], %5, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [d3], [x7], %5, %6, pt;\n\t}"
      ::"r"(d0), "r"(a0), "l"(bh0), "l"(bl0), "l"(bh1), "l"(bl1), "r"(idesc), "r"(accumulate),
        "r"(1u)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (both f16, D f32), issued by a converged warp;
// the operand majors (K or MN) are in the instruction descriptor.
__device__ __forceinline__ void mma_f16_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// tcgen05.commit from one elected lane of a converged warp.
__device__ __forceinline__ void commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
      ::"r"(smem_u32(bar))
      : "memory");
}


// ---- TMEM <-> registers (32 lanes x 32-bit, one lane per thread of the warp) ----
__device__ __forceinline__ void ld_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void ld_x4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st_x2(uint32_t taddr, uint32_t a, uint32_t b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(a),
               "r"(b)
               : "memory");
}
__device__ __forceinline__ void st_x4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c,
                                      uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Round to TF32 (nearest, ties away from zero): the 32-bit pattern with the low 13 mantissa
// bits zero. Done on the bit pattern -- add half a TF32 ulp (bit 12; a carry moves into the
// exponent, as rounding up to the next binade requires), then clear bits 0..12 -- in two
// integer instructions; the same result as cvt.rna.tf32.f32 for every finite input and for
// infinities (tests/test_scale_math.py checks the rounding on the CPU). The kernels never
// split a NaN.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

// 3xTF32 split: hi = x rounded to TF32; lo = x - hi (exact in FP32), fed as is: the tensor
// core reads only its TF32 bits of lo, an error of at most 2^-21 |x|.
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = to_tf32(x);
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// Shared-memory matrix descriptor, K-major, no swizzle ("interleave" canonical layout):
// core matrices of 8 rows x 16 bytes stored contiguously; `lbo` = byte distance between
// the two 16-byte K halves of one 8-element (32-byte) K step, `sbo` = byte distance
// between consecutive 8-row groups. Version field = 1 (sm_100), base offset 0.
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t smem_addr, uint32_t lbo,
                                                     uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  // base_offset = 0, lbo mode = 0, layout type (bits 61..63) = 0: no swizzle
  return d;
}


// Instruction descriptor for kind::tf32: D f32, A/B tf32, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (2u << 7)                                // A format: tf32
         | (2u << 10)                               // B format: tf32
         | (0u << 15) | (0u << 16)                  // A, B K-major
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Instruction-descriptor bits selecting MN-major A (bit 15) and B (bit 16) operands.
constexpr uint32_t kIdescAMnMajor = 1u << 15, kIdescBMnMajor = 1u << 16;

// Instruction descriptor for kind::f16 with f16 A and B (format 0), D f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (0u << 7)                                // A format: f16
         | (0u << 10)                               // B format: f16
         | (0u << 15) | (0u << 16)                  // A, B K-major
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

}  // namespace tc

// The epilogues' accumulator-column order: the B operand's row (accumulator column within a
// component) k = 16s + 4a + t holds neuron 16a + 4s + t, so the 16 neurons an epilogue warp
// of block s owns (chunks a = 0..3, four neurons each) sit in 16 consecutive columns -- one
// tcgen05.ld.x16 per component. The map is its own inverse.
__host__ __device__ constexpr int neuron_of_column(int k) {
  return (k & 3) | (((k >> 4) & 3) << 2) | (((k >> 2) & 3) << 4);
}
static_assert(neuron_of_column(neuron_of_column(37)) == 37 && neuron_of_column(16) == 4,
              "column permutation");

}  // namespace fhb
