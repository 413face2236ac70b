// Shared device helpers for the fused forward-Laplacian kernels (sm_100a).
//
// Parameter ABI: the packed 12,737-float buffer of the reference (csrc/mlp_abi.cuh:8-17,
// src/fused_hoad/parameters.py:28-48): per linear layer W[out][in] row-major, then b[out],
// for the layers 2->64, 64->64 (x3), 64->1. Kept bit-identical so buffers packed by the
// reference's Python API drop straight in.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fused_hoad_b200.h"

namespace fhb {

constexpr int kIn = 2;
constexpr int kWidth = 64;
constexpr int kHiddenGemms = 3;                                // layers 1..3 are 64x64
constexpr int kB0 = kWidth * kIn;                              // 128
constexpr int kHiddenBase = kB0 + kWidth;                      // 192
constexpr int kHiddenStride = kWidth * kWidth + kWidth;        // 4160
constexpr int kOutBase = kHiddenBase + kHiddenGemms * kHiddenStride;  // 12672
constexpr int kParamCount = kOutBase + kWidth + 1;             // 12737
static_assert(kParamCount == 12737, "parameter ABI drifted");
// Parameters staged in shared memory: 12,736 floats by one bulk copy (50,944 B, a multiple
// of 16) plus b_out by a plain load; padded to a 16-byte multiple.
constexpr int kParamBulkFloats = 12736;
constexpr int kParamSmemFloats = 12740;

// Bounded waits: a wait that has not completed after this many nanoseconds gives up, sets
// a bit in the caller's status word and lets the kernel return instead of hanging.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_status(unsigned int* status, unsigned int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---- programmatic dependent launch ----
// A kernel launched with launch_dependent() may start while the kernel before it in the
// stream still runs, as soon as every CTA of that kernel has called allow_dependents() (or
// exited). Until it calls wait_for_prerequisites() it may read only what was complete before
// that earlier kernel started; after the call, everything the earlier kernel wrote is
// visible (generic and bulk-copy reads alike). Both are no-ops for an ordinary launch.
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_for_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- mbarrier + bulk copy (non-multicast) ----

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread may stay suspended until the phase
// completes or about hint_ns nanoseconds pass, instead of the shorter system-dependent
// limit of the plain form, so a warp that has to wait re-polls -- and issues the loop's
// instructions -- rarely. Completion still wakes it at once.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_for(uint64_t* bar, uint32_t phase,
                                                  uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Wait for `phase` of `bar` to complete, giving up after kWaitLimitNs. Returns false on
// timeout (and records `bits` in *status).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase,
                                                  unsigned int* status, unsigned int bits) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_for(bar, phase, kSuspendHintNs)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) {
      report_status(status, bits);
      return false;
    }
  }
}

// Plain arrival (no transaction count) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One bulk (TMA, non-multicast) copy global -> this CTA's shared memory, completing on bar.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Stage the whole packed parameter buffer into shared memory, once per CTA. When the
// buffer is 16-byte aligned one thread issues a single bulk copy; otherwise the CTA copies
// it with plain loads. Ends with __syncthreads(). Returns false if the copy timed out.
__device__ __forceinline__ bool stage_parameters(float* sp, const float* __restrict__ params,
                                                 uint64_t* bar, bool aligned,
                                                 unsigned int* status) {
  bool ok = true;
  if (aligned) {
    if (threadIdx.x == 0) {
      mbar_init(bar, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(bar, kParamBulkFloats * 4);
      bulk_copy_g2s(sp, params, kParamBulkFloats * 4, bar);
    }
    if (threadIdx.x == 32) {
      for (int k = kParamBulkFloats; k < kParamCount; ++k) sp[k] = params[k];
    }
    __syncthreads();  // barrier initialised before anyone waits on it
    ok = mbar_wait_bounded(bar, 0, status, FHB_STATUS_STAGE_TIMEOUT);
  } else {
    for (int k = threadIdx.x; k < kParamCount; k += blockDim.x) sp[k] = params[k];
  }
  __syncthreads();
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// The largest power of 2 <= 2^c / y, y = max(x, 1e-30), clamped to [2^-126, 2^127], from the
// exponent and mantissa bits alone: for y = m 2^e (m in [1, 2)) the quotient is 2^(c-e) when
// m = 1 and lies in (2^(c-e-1), 2^(c-e)) otherwise (a correctly rounded division never reaches
// 2^(c-e) then, so this equals flooring the divided value; an infinite y divides to 0 and
// clamps to 2^-126). tests/test_scale_math.py checks the equality over the float32 range.
__device__ __forceinline__ float pow2_floor_ratio(int c, float x) {
  const uint32_t b = __float_as_uint(fmaxf(x, 1e-30f));
  int k = c - (static_cast<int>(b >> 23) - 127) - ((b & 0x7FFFFFu) != 0u ? 1 : 0);
  if (b >= 0x7F800000u) k = -126;  // an overflowed (infinite) bound: the quotient is 0
  k = min(max(k, -126), 127);
  return __uint_as_float(static_cast<uint32_t>(k + 127) << 23);
}

// Two FP32 fmas in one instruction (fma.rn.f32x2, sm_100a): d0 = a0 b0 + d0, d1 = a1 b1 + d1,
// each rounded exactly as fmaf. The FP32 pipe's rate is the same as two scalar fmas; the
// packed form halves the issue slots they take.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0,
                                     float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Two FP32 products in one instruction (mul.rn.f32x2): d0 *= a0, d1 *= a1, rounded as a
// scalar multiply.
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1) {
  asm("{\n\t.reg .b64 ra, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rd, {%0, %1};\n\t"
      "mul.rn.f32x2 rd, rd, ra;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}

// max(a, b, c) in one instruction (the three-input form of max.f32 on sm_100a); as fmaxf, a
// NaN input is ignored when another input is a number.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum over the warp of a non-negative float (non-negative floats order as their bit
// patterns): one redux instruction.
__device__ __forceinline__ float warp_max_nonneg(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}

// 1 / x for a positive power of 2 x: exact, from the exponent field, when the result is a
// normal float; otherwise the division (1 / inf = 0, 1 / 2^127 is subnormal).
__device__ __forceinline__ float inv_pow2(float x) {
  const uint32_t e = __float_as_uint(x) >> 23;
  return (e >= 1u && e <= 253u) ? __uint_as_float((254u - e) << 23) : 1.0f / x;
}

// f16 operand pairs: hi = x rounded to f16 (11 significant bits), lo = x - hi
// rounded to f16, element a (even K) in the low halves. x - hi is exact in FP32 and comes
// from one mixed-precision fma (f16 hi times -1 plus the FP32 x), so a pair costs four
// instructions: two packs and two fmas. Inside the scaled range (|x| <= 2^14) hi is a normal
// f16; values below 2^-14 lose precision, at most 2^-25 absolute in scaled units.
__device__ __forceinline__ void split_f16_pair_fast(float a, float b, uint32_t& hi,
                                                    uint32_t& lo) {
  asm("{\n\t.reg .b16 h0, h1, m;\n\t.reg .f32 la, lb;\n\t"
      "cvt.rn.f16x2.f32 %0, %3, %2;\n\t"
      "mov.b32 {h0, h1}, %0;\n\t"
      "mov.b16 m, 0xBC00;\n\t"
      "fma.rn.f32.f16 la, h0, m, %2;\n\t"
      "fma.rn.f32.f16 lb, h1, m, %3;\n\t"
      "cvt.rn.f16x2.f32 %1, lb, la;\n\t}"
      : "=r"(hi), "=r"(lo)
      : "f"(a), "f"(b));
}

// ---- the tanh jet and its adjoint ----
//
// Forward (reference csrc/fused_residual.cu:16-23): a = tanh(z_v), s = 1 - a^2,
//   v = a, J_d = s z_Jd, L = s z_L - 2 a s (z_J0^2 + z_J1^2).
__device__ __forceinline__ void tanh_jet(float zv, float zj0, float zj1, float zl, float& v,
                                         float& j0, float& j1, float& l) {
  const float a = tanhf(zv);
  const float s = fmaf(-a, a, 1.0f);
  const float q = fmaf(zj0, zj0, zj1 * zj1);
  v = a;
  j0 = s * zj0;
  j1 = s * zj1;
  l = fmaf(s, zl, -2.0f * a * s * q);
}

// Adjoint (reference csrc/fused_backward.cu:29-33): with s2 = -2 a s, s3 = -2 s^2 + 4 a^2 s,
// q = z_J0^2 + z_J1^2, maps (vbar, J0bar, J1bar, Lbar) in place to
//   zbar_v = vbar s + (Jbar . z_J) s2 + Lbar (z_L s2 + q s3)
//   zbar_Jd = Jbar_d s + 2 Lbar s2 z_Jd,   zbar_L = Lbar s.
__device__ __forceinline__ void tanh_jet_adjoint(float zv, float zj0, float zj1, float zl,
                                                 float& av, float& aj0, float& aj1, float& al) {
  const float a = tanhf(zv);
  const float s = fmaf(-a, a, 1.0f);
  const float s2 = -2.0f * a * s;
  const float s3 = fmaf(-2.0f * s, s, 4.0f * a * a * s);
  const float q = fmaf(zj0, zj0, zj1 * zj1);
  const float gv = av * s + fmaf(aj0, zj0, aj1 * zj1) * s2 + al * fmaf(zl, s2, q * s3);
  const float l2 = 2.0f * al * s2;
  const float g0 = fmaf(aj0, s, l2 * zj0);
  const float g1 = fmaf(aj1, s, l2 * zj1);
  av = gv;
  aj0 = g0;
  aj1 = g1;
  al = al * s;
}

// tanh from the identity tanh(x) = 1 - 2 / (exp(2x) + 1), with exp(2x) = 2^(2 log2(e) x)
// on the special-function unit (ex2.approx) and the reciprocal on the same unit
// (rcp.approx): 5 instructions. Absolute error is a few 1e-7 for every x (relative error
// grows as |x| -> 0, where tanh(x) ~ x, but the jet propagates absolute errors only); for
// large |x| the formula saturates to exactly +-1, and NaN stays NaN. Used by the tensor-core
// forward, whose 3xTF32 GEMMs carry errors of the same size; the GPU tests bound it against
// CUDA's tanhf over a dense sweep.
__device__ __forceinline__ float tanh_fast(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * 2.8853900817779268f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(e + 1.0f));
  return fmaf(-2.0f, r, 1.0f);
}

// tanh_jet with tanh_fast.
__device__ __forceinline__ void tanh_jet_fast(float zv, float zj0, float zj1, float zl, float& v,
                                              float& j0, float& j1, float& l) {
  const float a = tanh_fast(zv);
  const float s = fmaf(-a, a, 1.0f);
  const float q = fmaf(zj0, zj0, zj1 * zj1);
  v = a;
  j0 = s * zj0;
  j1 = s * zj1;
  l = fmaf(s, zl, -2.0f * a * s * q);
}

// ---- packed FP32 pair arithmetic (sm_100a .f32x2): each lane rounded as the scalar op ----
// r = a * b
__device__ __forceinline__ void mul2o(float& r0, float& r1, float a0, float a1, float b0,
                                      float b1) {
  asm("{\n\t.reg .b64 ra, rb, rr;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rr, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rr;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// r = a + b
__device__ __forceinline__ void add2o(float& r0, float& r1, float a0, float a1, float b0,
                                      float b1) {
  asm("{\n\t.reg .b64 ra, rb, rr;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rr, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rr;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// r = a * b + c
__device__ __forceinline__ void fma2o(float& r0, float& r1, float a0, float a1, float b0,
                                      float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rr;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rr, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rr;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// tanh_jet_fast of two neurons in packed pair arithmetic: bitwise the results of two
// tanh_jet_fast calls (the same operations in the same order; -a from 2r - 1, exact).
__device__ __forceinline__ void tanh_jet_fast2(float zv0, float zv1, float zj00, float zj01,
                                               float zj10, float zj11, float zl0, float zl1,
                                               float& v0, float& v1, float& j00, float& j01,
                                               float& j10, float& j11, float& l0, float& l1) {
  constexpr float k = 2.8853900817779268f;
  float x0, x1, e0, e1, p0, p1, r0, r1, a0, a1, n0, n1, s0, s1, t0, t1, q0, q1, m0, m1;
  mul2o(x0, x1, zv0, zv1, k, k);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(x0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(x1));
  add2o(p0, p1, e0, e1, 1.0f, 1.0f);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(p0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(p1));
  fma2o(a0, a1, -2.0f, -2.0f, r0, r1, 1.0f, 1.0f);    // a = 1 - 2r
  fma2o(n0, n1, 2.0f, 2.0f, r0, r1, -1.0f, -1.0f);    // -a
  fma2o(s0, s1, n0, n1, a0, a1, 1.0f, 1.0f);          // s = 1 - a^2
  mul2o(t0, t1, zj10, zj11, zj10, zj11);
  fma2o(q0, q1, zj00, zj01, zj00, zj01, t0, t1);      // |z_J|^2
  v0 = a0;
  v1 = a1;
  mul2o(j00, j01, s0, s1, zj00, zj01);
  mul2o(j10, j11, s0, s1, zj10, zj11);
  mul2o(m0, m1, -2.0f, -2.0f, a0, a1);
  mul2o(m0, m1, m0, m1, s0, s1);
  mul2o(m0, m1, m0, m1, q0, q1);
  fma2o(l0, l1, s0, s1, zl0, zl1, m0, m1);
}

// ---- the SiLU jet and its adjoint ----
//
// Reference src/fused_hoad/backends/forward_laplacian.py:34-38 (_silu_jet) with :60-67: for
// phi(z) = z sigma(z), p = sigma (1 - sigma),
//   phi' = sigma + z p,   phi'' = p (2 + z (1 - 2 sigma)),
//   phi''' = p ((1 - 2 sigma)(3 + z (1 - 2 sigma)) - 2 z p)   (the derivative of phi'');
// the jet is v = phi, J_d = phi' z_Jd, L = phi' z_L + phi'' |z_J|^2, and its adjoint has the
// tanh adjoint's form with (s, s2, s3) = (phi', phi'', phi''').
__device__ __forceinline__ float sigmoid(float z) { return 1.0f / (1.0f + expf(-z)); }

// sigmoid from 1 / (1 + 2^(-z log2(e))) on the special-function unit (ex2.approx, rcp.approx),
// the SiLU counterpart of tanh_fast: a few 1e-7 absolute; saturates to exactly 0 and 1.
__device__ __forceinline__ float sigmoid_fast(float z) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(z * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(e + 1.0f));
  return r;
}

__device__ __forceinline__ void silu_jet_from_sigmoid(float sg, float zv, float zj0, float zj1,
                                                      float zl, float& v, float& j0, float& j1,
                                                      float& l) {
  const float p = sg * (1.0f - sg);
  const float d1 = fmaf(zv, p, sg);
  const float d2 = p * fmaf(zv, fmaf(-2.0f, sg, 1.0f), 2.0f);
  const float q = fmaf(zj0, zj0, zj1 * zj1);
  v = zv * sg;
  j0 = d1 * zj0;
  j1 = d1 * zj1;
  l = fmaf(d1, zl, d2 * q);
}

__device__ __forceinline__ void silu_jet(float zv, float zj0, float zj1, float zl, float& v,
                                         float& j0, float& j1, float& l) {
  silu_jet_from_sigmoid(sigmoid(zv), zv, zj0, zj1, zl, v, j0, j1, l);
}

__device__ __forceinline__ void silu_jet_fast(float zv, float zj0, float zj1, float zl, float& v,
                                              float& j0, float& j1, float& l) {
  silu_jet_from_sigmoid(sigmoid_fast(zv), zv, zj0, zj1, zl, v, j0, j1, l);
}

// Maps (vbar, J0bar, J1bar, Lbar) in place to (zbar_v, zbar_J0, zbar_J1, zbar_L).
__device__ __forceinline__ void silu_jet_adjoint(float zv, float zj0, float zj1, float zl,
                                                 float& av, float& aj0, float& aj1, float& al) {
  const float sg = sigmoid(zv);
  const float p = sg * (1.0f - sg);
  const float m = fmaf(-2.0f, sg, 1.0f);  // 1 - 2 sigma
  const float s = fmaf(zv, p, sg);
  const float s2 = p * fmaf(zv, m, 2.0f);
  const float s3 = p * fmaf(m, fmaf(zv, m, 3.0f), -2.0f * zv * p);
  const float q = fmaf(zj0, zj0, zj1 * zj1);
  const float gv = av * s + fmaf(aj0, zj0, aj1 * zj1) * s2 + al * fmaf(zl, s2, q * s3);
  const float l2 = 2.0f * al * s2;
  const float g0 = fmaf(aj0, s, l2 * zj0);
  const float g1 = fmaf(aj1, s, l2 * zj1);
  av = gv;
  aj0 = g0;
  aj1 = g1;
  al = al * s;
}

// Activation policies for the kernel templates: jet (accurate), jet_fast (special-function
// unit, tensor-core epilogues) and the adjoint in terms of the pre-activation jet.
struct TanhAct {
  static constexpr int kCode = FHB_ACTIVATION_TANH;
  static __device__ __forceinline__ void jet(float zv, float zj0, float zj1, float zl, float& v,
                                             float& j0, float& j1, float& l) {
    tanh_jet(zv, zj0, zj1, zl, v, j0, j1, l);
  }
  static __device__ __forceinline__ void jet_fast(float zv, float zj0, float zj1, float zl,
                                                  float& v, float& j0, float& j1, float& l) {
    tanh_jet_fast(zv, zj0, zj1, zl, v, j0, j1, l);
  }
  // jet_fast of two neurons (packed pair arithmetic, bitwise two jet_fast calls)
  static __device__ __forceinline__ void jet_fast2(float zv0, float zv1, float zj00, float zj01,
                                                   float zj10, float zj11, float zl0, float zl1,
                                                   float& v0, float& v1, float& j00,
                                                   float& j01, float& j10, float& j11,
                                                   float& l0, float& l1) {
    tanh_jet_fast2(zv0, zv1, zj00, zj01, zj10, zj11, zl0, zl1, v0, v1, j00, j01, j10, j11, l0,
                   l1);
  }
  static __device__ __forceinline__ void adjoint(float zv, float zj0, float zj1, float zl,
                                                 float& av, float& aj0, float& aj1, float& al) {
    tanh_jet_adjoint(zv, zj0, zj1, zl, av, aj0, aj1, al);
  }
};
struct SiluAct {
  static constexpr int kCode = FHB_ACTIVATION_SILU;
  static __device__ __forceinline__ void jet(float zv, float zj0, float zj1, float zl, float& v,
                                             float& j0, float& j1, float& l) {
    silu_jet(zv, zj0, zj1, zl, v, j0, j1, l);
  }
  static __device__ __forceinline__ void jet_fast(float zv, float zj0, float zj1, float zl,
                                                  float& v, float& j0, float& j1, float& l) {
    silu_jet_fast(zv, zj0, zj1, zl, v, j0, j1, l);
  }
  static __device__ __forceinline__ void jet_fast2(float zv0, float zv1, float zj00, float zj01,
                                                   float zj10, float zj11, float zl0, float zl1,
                                                   float& v0, float& v1, float& j00,
                                                   float& j01, float& j10, float& j11,
                                                   float& l0, float& l1) {
    silu_jet_fast(zv0, zj00, zj10, zl0, v0, j00, j10, l0);
    silu_jet_fast(zv1, zj01, zj11, zl1, v1, j01, j11, l1);
  }
  static __device__ __forceinline__ void adjoint(float zv, float zj0, float zj1, float zl,
                                                 float& av, float& aj0, float& aj1, float& al) {
    silu_jet_adjoint(zv, zj0, zj1, zl, av, aj0, aj1, al);
  }
};

// Warp-wide sum with a fixed butterfly order (deterministic).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

}  // namespace fhb
