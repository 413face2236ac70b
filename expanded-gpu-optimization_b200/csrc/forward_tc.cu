// Tensor-core forward-Laplacian kernel, one template over the operand format:
// 3xFP16 (forward version 3, the default tensor-core path) and 3xTF32 (versions 4, 5).
//
// Same math as the FP32 kernel and the reference (csrc/fused_residual.cu:16-23), with the
// three hidden 64x64 jet GEMMs on the 5th-generation tensor cores. Each hidden layer is,
// per tile of 128 points and per jet component c in {v, d/dx, d/dy, L},
//     Z_c[128 x 64] = H_c[128 x 64] . W^T,
// run as tcgen05.mma with M = 128 points and N = 64 output neurons, the A operand
// (activations) in tensor memory and B (weights) in shared memory. FP32 accuracy comes from a
// split x = hi + lo into two low-precision parts and three products per product:
//   * 3xTF32 (kind::tf32, K = 8): hi = tf32(x), lo = x - hi;
//     Z += H_hi W_hi + H_lo W_hi + H_hi W_lo; a 16-neuron chunk is 24 MMAs;
//   * 3xFP16 (kind::f16, K = 16): hi = x rounded to 11 significant bits (tf32 rounding, exact
//     in f16), lo = f16(x - hi) -- 11 + 11 significant bits, the precision of the tf32 split --;
//     Z += H_hi W_hi + H_lo W_hi + H_hi W_lo; a chunk is 12 MMAs and writes half the bytes into
//     TMEM. The tf32 form spends its layer time on the MMAs and on the TMEM traffic between the
//     chunk stores and the MMAs (a chunk's 24 MMAs take 0.57-0.74 us instead of 0.39 us while
//     16 warps store the next chunk), which this halves.
//     Range: f16 holds magnitudes below 65,504 (normal from 2^-14), and the Laplacian jet grows
//     fast with the weight scale. Each launch derives power-of-2 scales from the weights:
//     tau_l maps max|W_l| to <= 16; sigma_{l,c} maps an upper bound of component c of GEMM l's
//     A operand to <= 2^14, so lo stays a normal f16 for every value within 2^17 of its bound
//     and the rest lose at most 2^-25 (scaled units). The bounds: |v| <= 1; |dv/dx|, |dv/dy|
//     grow by N_l = max row-abs-sum of W_l per layer; |Lv| becomes N_l |Lv| + 2 (N_l B_J)^2
//     (tanh' <= 1 and 2 |tanh tanh'| <= 1). The epilogue folds the scales into the jet
//     arithmetic (F16Consts: accumulators times exact powers of 2 in, the next GEMM's scaled
//     operand out). The scales depend on the weights only (fixed-order warp reductions), so
//     every CTA and every shard of a batch uses the same ones.
//
// Where the data lives (per CTA, one CTA per SM, persistent over tiles):
//   * weights: all three hidden layers pre-split once per CTA into the K-major no-swizzle
//     canonical layout in shared memory (hi, lo; tf32 96 KB, f16 48 KB), from a copy of the
//     whole parameter buffer that one bulk (TMA) copy brings into shared memory while warp 0
//     allocates TMEM (staging from the copy instead of ~50 scattered global loads per thread
//     took the set-up from ~6 to ~3 us after an L2 flush);
//   * TMEM (512 columns x 128 lanes, lane = point):
//       [0, 256)   accumulators D_c, component c at columns 64c..64c+63;
//       [256, 512) a ring of A-operand chunks; a chunk is 16 input neurons of the next
//                  layer's activations in (component, hi/lo) blocks: tf32 2 slots of 128
//                  columns; f16 4 slots (a whole layer) of 64 columns, two K elements per
//                  32-bit column (K 2j in the low half of column j).
//     The A operand lives in TMEM, not shared memory: with N = 64 an A tile read from
//     shared memory would need ~1.5x the shared-memory bandwidth an SM has.
//   * 16 epilogue warps (warpgroups 0-3): warp w serves TMEM lanes 32(w%4)..+31 (its
//     quadrant) and, with s = w/4, neurons 16a+4s+t. Per layer it loads its 4 x 16
//     accumulators (16 x tcgen05.ld.x4), applies the tanh jet in registers and writes hi/lo
//     activations chunk by chunk into the ring (tcgen05.st) for the next layer, then arrives
//     on the slot's "full" mbarrier. Warp s owns the strided neurons 16a+4s+{0..3} (a = 0..3),
//     so chunk j (neurons 16j..16j+15, natural K order) gets 4 neurons from every warp;
//   * an MMA warpgroup (warps 16-19; warp 16 issues, 17-19 idle): for each chunk in order it
//     waits for the slot's 16 arrivals, issues the MMAs as a converged warp (elect.sync picks
//     the lane; issued from a divergent lane these small MMAs cost ~4x their execution time),
//     then (tf32) tcgen05.commit to free the slot, and after a layer's 4th chunk a commit that
//     marks D complete. A warp contributes to chunk 0 of layer l+1 only after it has read D
//     of layer l, so once chunk 0 is full D may be overwritten -- no separate "D free"
//     barrier. The f16 ring holds a whole layer, so the "D complete" wait before a layer's
//     epilogue also frees every slot it writes: f16 has no slot-free commit or wait.
//   So the MMAs of layer l+1 consume chunk j while the epilogue of layer l produces chunk
//   j+1. The tensor core has no deep instruction queue: issuing a chunk's MMAs occupies the
//   issuing warp for their whole execution (500-1100 cycles beside the epilogue's TMEM
//   stores). Issued by the epilogue warp that completed the chunk (an earlier form), that
//   warp fell behind, completed the next chunk last and issued again, putting every MMA on
//   the epilogue's critical path. A fifth warp per SM sub-partition caps registers at 96,
//   so the MMA warpgroup gives its registers to the epilogue with setmaxnreg: launched at 96
//   per thread (640 x 96), it drops to 24 and the epilogue warpgroups rise to 112
//   (128 x 72 freed >= 512 x 16 taken). The host checks that the kernel was built with 96
//   registers per thread: with fewer, the raise could never be granted.
// Layer 0 (2 inputs) and the output layer (1 output) are elementwise/epilogue work: tanh_fast
// (SFU exp2 + reciprocal), the split, and 16-neuron chunks to halve the synchronisation.
// Every mbarrier wait is bounded; a wait that gives up raises FHB_STATUS_MMA_TIMEOUT, sets
// a CTA abort flag that stops the other warps, and the kernel frees TMEM and returns.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace fhb {
namespace {

constexpr int kTile = 128;            // points per tile = MMA M = TMEM lanes
constexpr int kWarps = 16;              // epilogue warps, 4 per TMEM lane quadrant
constexpr int kThreads = kWarps * 32;   // epilogue threads
constexpr int kMmaWarp = kWarps;        // warp 16: first warp of the MMA warpgroup
constexpr int kBlockThreads = kThreads + 128;
// Registers per thread: at launch (__launch_bounds__(640, 1) caps ptxas at 96), the MMA
// warpgroup after setmaxnreg.dec, the epilogue warpgroups after setmaxnreg.inc.
constexpr int kLaunchRegs = 96, kMmaRegs = 24, kEpiRegs = 112;
static_assert((kLaunchRegs - kMmaRegs) * 128 >= (kEpiRegs - kLaunchRegs) * kThreads,
              "register split exceeds the launch's registers");
constexpr int kChunks = 4;            // chunks of 16 neurons per 64-wide layer
constexpr int kChunksPerTile = kHiddenGemms * kChunks;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kRingCol = 256;
constexpr uint32_t kLbo = 128;        // K-adjacent core matrices of the canonical layout

// Operand formats. One [64 x 64] weight operand is kOperandBytes in the K-major no-swizzle
// canonical layout: core matrices of 8 rows x 16 bytes (4 tf32 or 8 f16 elements), K chunks at
// LBO = 128 B, 8-row groups at kSbo. kOperands weight operands per hidden layer.
template <bool F16>
struct Format;
template <>
struct Format<false> {  // 3xTF32, kind::tf32, K = 8 per MMA
  static constexpr int kRing = 2;
  static constexpr uint32_t kSlotCols = 128;  // 4 components x {hi, lo} x 16 K positions
  static constexpr uint32_t kIdesc = tc::idesc_tf32(128, 64);
  static constexpr int kOperandBytes = kWidth * kWidth * 4;  // 16 KB
  static constexpr int kOperands = 2;                        // W_hi, W_lo
  static constexpr uint32_t kSbo = 2048;
};
template <>
struct Format<true> {  // 3xFP16, kind::f16, K = 16 per MMA
  static constexpr int kRing = 4;
  static constexpr uint32_t kSlotCols = 64;   // 4 components x {hi, lo} x 8 columns of pairs
  static constexpr uint32_t kIdesc = tc::idesc_f16(128, 64);
  static constexpr int kOperandBytes = kWidth * kWidth * 2;  // 8 KB
  static constexpr int kOperands = 2;                        // W_hi, W_lo (tau-scaled)
  static constexpr uint32_t kSbo = 1024;
};

// Shared memory layout (bytes): the weight operands, then the rest.
template <bool F16>
struct Layout {
  static constexpr int kSmallOff =
      kHiddenGemms * Format<F16>::kOperands * Format<F16>::kOperandBytes;
  static constexpr int kRedOff = kSmallOff + 512 * 4;     // small params, then [8][128] sums
  // mbarriers: empty[kRing], full[kRing], dfull, red, the parameter copy
  static constexpr int kBarOff = kRedOff + 8 * kTile * 4;
  static constexpr int kMiscOff = kBarOff + 16 * 8;        // TMEM base, abort flag
  static constexpr int kScaleOff = kMiscOff + 16;          // f16: F16Consts
  static constexpr int kParamOff = kScaleOff + (F16 ? 4096 : 1024);  // staged parameters
  static constexpr int kSmemUsed = kParamOff + kParamSmemFloats * 4;
  // Padded so two CTAs never share an SM (each allocates all 512 TMEM columns).
  static constexpr int kSmemBytes = kSmemUsed > 120 * 1024 ? (kSmemUsed + 1023) / 1024 * 1024
                                                           : 120 * 1024;
};
constexpr int kSmW0 = 0, kSmB0 = 128, kSmB = 192, kSmWout = 384, kSmBout = 448;
constexpr int kSmallFloats = 512;
static_assert(Layout<false>::kSmemBytes <= 227 * 1024 && Layout<true>::kSmemBytes <= 227 * 1024,
              "shared memory layout overflow");
static_assert(2 * Format<true>::kRing + 3 <= 16, "mbarrier space");

struct Ctx {
  uint8_t* smem;
  uint64_t* empty;            // [kRing] ring slot consumed by its MMAs (tcgen05.commit)
  uint64_t* full;             // [kRing] ring slot written by the 16 epilogue warps
  uint64_t* dfull;            // accumulators complete (tcgen05.commit)
  uint64_t* red;              // output-layer partial sums written (16 warps arrive)
  volatile uint32_t* abort_flag;
  unsigned int* status;
  uint32_t tmem;
  const float* f16c;          // f16: the F16Consts words
};

// f16 constants in shared memory (floats at Layout::kScaleOff). GEMM l's A operand,
// component c, is the true activation times sigma[l][c] (a power of 2; sigma_x = sigma_y),
// its weights are times tau[l], so its accumulators D are the true products times
// sigma tau. With us = 1 / (sigma_l tau_l), s' = sigma_{l+1} and k = 2 / ln 2, the epilogue
// of GEMM l (l = 0, 1) turns D straight into the next GEMM's scaled operand:
//   z' = k z = D_v (k us_v) + k b,  r = 1 / (2^z' + 1),  a = tanh z = 1 - 2r,
//   t = r (1 - r) = (1 - a^2) / 4,
//   v' = s'_v a = s'_v - 2 s'_v r,   J' = 4 t E1 D_J,
//   L' = 4 t (E2 D_L + E3 a |D_J|^2) = t (4 E2 D_L + (4 E3 - 8 E3 r) |D_J|^2),
// with E1 = s'_J us_J, E2 = s'_L us_L, E3 = -2 s'_L us_J^2 -- every constant a product of
// powers of 2 (exact) except k. The output stage (after GEMM 2) forms
//   u = sum_o w_o a_o + b_out,   lap = sum_o w_o t_o (4 us_L D_L - 8 us_J^2 a_o |D_J|^2),
// and layer 0 (2 inputs, z_L = 0, z_J = the row of W0) writes
//   v' = sigma_v a,  J'_d = 4 t sigma_J W0[o][d],  L' = t (4 C0 - 8 C0 r),
//   C0 = -2 sigma_L |W0[o]|^2.
struct F16Consts {
  static constexpr int kTau = 0;       // [3] tau_l (one pad word)
  static constexpr int kHid = 4;       // [2][8] GEMM l = 0, 1: k us_v, s'_v, -2 s'_v, 4 E1,
                                       //        4 E2, 4 E3, -8 E3, 0
  static constexpr int kOut = 20;      // k us_v, 4 us_L, -8 us_J^2 of GEMM 2; sigma_v and
                                       // -2 sigma_v of GEMM 0's operand (layer 0); pad
  static constexpr int kBias = 32;     // [3][64] k b of hidden layers 1..3
  static constexpr int kL0 = 224;      // [7][64] per layer-0 neuron: k W0[o][0], k W0[o][1],
                                       // k b0[o], 4 sigma_J W0[o][0], 4 sigma_J W0[o][1],
                                       // 4 C0, -8 C0
  static constexpr int kWords = 672;
};
constexpr int kScaleFloats = 1024;
static_assert(F16Consts::kWords <= kScaleFloats, "the F16Consts words fit the scale region");

// Bounded wait that also gives up when another warp has aborted the CTA.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Ctx& cx) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_for(bar, parity, kSuspendHintNs)) return true;
    if (*cx.abort_flag) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      *cx.abort_flag = 1u;
      report_status(cx.status, FHB_STATUS_MMA_TIMEOUT);
      return false;
    }
  }
}

// Every lane polls; the vote makes the outcome warp-uniform (it can differ between lanes only
// when the time limit expires just as the phase completes), because the aligned tcgen05
// ld/st and elect.sync that follow need the whole warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const Ctx& cx) {
  return __all_sync(0xffffffffu, wait_or_abort(bar, parity, cx) ? 1 : 0) != 0;
}

// f16 pairs of a split: hi = x rounded to 11 significant bits (tf32 rounding; exact in f16
// inside the scaled range), lo = x - hi (exact in FP32, rounded to f16); element a (even K)
// in the low halves. Values below f16's normal range (2^-14, 2^28 below a scaled bound) lose
// precision, an absolute error of at most 2^-25 in scaled units.
__device__ __forceinline__ void split_f16_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const float ha = __uint_as_float(tc::to_tf32(a)), hb = __uint_as_float(tc::to_tf32(b));
  const __half2 h = __floats2half2_rn(ha, hb);
  const __half2 l = __floats2half2_rn(a - ha, b - hb);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// r = 1 / (2^zp + 1) on the special-function unit (ex2.approx, rcp.approx), zp = 2 z / ln 2
// already scaled by the caller's constants: tanh z = 1 - 2r (tanh_fast's formula, <= 5e-7
// from tanhf). 2^zp overflows to +inf for large z (r = 0, tanh = 1) and underflows to 0 for
// very negative z (r = 1, tanh = -1): never NaN.
__device__ __forceinline__ float tanh_r_scaled(float zp) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(zp));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(e + 1.0f));
  return r;
}

constexpr float kTwoOverLn2 = 2.8853900817779268f;  // 2 / ln 2 = 2 log2(e)

// tanh_r_scaled of two values, the sum 2^zp + 1 as one packed add (rounded as the scalar
// add): bitwise the results of two tanh_r_scaled calls.
__device__ __forceinline__ void tanh_r_scaled2(float zp0, float zp1, float& r0, float& r1) {
  float e0, e1, p0, p1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(zp0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(zp1));
  add2o(p0, p1, e0, e1, 1.0f, 1.0f);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(p0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(p1));
}


__device__ __forceinline__ float4 ld_f4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
__device__ __forceinline__ float at(const float4& v, int t) {
  return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// The MMAs of chunk j (input neurons 16j..16j+15) of hidden GEMM `layer`, A from ring slot
// `slot`, then (tf32) a commit that frees the slot, and after the 4th chunk one that marks D
// complete. tf32: 2 K steps x 4 components x (H_hi W_hi + H_lo W_hi + H_hi W_lo), A block
// (component c, hi/lo sp, K step kk) at columns 32c + 16sp + 8kk of the slot. f16: 4
// components x (H_hi W_hi + H_lo W_hi + H_hi W_lo), A block (c, sp) at 16c + 8sp. One elected
// lane issues a chunk's MMAs in one block (issued one call each, with their own election and
// predicate set-up, the chunk's MMAs took ~80 issue cycles apiece).
template <bool F16>
__device__ __forceinline__ void issue_chunk_mmas(const Ctx& cx, int layer, int j, uint32_t slot) {
  using F = Format<F16>;
  const uint32_t slot_col = cx.tmem + kRingCol + F::kSlotCols * slot;
  if constexpr (F16) {
    const uint32_t w0 = smem_u32(cx.smem + (2 * layer) * F::kOperandBytes + 256 * j);
    const uint64_t b_hi = tc::smem_desc_kmajor(w0, kLbo, F::kSbo);
    const uint64_t b_lo = tc::smem_desc_kmajor(w0 + F::kOperandBytes, kLbo, F::kSbo);
    tc::mma_f16_ts_chunk_warp(cx.tmem, slot_col, b_hi, b_lo, F::kIdesc, j > 0 ? 1u : 0u);
  } else {
    const uint32_t w0 = smem_u32(cx.smem + (2 * layer) * F::kOperandBytes + 512 * j);
    const uint64_t bh0 = tc::smem_desc_kmajor(w0, kLbo, F::kSbo);
    const uint64_t bl0 = tc::smem_desc_kmajor(w0 + F::kOperandBytes, kLbo, F::kSbo);
    const uint64_t bh1 = tc::smem_desc_kmajor(w0 + 256, kLbo, F::kSbo);
    const uint64_t bl1 = tc::smem_desc_kmajor(w0 + 256 + F::kOperandBytes, kLbo, F::kSbo);
    tc::mma_tf32_ts_chunk_warp(cx.tmem, slot_col, bh0, bl0, bh1, bl1, F::kIdesc,
                               j > 0 ? 1u : 0u);
  }
  if constexpr (!F16) tc::commit_warp(&cx.empty[slot]);  // f16: see produce_chunk
  if (j == kChunks - 1) tc::commit_warp(cx.dfull);
}

// Write chunk `n` (this warp's 4 neurons x 4 components as hi/lo parts; f16: h is already
// the scaled operand) into ring slot n % kRing; the warp completing the chunk last issues its
// MMAs. False if aborted.
template <bool F16>
__device__ __forceinline__ bool produce_chunk(uint32_t n, int j, const float (&h)[4][4],
                                              uint32_t tmem_warp, int s, const Ctx& cx) {
  using F = Format<F16>;
  // n = 12 tile + 4 layer + j, and the ring size divides 4: the slot is j % kRing, known at
  // compile time in the unrolled chunk loops (so are the TMEM store addresses).
  const uint32_t slot = static_cast<uint32_t>(j) % F::kRing;
  // A slot is free once the MMAs of the chunk that used it before have completed. Chunks 0
  // and 1 of a GEMM (and every f16 chunk: the f16 ring holds a whole layer) reuse a slot of
  // the previous GEMM, whose MMAs the "D complete" commit that this warp waited on before
  // computing the chunk already covers; only tf32 chunks 2 and 3, which reuse the slots of
  // chunks 0 and 1 of the same GEMM, wait for a slot's commit (a wait that cannot block still
  // measured ~300 cycles per chunk). The commits still come once per chunk, so the parity of
  // the waits that remain counts every chunk of the slot.
  if constexpr (!F16) {
    if (j >= F::kRing) {  // n % kChunks == j
      if (!warp_wait(&cx.empty[slot], ((n / F::kRing) & 1u) ^ 1u, cx)) return false;
      tc::fence_after_sync();
    }
  }
  const uint32_t slot_col = tmem_warp + kRingCol + F::kSlotCols * slot;
  if constexpr (F16) {
    const uint32_t base = slot_col + 2u * s;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hi0, lo0, hi1, lo1;
      split_f16_pair_fast(h[c][0], h[c][1], hi0, lo0);
      split_f16_pair_fast(h[c][2], h[c][3], hi1, lo1);
      tc::st_x2(base + 16u * c, hi0, hi1);
      tc::st_x2(base + 16u * c + 8u, lo0, lo1);
    }
  } else {
    const uint32_t base = slot_col + 4u * s;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) tc::split_tf32(h[c][t], hi[t], lo[t]);
      tc::st_x4(base + 32u * c, hi[0], hi[1], hi[2], hi[3]);
      tc::st_x4(base + 32u * c + 16u, lo[0], lo[1], lo[2], lo[3]);
    }
  }
  tc::wait_st();
  tc::fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&cx.full[slot]);
  return true;
}

// Barrier 1 over the 16 epilogue warps (the MMA warpgroup skips the weight staging).
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
}
// Register reallocation within the block's launch budget (whole warpgroups, warp-uniform).
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Small parameter of thread i: W0, b0, b1..b3, w_out, b_out in the order of `small`.
__device__ __forceinline__ float small_param(const float* __restrict__ params, int i) {
  if (i < kSmB0) return params[i];                                          // W0
  if (i < kSmB) return params[kB0 + (i - kSmB0)];                           // b0
  if (i < kSmWout) {                                                        // b1..b3
    const int l = (i - kSmB) >> 6, o = (i - kSmB) & 63;
    return params[kHiddenBase + l * kHiddenStride + kWidth * kWidth + o];
  }
  if (i < kSmBout) return params[kOutBase + (i - kSmWout)];                 // w_out
  if (i == kSmBout) return params[kOutBase + kWidth];                       // b_out
  return 0.0f;
}

// tf32 set-up: the small parameters and the hi/lo split of the hidden weights. Element
// (row, k) of a layer's operand sits at word (row / 8) 512 + (k / 4) 32 + (row % 8) 4 + k % 4
// of the canonical K-major layout. Pass j of warp w covers row group g = j % 8 of layer j / 8
// with the K chunks rotated by w: lane (r = lane / 4, t = lane % 4) takes row 8g + r and
// k = 4 ((r + w) % 16) + t, so the row-major read (bank k % 32) and the canonical store
// (bank 4r + t) each touch 32 distinct banks. All 25 loads of a thread (24 weights, one
// small parameter) are issued before any is used.
__device__ __forceinline__ void stage_tf32(const float* __restrict__ params, uint8_t* smem,
                                           float* small, int warp, int lane) {
  using F = Format<false>;
  const float sv = small_param(params, threadIdx.x);
  constexpr int kPasses = kHiddenGemms * kWidth * kWidth / kThreads;  // 24
  const int r = lane >> 2, t = lane & 3;
  const int kc = (r + warp) & 15;  // this lane's K chunk of 4
  const int k = 4 * kc + t;
  float w[kPasses];
#pragma unroll
  for (int j = 0; j < kPasses; ++j) {
    const int layer = j >> 3, row = 8 * (j & 7) + r;
    w[j] = params[kHiddenBase + layer * kHiddenStride + neuron_of_column(row) * kWidth + k];
  }
#pragma unroll
  for (int j = 0; j < kPasses; ++j) {
    const int layer = j >> 3, g = j & 7;
    const uint32_t hi = tc::to_tf32(w[j]);
    const uint32_t lo = tc::to_tf32(w[j] - __uint_as_float(hi));
    const int word = g * 512 + kc * 32 + 4 * r + t;
    reinterpret_cast<uint32_t*>(smem + (2 * layer) * F::kOperandBytes)[word] = hi;
    reinterpret_cast<uint32_t*>(smem + (2 * layer + 1) * F::kOperandBytes)[word] = lo;
  }
  small[threadIdx.x] = sv;
}

// f16 set-up: the small parameters, the operand scales and the epilogue constants
// (F16Consts), then the split of the tau-scaled hidden weights into W_hi and W_lo. Power-of-2
// scales keep every f16 operand in range: tau_l maps max|W_l| to <= 16; sigma_{l,c} maps a
// bound of component c of GEMM l's A operand to <= 2^14 (one sigma for d/dx and d/dy, from
// the larger bound). Bounds: |v| <= 1; |d/dx|, |d/dy| grow by N_l (max row-abs-sum of W_l)
// per layer; |L| becomes N_l |L| + (N_l Bx)^2 + (N_l By)^2 (tanh' <= 1, 2 |tanh tanh'| <= 1).
// Statistics: threads 0..383 take half a hidden-weight row each (row tid / 2, 32 elements
// read in a rotated order, so a warp's 32 reads touch 32 banks), threads 384..447 one row of
// W0; per-warp maxima by redux (non-negative floats order as their bit patterns). All sums
// run in a fixed order, so every CTA derives the same scales. Contains one barrier of the
// epilogue warps.
__device__ __forceinline__ void stage_f16(const float* __restrict__ params, uint8_t* smem,
                                          float* small, float* red, float* cst, int warp,
                                          int lane) {
  using F = Format<true>;
  constexpr int kPairs = kHiddenGemms * kWidth * kWidth / 2;       // 6144
  constexpr int kPairsPerThread = kPairs / kThreads;               // 12
  static_assert(kPairs % kThreads == 0, "whole pairs per thread");
  constexpr int kStatThreads = 2 * kHiddenGemms * kWidth;          // 384
  using C = F16Consts;
  float wp[kPairsPerThread][2];
  {
    const float sv = small_param(params, threadIdx.x);
#pragma unroll
    for (int j = 0; j < kPairsPerThread; ++j) {
      const int it = warp + kWarps * j;  // layer it / 64, row group (it / 8) % 8, rotation it % 8
      const int layer = it >> 6, row = 8 * ((it >> 3) & 7) + (lane >> 2);
      const int kk = 8 * (((lane >> 2) + it) & 7) + 2 * (lane & 3);
      const float2 v = *reinterpret_cast<const float2*>(
          params + kHiddenBase + layer * kHiddenStride + neuron_of_column(row) * kWidth + kk);
      wp[j][0] = v.x;
      wp[j][1] = v.y;
    }
    float m0 = 0.0f, m1 = 0.0f;  // hidden rows: abs-sum, max |w|; W0 rows: max |w|, |w|^2
    if (threadIdx.x < kStatThreads) {
      const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
      const float* wr = params + kHiddenBase + (r >> 6) * kHiddenStride + (r & 63) * kWidth +
                        32 * h;
      float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = fabsf(wr[(j + threadIdx.x) & 31]);
        a[j & 3] += x;
        m1 = fmaxf(m1, x);
      }
      m0 = (a[0] + a[1]) + (a[2] + a[3]);
      m0 += __shfl_xor_sync(0xffffffffu, m0, 1);  // the row's two halves
    } else if (threadIdx.x < kStatThreads + kWidth) {
      const int o = threadIdx.x - kStatThreads;
      const float wx = params[2 * o], wy = params[2 * o + 1];
      m0 = fmaxf(fabsf(wx), fabsf(wy));
      m1 = fmaf(wx, wx, wy * wy);
    }
    const uint32_t r0 = __reduce_max_sync(0xffffffffu, __float_as_uint(m0));
    const uint32_t r1 = __reduce_max_sync(0xffffffffu, __float_as_uint(m1));
    if (lane == 0) {  // warps 4l..4l+3: layer l's rows; warps 12, 13: W0
      red[warp] = __uint_as_float(r0);
      red[16 + warp] = __uint_as_float(r1);
    }
    small[threadIdx.x] = sv;
  }
  epi_sync();
  // Every warp derives the scales itself (no second barrier); warp 0 stores the constants.
  // Lane l < 3 derives tau_l; the bound recursion over the layers runs in every lane.
  float nrm[3];
#pragma unroll
  for (int l = 0; l < 3; ++l)
    nrm[l] = fmaxf(fmaxf(red[4 * l], red[4 * l + 1]), fmaxf(red[4 * l + 2], red[4 * l + 3]));
  const int lt = lane < 3 ? lane : 0;
  const float wmax = fmaxf(fmaxf(red[16 + 4 * lt], red[17 + 4 * lt]),
                           fmaxf(red[18 + 4 * lt], red[19 + 4 * lt]));
  const float tau_mine = pow2_floor_ratio(4, wmax);
  float tau[3];
#pragma unroll
  for (int l = 0; l < 3; ++l) tau[l] = __shfl_sync(0xffffffffu, tau_mine, l);
  float sig[3][3];  // sig[l]: v, J, L
  {
    float bj = fmaxf(red[12], red[13]);
    float bl = fmaxf(red[28], red[29]);
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      sig[l][0] = 16384.0f;
      sig[l][1] = pow2_floor_ratio(14, bj);
      sig[l][2] = pow2_floor_ratio(14, bl);
      const float nj = nrm[l] * bj;
      bl = fmaf(nrm[l], bl, 2.0f * nj * nj);
      bj = nj;
    }
  }
  if (warp == 0) {
    float us[3][3];  // 1 / (sigma tau) of GEMM l's accumulators, per component (exact)
#pragma unroll
    for (int l = 0; l < 3; ++l)
#pragma unroll
      for (int c = 0; c < 3; ++c) us[l][c] = inv_pow2(sig[l][c] * tau[l]);
    if (lane < 3) cst[C::kTau + lane] = tau_mine;
    if (lane < 2) {  // hidden epilogues: GEMM l's accumulators -> GEMM l+1
      const int l = lane;
      const float u1 = l == 0 ? us[0][1] : us[1][1], u2 = l == 0 ? us[0][2] : us[1][2];
      const float u0 = l == 0 ? us[0][0] : us[1][0];
      const float s0 = l == 0 ? sig[1][0] : sig[2][0], s1 = l == 0 ? sig[1][1] : sig[2][1];
      const float s2 = l == 0 ? sig[1][2] : sig[2][2];
      const float e1 = s1 * u1, e2 = s2 * u2, e3 = -2.0f * s2 * u1 * u1;
      float* k = cst + C::kHid + 8 * l;
      k[0] = kTwoOverLn2 * u0;
      k[1] = s0;
      k[2] = -2.0f * s0;
      k[3] = 4.0f * e1;
      k[4] = 4.0f * e2;
      k[5] = 4.0f * e3;
      k[6] = -8.0f * e3;
      k[7] = 0.0f;
    } else if (lane == 2) {
      float* k = cst + C::kOut;  // the output stage, and layer 0's value scale
      k[0] = kTwoOverLn2 * us[2][0];
      k[1] = 4.0f * us[2][2];
      k[2] = -8.0f * us[2][1] * us[2][1];
      k[3] = 0.0f;
      k[4] = sig[0][0];
      k[5] = -2.0f * sig[0][0];
    }
  }
  if (threadIdx.x < kWidth) {  // layer-0 jets: J = W0 columns, L = -2 a s |W0 row|^2
    const int o = threadIdx.x;
    const float w0 = small[kSmW0 + 2 * o], w1 = small[kSmW0 + 2 * o + 1];
    const float c0 = -2.0f * sig[0][2] * fmaf(w0, w0, w1 * w1);
    float* l0 = cst + C::kL0;
    l0[0 * kWidth + o] = kTwoOverLn2 * w0;
    l0[1 * kWidth + o] = kTwoOverLn2 * w1;
    l0[2 * kWidth + o] = kTwoOverLn2 * small[kSmB0 + o];
    l0[3 * kWidth + o] = 4.0f * sig[0][1] * w0;
    l0[4 * kWidth + o] = 4.0f * sig[0][1] * w1;
    l0[5 * kWidth + o] = 4.0f * c0;
    l0[6 * kWidth + o] = -8.0f * c0;
  }
  if (threadIdx.x < 3 * kWidth)  // hidden biases in the scaled tanh argument
    cst[C::kBias + threadIdx.x] = kTwoOverLn2 * small[kSmB + threadIdx.x];
  // The split: pair (row, kk..kk+1) of a layer's operand is word
  // (row / 8) 256 + (kk / 8) 32 + (row % 8) 4 + (kk % 8) / 2 of the canonical K-major layout.
  // Pass j of warp w is iteration it = w + 16 j: row group (it / 8) % 8 of layer it / 64, with
  // the K chunks of 8 rotated by it % 8. Lane (r = lane / 4, p = lane % 4) takes row
  // 8 ((it / 8) % 8) + r and the pair at kk = 8 ((r + it) % 8) + 2p: the row-major float2 read
  // touches 16 distinct bank pairs per half warp and the canonical store banks 4r + p.
#pragma unroll
  for (int j = 0; j < kPairsPerThread; ++j) {
    const int it = warp + kWarps * j;
    const int layer = it >> 6;  // = j / 4
    const float t = tau[j >> 2];
    uint32_t hi, lo;
    split_f16_pair(wp[j][0] * t, wp[j][1] * t, hi, lo);
    const int word = ((it >> 3) & 7) * 256 + (((lane >> 2) + it) & 7) * 32 + lane;
    uint32_t* base = reinterpret_cast<uint32_t*>(smem + (2 * layer) * F::kOperandBytes);
    base[word] = hi;
    base[word + F::kOperandBytes / 4] = lo;
  }
}

// Layer 0 of one tile, for the point (x0, x1) of this thread: z = W0 x + b0, z_J = the row of
// W0, z_L = 0, through the activation into the four chunks of GEMM 0's A operand (f16: the
// scaled operand directly). Advances the chunk counter; false if a wait gave up.
template <bool F16, class Act>
__device__ __forceinline__ bool produce_layer0(float x0, float x1, uint32_t& chunk,
                                               uint32_t tmem_warp, int s, const Ctx& cx,
                                               const float* small) {
  if constexpr (F16) {
    using C = F16Consts;
    const float sv = cx.f16c[C::kOut + 4], sv2 = cx.f16c[C::kOut + 5];
    const float* l0 = cx.f16c + C::kL0 + 4 * s;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const float* c0 = l0 + 16 * j;  // neurons 16j + 4s + t, t = 0..3
      const float4 wx = ld_f4(c0), wy = ld_f4(c0 + kWidth), bz = ld_f4(c0 + 2 * kWidth);
      const float4 kj0 = ld_f4(c0 + 3 * kWidth), kj1 = ld_f4(c0 + 4 * kWidth);
      const float4 kl = ld_f4(c0 + 5 * kWidth), kl2 = ld_f4(c0 + 6 * kWidth);
      float h[4][4];
      // neuron pairs (t, t + 1) in packed FP32 arithmetic, each lane rounded as the scalar op
#pragma unroll
      for (int t = 0; t < 4; t += 2) {
        float z0, z1, r0, r1, tt0, tt1, m0, m1;
        fma2o(z0, z1, at(wy, t), at(wy, t + 1), x1, x1, at(bz, t), at(bz, t + 1));
        fma2o(z0, z1, at(wx, t), at(wx, t + 1), x0, x0, z0, z1);
        tanh_r_scaled2(z0, z1, r0, r1);
        fma2o(tt0, tt1, -r0, -r1, r0, r1, r0, r1);  // (1 - tanh^2) / 4
        fma2o(h[0][t], h[0][t + 1], sv2, sv2, r0, r1, sv, sv);
        mul2o(h[1][t], h[1][t + 1], tt0, tt1, at(kj0, t), at(kj0, t + 1));
        mul2o(h[2][t], h[2][t + 1], tt0, tt1, at(kj1, t), at(kj1, t + 1));
        fma2o(m0, m1, at(kl2, t), at(kl2, t + 1), r0, r1, at(kl, t), at(kl, t + 1));
        mul2o(h[3][t], h[3][t + 1], tt0, tt1, m0, m1);
      }
      if (!produce_chunk<F16>(chunk++, j, h, tmem_warp, s, cx)) return false;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      float h[4][4];
#pragma unroll
      for (int t = 0; t < 4; t += 2) {  // neuron pairs o, o + 1
        const int o = 16 * j + 4 * s + t;
        const float w0a = small[kSmW0 + 2 * o], w1a = small[kSmW0 + 2 * o + 1];
        const float w0b = small[kSmW0 + 2 * o + 2], w1b = small[kSmW0 + 2 * o + 3];
        float za, zb;
        fma2o(za, zb, w1a, w1b, x1, x1, small[kSmB0 + o], small[kSmB0 + o + 1]);
        fma2o(za, zb, w0a, w0b, x0, x0, za, zb);
        Act::jet_fast2(za, zb, w0a, w0b, w1a, w1b, 0.0f, 0.0f, h[0][t], h[0][t + 1], h[1][t],
                       h[1][t + 1], h[2][t], h[2][t + 1], h[3][t], h[3][t + 1]);
      }
      if (!produce_chunk<F16>(chunk++, j, h, tmem_warp, s, cx)) return false;
    }
  }
  return true;
}

template <bool F16, class Act>
__global__ void __launch_bounds__(kBlockThreads, 1)
    forward_tc_kernel(const float* __restrict__ coords, const float* __restrict__ params,
                      float* __restrict__ u_out, float* __restrict__ lap_out, int64_t n,
                      int64_t tiles, int params_aligned, unsigned int* status) {
  using F = Format<F16>;
  using L = Layout<F16>;
  // The f16 range scales bound the jets with |tanh| <= 1 and tanh' <= 1: tanh only.
  static_assert(!F16 || Act::kCode == FHB_ACTIVATION_TANH, "3xFP16 operands need the tanh bounds");
  extern __shared__ __align__(1024) uint8_t smem[];
  float* small = reinterpret_cast<float*>(smem + L::kSmallOff);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  Ctx cx;
  cx.smem = smem;
  cx.empty = bars;
  cx.full = bars + F::kRing;
  cx.dfull = bars + 2 * F::kRing;
  cx.red = bars + 2 * F::kRing + 1;
  cx.abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L::kMiscOff + 4);
  cx.status = status;
  cx.f16c = reinterpret_cast<const float*>(smem + L::kScaleOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The first tile's point, requested first: its latency overlaps the set-up below.
  const int row0 = 32 * (warp & 3) + lane;
  float nx0 = 0.0f, nx1 = 0.0f;
  if (warp < kWarps) {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kTile + row0;
    if (p < n) {
      nx0 = coords[2 * p];
      nx1 = coords[2 * p + 1];
    }
  }

  // ---- set-up ----
  // Barriers first, then one bulk copy of the parameter buffer into shared memory and the
  // TMEM allocation while it is in flight; the statistics and the split read the staged copy.
  float* sp = reinterpret_cast<float*>(smem + L::kParamOff);
  uint64_t* pbar = bars + 2 * F::kRing + 2;
  if (threadIdx.x == 0) {
    for (int r = 0; r < F::kRing; ++r) {
      mbar_init(&cx.empty[r], 1);
      mbar_init(&cx.full[r], kWarps);
    }
    mbar_init(cx.dfull, 1);
    mbar_init(cx.red, kWarps);
    mbar_init(pbar, 1);
    *cx.abort_flag = 0u;
    fence_barrier_init();
    if (params_aligned) {
      mbar_arrive_expect_tx(pbar, kParamBulkFloats * 4);
      bulk_copy_g2s(sp, params, kParamBulkFloats * 4, pbar);
    }
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  if (!params_aligned) {
    for (int k = threadIdx.x; k < kParamCount; k += kBlockThreads) sp[k] = params[k];
  } else if (threadIdx.x == 32) {
    for (int k = kParamBulkFloats; k < kParamCount; ++k) sp[k] = params[k];
  }
  __syncthreads();  // barriers initialised; plain-loaded parameters written
  const bool staged =
      !params_aligned || mbar_wait_bounded(pbar, 0, status, FHB_STATUS_STAGE_TIMEOUT);
  if (__syncthreads_and(staged ? 1 : 0) == 0) {
    if (threadIdx.x == 0) *cx.abort_flag = 1u;
  } else if (warp < kWarps) {
    static_assert(kSmallFloats == kThreads, "one small parameter per thread");
    if constexpr (F16) {
      stage_f16(sp, smem, small, red, reinterpret_cast<float*>(smem + L::kScaleOff), warp, lane);
    } else {
      stage_tf32(sp, smem, small, warp, lane);
    }
  }
  tc::fence_proxy_async_smem();  // weight operands visible to the tensor core
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  cx.tmem = *tmem_base_slot;

  const bool run = *cx.abort_flag == 0u;
  if (warp >= kWarps) {
    // ---- MMA warpgroup: warp 16 issues every chunk of this CTA's tiles in order ----
    regs_dec<kMmaRegs>();
    if (warp == kMmaWarp && run) {
      const int64_t mine = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      const uint32_t total = static_cast<uint32_t>(mine) * kChunksPerTile;
      for (uint32_t n = 0; n < total; ++n) {
        const uint32_t slot = n % F::kRing;
        if (!warp_wait(&cx.full[slot], (n / F::kRing) & 1u, cx)) break;
        tc::fence_after_sync();
        const uint32_t in_tile = n % kChunksPerTile;
        issue_chunk_mmas<F16>(cx, static_cast<int>(in_tile / kChunks),
                              static_cast<int>(in_tile % kChunks), slot);
        __syncwarp();
      }
    }
  } else {
    // ---- epilogue warpgroups ----
    regs_inc<kEpiRegs>();
    const int q = warp & 3;   // TMEM lane quadrant
    const int s = warp >> 2;  // neuron block 16s..16s+15
    const uint32_t tmem_warp = cx.tmem + (static_cast<uint32_t>(32 * q) << 16);
    const int row = 32 * q + lane;
    uint32_t chunk = 0, mlayer = 0, tile_count = 0;
    bool ok = run;
    // Layer 0 of a tile runs at the end of the previous tile (right after GEMM 2's
    // accumulators are loaded, before that tile's output stage), so GEMM 0 of the next tile
    // runs on the tensor core while the warps finish the output stage. The first tile's
    // layer 0 runs here. Points are loaded one tile ahead, so the load latency (long when the
    // points sit in pinned host memory read over the host link) overlaps a tile of work.
    if (ok && static_cast<int64_t>(blockIdx.x) < tiles)
      ok = produce_layer0<F16, Act>(nx0, nx1, chunk, tmem_warp, s, cx, small);
    for (int64_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tile_count) {
      const int64_t p = tile * kTile + row;
      const bool active = p < n;
      const bool has_next = tile + gridDim.x < tiles;
      {
        const int64_t pn = p + static_cast<int64_t>(gridDim.x) * kTile;
        nx0 = pn < n ? coords[2 * pn] : 0.0f;
        nx1 = pn < n ? coords[2 * pn + 1] : 0.0f;
      }

      for (int l = 0; ok && l < kHiddenGemms; ++l, ++mlayer) {
        if (!(ok = warp_wait(cx.dfull, mlayer & 1u, cx))) break;
        tc::fence_after_sync();
        // d[c][4a + t] = component c of neuron 16a + 4s + t: 16 consecutive accumulator
        // columns (the B rows are permuted, neuron_of_column)
        float d[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::ld_x16(tmem_warp + 64u * c + 16u * s, d[c]);
        tc::wait_ld();
        float pu = 0.0f, pl = 0.0f;  // output stage: this warp's share of u and lap
        if constexpr (F16) {
          using C = F16Consts;
          const float* bias = cx.f16c + C::kBias + 64 * l + 4 * s;  // k b, layer l + 1
          if (l + 1 < kHiddenGemms) {  // accumulators -> the next GEMM's scaled operand
            const float4 ka = ld_f4(cx.f16c + C::kHid + 8 * l);
            const float4 kb = ld_f4(cx.f16c + C::kHid + 8 * l + 4);
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
              const float4 bb = ld_f4(bias + 16 * j);
              float h[4][4];
              // neuron pairs (t, t + 1) in packed FP32 arithmetic, rounded as the scalar ops
#pragma unroll
              for (int t = 0; t < 4; t += 2) {
                const int i = 4 * j + t;
                float z0, z1, r0, r1, tt0, tt1, sk0, sk1, q0, q1, g0, g1, m0, m1;
                fma2o(z0, z1, d[0][i], d[0][i + 1], ka.x, ka.x, at(bb, t), at(bb, t + 1));
                tanh_r_scaled2(z0, z1, r0, r1);
                fma2o(tt0, tt1, -r0, -r1, r0, r1, r0, r1);  // (1 - tanh^2) / 4
                mul2o(sk0, sk1, tt0, tt1, ka.w, ka.w);
                mul2o(q0, q1, d[2][i], d[2][i + 1], d[2][i], d[2][i + 1]);
                fma2o(q0, q1, d[1][i], d[1][i + 1], d[1][i], d[1][i + 1], q0, q1);
                fma2o(g0, g1, kb.z, kb.z, r0, r1, kb.y, kb.y);
                fma2o(h[0][t], h[0][t + 1], ka.z, ka.z, r0, r1, ka.y, ka.y);
                mul2o(h[1][t], h[1][t + 1], sk0, sk1, d[1][i], d[1][i + 1]);
                mul2o(h[2][t], h[2][t + 1], sk0, sk1, d[2][i], d[2][i + 1]);
                mul2o(m0, m1, kb.x, kb.x, d[3][i], d[3][i + 1]);
                fma2o(m0, m1, g0, g1, q0, q1, m0, m1);
                mul2o(h[3][t], h[3][t + 1], tt0, tt1, m0, m1);
              }
              if (!(ok = produce_chunk<F16>(chunk++, j, h, tmem_warp, s, cx))) break;
            }
            continue;
          }
          if (has_next && !(ok = produce_layer0<F16, Act>(nx0, nx1, chunk, tmem_warp, s, cx,
                                                          small)))
            break;
          // output layer: u = w.a + b, lap = w.L, over this warp's 16 neurons
          const float4 ko = ld_f4(cx.f16c + C::kOut);
          const float* wout = small + kSmWout + 4 * s;
#pragma unroll
          for (int j = 0; j < kChunks; ++j) {
            const float4 bb = ld_f4(bias + 16 * j), ww = ld_f4(wout + 16 * j);
#pragma unroll
            for (int t = 0; t < 4; t += 2) {
              const int i = 4 * j + t;
              float z0, z1, r0, r1, tt0, tt1, a0, a1, q0, q1, m0, m1, n0, n1, w0, w1;
              fma2o(z0, z1, d[0][i], d[0][i + 1], ko.x, ko.x, at(bb, t), at(bb, t + 1));
              tanh_r_scaled2(z0, z1, r0, r1);
              fma2o(tt0, tt1, -r0, -r1, r0, r1, r0, r1);
              fma2o(a0, a1, -2.0f, -2.0f, r0, r1, 1.0f, 1.0f);
              mul2o(q0, q1, d[2][i], d[2][i + 1], d[2][i], d[2][i + 1]);
              fma2o(q0, q1, d[1][i], d[1][i + 1], d[1][i], d[1][i + 1], q0, q1);
              mul2o(m0, m1, ko.z, ko.z, a0, a1);
              mul2o(n0, n1, ko.y, ko.y, d[3][i], d[3][i + 1]);
              fma2o(m0, m1, m0, m1, q0, q1, n0, n1);  // inner
              mul2o(w0, w1, at(ww, t), at(ww, t + 1), tt0, tt1);
              // the sums in neuron order, as scalar fmas
              pu = fmaf(at(ww, t), a0, pu);
              pl = fmaf(w0, m0, pl);
              pu = fmaf(at(ww, t + 1), a1, pu);
              pl = fmaf(w1, m1, pl);
            }
          }
        } else {
          const float* bias = small + kSmB + 64 * l;
          if (l + 1 < kHiddenGemms) {
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
              float h[4][4];
#pragma unroll
              for (int t = 0; t < 4; t += 2) {
                const int i = 4 * j + t;
                float z0, z1;
                add2o(z0, z1, d[0][i], d[0][i + 1], bias[16 * j + 4 * s + t],
                      bias[16 * j + 4 * s + t + 1]);
                Act::jet_fast2(z0, z1, d[1][i], d[1][i + 1], d[2][i], d[2][i + 1], d[3][i],
                               d[3][i + 1], h[0][t], h[0][t + 1], h[1][t], h[1][t + 1], h[2][t],
                               h[2][t + 1], h[3][t], h[3][t + 1]);
              }
              if (!(ok = produce_chunk<F16>(chunk++, j, h, tmem_warp, s, cx))) break;
            }
            continue;
          }
          if (has_next && !(ok = produce_layer0<F16, Act>(nx0, nx1, chunk, tmem_warp, s, cx,
                                                          small)))
            break;
          // output layer: u = w.v + b, lap = w.L, over this warp's 16 neurons (pairs of
          // neuron slots i, i + 1 = neurons o, o + 1; the sums in neuron order)
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int o = 16 * (i >> 2) + 4 * s + (i & 3);
            float za, zb, va, vb, j0a, j0b, j1a, j1b, la, lb;
            add2o(za, zb, d[0][i], d[0][i + 1], bias[o], bias[o + 1]);
            Act::jet_fast2(za, zb, d[1][i], d[1][i + 1], d[2][i], d[2][i + 1], d[3][i],
                           d[3][i + 1], va, vb, j0a, j0b, j1a, j1b, la, lb);
            const float wa = small[kSmWout + o], wb = small[kSmWout + o + 1];
            pu = fmaf(wa, va, pu);
            pl = fmaf(wa, la, pl);
            pu = fmaf(wb, vb, pu);
            pl = fmaf(wb, lb, pl);
          }
        }
        {
          red[s * kTile + row] = pu;
          red[(4 + s) * kTile + row] = pl;
          __syncwarp();
          if (lane == 0) mbar_arrive(cx.red);
          // The s = 0 warps finish the tile. Nobody rewrites `red` before they are done:
          // the next tile's output stage needs the next tile's chunks from them first.
          if (s == 0) {
            if (!(ok = warp_wait(cx.red, tile_count & 1u, cx))) break;
            if (active) {
              float uu = small[kSmBout], ll = 0.0f;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uu += red[k * kTile + row];
                ll += red[(4 + k) * kTile + row];
              }
              u_out[p] = uu;
              lap_out[p] = ll;
            }
          }
        }
      }
    }

  }
  // ---- teardown: every warp arrives here (all waits are bounded); free TMEM ----
  // On the normal path each warp waited for the last dfull phase, so every MMA finished.
  // After an abort, MMAs issued before it may still run: give them time to drain (they
  // take microseconds) before the columns are released.
  tc::fence_before_sync();
  __syncthreads();
  if (*cx.abort_flag) {
    const uint64_t start = global_timer_ns();
    while (global_timer_ns() - start < 2000000ull) {
    }
  }
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(cx.tmem, kTmemCols);
  }
}

}  // namespace

template <bool F16, class Act>
cudaError_t set_attributes() {
  // The setmaxnreg split assumes kLaunchRegs per thread at launch; a build with fewer would
  // leave the epilogue's register raise waiting forever, so it is refused here.
  cudaFuncAttributes attr;
  const cudaError_t e = cudaFuncGetAttributes(&attr, forward_tc_kernel<F16, Act>);
  if (e != cudaSuccess) return e;
  if (attr.numRegs != kLaunchRegs) return cudaErrorInvalidKernelImage;
  return cudaFuncSetAttribute(forward_tc_kernel<F16, Act>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Layout<F16>::kSmemBytes);
}

cudaError_t prepare_forward_tc() {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {set_attributes<true, TanhAct>(), set_attributes<false, TanhAct>(),
                        set_attributes<false, SiluAct>()})
    if (e == cudaSuccess) e = r;
  return e;
}

cudaError_t launch_forward_tc(const float* coords, const float* params, float* u, float* lap,
                              int64_t n, bool f16, int activation, const DeviceInfo& dev,
                              cudaStream_t stream) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sms));
  const int aligned = (reinterpret_cast<uintptr_t>(params) % 16) == 0;
  if (activation == FHB_ACTIVATION_SILU) {  // unbounded activations: the 3xTF32 format
    forward_tc_kernel<false, SiluAct><<<grid, kBlockThreads, Layout<false>::kSmemBytes, stream>>>(
        coords, params, u, lap, n, tiles, aligned, dev.status);
  } else if (f16) {
    forward_tc_kernel<true, TanhAct><<<grid, kBlockThreads, Layout<true>::kSmemBytes, stream>>>(
        coords, params, u, lap, n, tiles, aligned, dev.status);
  } else {
    forward_tc_kernel<false, TanhAct><<<grid, kBlockThreads, Layout<false>::kSmemBytes, stream>>>(
        coords, params, u, lap, n, tiles, aligned, dev.status);
  }
  return cudaGetLastError();
}

}  // namespace fhb
