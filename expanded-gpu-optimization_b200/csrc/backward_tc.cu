// Tensor-core adjoint-jet backward and fused Poisson step (backward version 6).
//
// Math: the reverse pass of the reference backward (csrc/fused_backward.cu:15-33 adjoint
// formulas, :208-233 output seed, :262-321 weight gradient and input adjoint, :324-359 layer
// 0), on 128-point tiles with the two per-point contractions on the tensor cores:
//   * forward recompute Z_l = H_{l-1} W_l^T (the forward kernel's 3xTF32 tcgen05 GEMMs);
//   * input adjoint Hbar_{l-1} = Zbar_l W_l, also a 3xTF32 tcgen05 GEMM (M = 128 points,
//     N = 64, K = 64) whose B operand is W_l^T;
// and the third, dW_l = sum over points and jet components of zbar_l (x) h_{l-1}, on the
// FP32 CUDA cores (a reduction over points: its operands would have to be transposed into
// shared memory for the tensor core, and shared memory is full).
//
// Where the data lives (one CTA per SM, persistent over tiles):
//   * TMEM exactly as in the forward kernel: accumulators D_c at columns 64c..64c+63, a ring
//     of two A-operand chunks (16 K positions x 4 components x hi/lo) at [256, 512);
//   * shared memory: three weight slots (hi + lo, 32 KB each). A slot holds W_l for the
//     forward GEMM and W_l^T for the backward one: both are K-major B operands (the
//     tensor core's MN-major tf32 operand form is not used). A one-thread bulk copy reloads
//     a slot from a pre-split global copy of all six operands as soon as the GEMM that
//     used it has completed, long before the next GEMM needs it;
//   * per-CTA scratch in global memory, small enough to stay in L2 (512 KB per CTA): the
//     activations h_0, h_1, h_2 written during the forward recompute and zbar_l of the
//     current layer, as [component][point half][neuron][64 points] planes whose 16-byte
//     point groups are XOR-swizzled by neuron (conflict-free shared-memory reads after a
//     plain bulk copy). The adjoint reads its own h values back from there; the weight
//     gradient stages (component, point-half) planes of zbar and h through two 32 KB
//     shared-memory buffers filled by bulk copies one round ahead;
//   * registers: per thread one point (TMEM lane) and 16 neurons 16a+4s+t, as in the
//     forward kernel; 8 weight-gradient entries per layer, folded into a shared-memory
//     accumulator at the end of every layer of every tile.
// The adjoint is written in terms of the stored activation h = (a, a'z_J, L-part) rather
// than the pre-activation: with s = 1 - a^2 it needs a, s, h_J and h_L only, the same
// quantities the forward produced, so nothing else is stored.
// Reductions over points are in a fixed order (warp butterflies, then quadrants in index
// order, then tiles in loop order, then one partial row per CTA summed in row order), so
// results are bitwise reproducible for a given grid. Every wait is bounded; a wait that
// gives up sets the CTA abort flag, the warps leave together at the next block-wide
// barrier, and TMEM is freed.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace fhb {
namespace {

constexpr int kTile = 128;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kChunks = 4;                       // 16-neuron chunks per 64-wide GEMM
constexpr int kGemmsPerTile = 6;                 // forward W1..W3, backward W3^T, W2^T, W1^T
constexpr int kChunksPerTile = kGemmsPerTile * kChunks;
constexpr int kRing = 2;
constexpr uint32_t kSlotCols = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kRingCol = 256;
constexpr uint32_t kIdesc = tc::idesc_tf32(128, 64);
constexpr uint32_t kLbo = 128, kSbo = 2048;      // K-major no-swizzle canonical operand

constexpr int kOperandBytes = kWidth * kWidth * 4;   // 16 KB
constexpr int kLayerBytes = 2 * kOperandBytes;       // hi + lo
constexpr int kWeightBlocks = 6;                     // W1, W2, W3, W1^T, W2^T, W3^T

// Scratch planes (floats): [component 4][half 2][neuron 64][point 64 + 1 pad]. The pad
// makes rows 8 apart 8 banks apart, so the weight-gradient reads are conflict-free.
constexpr int kRowFloats = 65;
constexpr int kPlaneFloats = kWidth * kRowFloats;
constexpr int kJetFloats = 4 * 2 * kPlaneFloats;     // one activation jet of a tile: 128 KB
constexpr int kScratchJets = 4;                      // h0, h1, h2, zbar

// Shared memory (bytes).
constexpr int kWOff = 0;                                  // 3 weight slots
constexpr int kStageOff = 3 * kLayerBytes;                // 2 x (zbar plane, h plane)
constexpr int kStageBytes = 2 * kPlaneFloats * 4;         // 32.5 KB
constexpr int kAccOff = kStageOff + 2 * kStageBytes;      // dW accumulators [3][8][512]
constexpr int kSmallOff = kAccOff + 3 * 8 * kThreads * 4; // parameters for elementwise work
constexpr int kSmW0 = 0, kSmB0 = 128, kSmB = 192, kSmWout = 384, kSmBout = 448;
constexpr int kSmallFloats = 512;
constexpr int kGradOff = kSmallOff + kSmallFloats * 4;    // small-gradient accumulators
constexpr int kGW0 = 0, kGBias = 128, kGWout = 384, kGBout = 448, kGLoss = 449;
constexpr int kGradFloats = 512;
constexpr int kRedOff = kGradOff + kGradFloats * 4;       // [8][128]: output sums, dx
constexpr int kPartOff = kRedOff + 8 * kTile * 4;         // per-quadrant partials
constexpr int kPWout = 0, kPB0 = 256, kPW0x = 512, kPW0y = 768, kPLoss = 1024, kPBout = 1028;
constexpr int kPartFloats = 1032;
constexpr int kXsOff = kPartOff + kPartFloats * 4;        // the tile's points: x[512], y[512]
constexpr int kBarOff = kXsOff + 2 * kThreads * 4;        // empty[2] dfull red wfull[3] stage[2]
constexpr int kNumBars = 9;
constexpr int kCountOff = kBarOff + kNumBars * 8;
constexpr int kMiscOff = kCountOff + 4 * 4;               // TMEM base, abort flag
constexpr int kSmemBytes = kMiscOff + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory layout overflow");
static_assert(kStageOff % 1024 == 0 && kAccOff % 16 == 0 && kBarOff % 8 == 0, "alignment");
static_assert((kPlaneFloats * 4) % 16 == 0, "bulk copies move whole 16-byte units");

// Shared-memory objects are addressed as constant offsets of the dynamic shared-memory base
// (no pointers kept in registers across the tile loop).
__device__ __forceinline__ uint8_t* dsmem() {
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  return smem_dyn;
}
__device__ __forceinline__ uint64_t* bar_at(int k) {
  return reinterpret_cast<uint64_t*>(dsmem() + kBarOff) + k;
}
__device__ __forceinline__ uint64_t* bar_empty(uint32_t r) { return bar_at(static_cast<int>(r)); }
__device__ __forceinline__ uint64_t* bar_dfull() { return bar_at(kRing); }
__device__ __forceinline__ uint64_t* bar_red() { return bar_at(kRing + 1); }
__device__ __forceinline__ uint64_t* bar_wfull(int k) { return bar_at(kRing + 2 + k); }
__device__ __forceinline__ uint64_t* bar_stage(int b) { return bar_at(kRing + 5 + b); }
__device__ __forceinline__ uint32_t* ring_count(uint32_t r) {
  return reinterpret_cast<uint32_t*>(dsmem() + kCountOff) + r;
}
__device__ __forceinline__ volatile uint32_t* abort_flag() {
  return reinterpret_cast<volatile uint32_t*>(dsmem() + kMiscOff + 4);
}
__device__ __forceinline__ unsigned int** status_slot() {
  return reinterpret_cast<unsigned int**>(dsmem() + kMiscOff + 8);
}

struct Ctx {
  uint32_t tmem;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Ctx& cx) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag()) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      *abort_flag() = 1u;
      report_status(*status_slot(), FHB_STATUS_MMA_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform bounded wait (the tcgen05 ld/st and elect.sync after it need the whole warp).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const Ctx& cx) {
  return __all_sync(0xffffffffu, wait_or_abort(bar, parity, cx) ? 1 : 0) != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t count_contribution(uint32_t* counter) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
               : "=r"(old)
               : "r"(smem_u32(counter))
               : "memory");
  return old;
}

// Generic-proxy global writes of this thread -> visible to later bulk copies (async proxy).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Block-wide barrier that also tells every warp whether any warp has aborted.
__device__ __forceinline__ bool barrier_ok(const Ctx& cx) {
  return __syncthreads_or(*abort_flag() != 0u ? 1 : 0) == 0;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tc::to_tf32(x);
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// Weight slot used by GEMM g of a tile and the parity of the slot load it needs: slot l-1
// holds W_l (forward GEMM g = l-1, even load) then W_l^T (backward GEMM g = 6-l, odd load).
__device__ __forceinline__ int weight_slot(int g) { return g < 3 ? g : 5 - g; }

// The 24 MMAs of chunk j of GEMM g (A from ring slot `slot`); the first chunk of a GEMM
// first waits for its weight slot. False if that wait gave up (nothing is issued).
__device__ __forceinline__ bool issue_chunk_mmas(const Ctx& cx, int g, int j, uint32_t slot) {
  const int ws = weight_slot(g);
  if (j == 0 && !warp_wait(bar_wfull(ws), g >= 3 ? 1u : 0u, cx)) return false;
  tc::fence_after_sync();
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const uint32_t w_hi = smem_u32(dsmem() + kWOff + ws * kLayerBytes + 256 * (2 * j + kk));
    const uint64_t bhi = tc::smem_desc_kmajor(w_hi, kLbo, kSbo);
    const uint64_t blo = tc::smem_desc_kmajor(w_hi + kOperandBytes, kLbo, kSbo);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t d = cx.tmem + 64u * c;
      const uint32_t a_hi = cx.tmem + kRingCol + kSlotCols * slot + 32u * c + 8u * kk;
      const uint32_t a_lo = a_hi + 16u;
      tc::mma_tf32_ts_warp(d, a_hi, bhi, kIdesc, (j > 0 || kk > 0) ? 1u : 0u);
      tc::mma_tf32_ts_warp(d, a_lo, bhi, kIdesc, 1u);
      tc::mma_tf32_ts_warp(d, a_hi, blo, kIdesc, 1u);
    }
  }
  tc::commit_warp(bar_empty(slot));
  if (j == kChunks - 1) tc::commit_warp(bar_dfull());
  return true;
}

// Write chunk `n` (this warp's 4 neurons x 4 components, hi and lo) into ring slot n % 2;
// the warp completing the chunk last issues its MMAs. False if a wait gave up.
__device__ __forceinline__ bool produce_chunk(uint32_t n, const float (&h)[4][4],
                                              uint32_t tmem_warp, int s, const Ctx& cx) {
  const uint32_t slot = n % kRing;
  if (!warp_wait(bar_empty(slot), ((n / kRing) & 1u) ^ 1u, cx)) return false;
  tc::fence_after_sync();
  const uint32_t base = tmem_warp + kRingCol + kSlotCols * slot + 4u * s;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) split_tf32(h[c][t], hi[t], lo[t]);
    tc::st_x4(base + 32u * c, hi[0], hi[1], hi[2], hi[3]);
    tc::st_x4(base + 32u * c + 16u, lo[0], lo[1], lo[2], lo[3]);
  }
  tc::wait_st();
  tc::fence_before_sync();
  __syncwarp();
  uint32_t last = 0;
  if ((threadIdx.x & 31) == 0) last = (count_contribution(ring_count(slot)) % kWarps) == kWarps - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  bool ok = true;
  if (last) {
    tc::fence_after_sync();
    const uint32_t in_tile = n % kChunksPerTile;
    ok = issue_chunk_mmas(cx, static_cast<int>(in_tile / kChunks),
                          static_cast<int>(in_tile % kChunks), slot);
    __syncwarp();
  }
  return ok;
}

// Adjoint of the tanh jet in terms of the activation it produced. With h = (a, h_J0, h_J1,
// h_L), s = 1 - a^2 and the upstream adjoint (gv, g0, g1, gl) of h, the pre-activation
// adjoint is (same formulas as tanh_jet_adjoint after substituting h_J = s z_J and
// h_L = s z_L - 2 a s |z_J|^2):
//   zbar_v = gv s - 2 a (g . h_J) - 2 gl (a h_L + |h_J|^2)
//   zbar_Jd = gd s - 4 a gl h_Jd,   zbar_L = gl s.
__device__ __forceinline__ void adjoint_h(float a, float hj0, float hj1, float hl, float& gv,
                                          float& g0, float& g1, float& gl) {
  const float s = fmaf(-a, a, 1.0f);
  const float gj = fmaf(g0, hj0, g1 * hj1);
  const float t = fmaf(a, hl, fmaf(hj0, hj0, hj1 * hj1));
  const float zv = fmaf(gv, s, -2.0f * fmaf(a, gj, gl * t));
  const float f = 4.0f * a * gl;
  const float z0 = fmaf(g0, s, -f * hj0);
  const float z1 = fmaf(g1, s, -f * hj1);
  gl = gl * s;
  gv = zv;
  g0 = z0;
  g1 = z1;
}

// One weight-gradient round over a staged (component, point-half) plane pair. Thread
// (warp w, lane) owns the 8x8 block o = o0 + jj, i = i0 + kk (o0 = 8*(w>>1),
// i0 = 8*(4*(w&1) + lane/8)) and the interleaved point slice p = sl + 8m (sl = lane%8,
// m < 8) of the plane's 64 points: acc[jj][kk] += zbar[o][p] h[i][p]. Per point a warp
// reads 8 consecutive words of one zbar row (broadcast to the 4 blocks) and of 4 h rows 8
// apart, which the 65-float row stride puts 8 banks apart. kBias: also sum zbar into db.
template <bool kBias>
__device__ __forceinline__ void dw_round(const float* __restrict__ zs,
                                         const float* __restrict__ hs, int o0, int i0,
                                         int sl, float (&acc)[8][8], float (&db)[8]) {
  const float* zrow = zs + o0 * kRowFloats + sl;
  const float* hrow = hs + i0 * kRowFloats + sl;
#pragma unroll 1
  for (int m = 0; m < 8; ++m) {
    float zv[8], hv[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) zv[jj] = zrow[jj * kRowFloats + 8 * m];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) hv[kk] = hrow[kk * kRowFloats + 8 * m];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) acc[jj][kk] = fmaf(zv[jj], hv[kk], acc[jj][kk]);
    if (kBias) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) db[jj] += zv[jj];
    }
  }
}

// Sum acc[8][8] over the 8 lanes of a point slice group (lane bits 0..2) by a fixed
// reduce-scatter: lane sl ends with out[v] = sum for jj = 4*b2 + 2*b0 + (v>>2),
// kk = 4*b1 + (v&3), where b_k is bit k of sl.
__device__ __forceinline__ void reduce_scatter_slices(float (&acc)[8][8], int sl,
                                                      float (&out)[8]) {
  const bool b2 = (sl & 4) != 0, b1 = (sl & 2) != 0, b0 = (sl & 1) != 0;
  float r4[4][8];  // jj' = jj - 4*b2
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float keep = b2 ? acc[4 + j][k] : acc[j][k];
      const float send = b2 ? acc[j][k] : acc[4 + j][k];
      r4[j][k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  float r2[4][4];  // kk' = kk - 4*b1
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float keep = b1 ? r4[j][4 + k] : r4[j][k];
      const float send = b1 ? r4[j][k] : r4[j][4 + k];
      r2[j][k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float keep = b0 ? r2[2 + j][k] : r2[j][k];
      const float send = b0 ? r2[j][k] : r2[2 + j][k];
      out[4 * j + k] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
    }
}

__device__ __forceinline__ void load_weight_slot(const Ctx& cx, int slot, const float* src) {
  mbar_arrive_expect_tx(bar_wfull(slot), kLayerBytes);
  bulk_copy_g2s(dsmem() + kWOff + slot * kLayerBytes, src, kLayerBytes, bar_wfull(slot));
}

// Round r of a layer's weight gradient: plane (c = r/2, half = r%2) of zbar and of h into
// staging buffer r % 2.
__device__ __forceinline__ void issue_round(const Ctx& cx, int r, const float* zsrc,
                                            const float* hsrc) {
  const int b = r & 1;
  uint8_t* dst = dsmem() + kStageOff + b * kStageBytes;
  const int plane = (r >> 1) * 2 + (r & 1);
  mbar_arrive_expect_tx(bar_stage(b), kStageBytes);
  bulk_copy_g2s(dst, zsrc + plane * kPlaneFloats, kPlaneFloats * 4, bar_stage(b));
  bulk_copy_g2s(dst + kPlaneFloats * 4, hsrc + plane * kPlaneFloats, kPlaneFloats * 4,
                bar_stage(b));
}

// Pre-split weights for the tensor-core backward: six K-major canonical tf32 operands, hi
// then lo, of W1, W2, W3 ([out][in], forward GEMMs) and W1^T, W2^T, W3^T ([in][out], input
// adjoint GEMMs). Element e of an operand sits at word e (row = ((e>>9)<<3)|((e>>2)&7),
// K = (((e>>5)&15)<<2)|(e&3)), the layout of the forward kernel's shared-memory operands.
__global__ void __launch_bounds__(256) prep_weights_kernel(const float* __restrict__ params,
                                                           float* __restrict__ wsplit) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= kWeightBlocks * 4096) return;
  const int blk = idx >> 12, e = idx & 4095;
  const int layer = blk % 3;
  const int row = ((e >> 9) << 3) | ((e >> 2) & 7);
  const int k = (((e >> 5) & 15) << 2) | (e & 3);
  const float* W = params + kHiddenBase + layer * kHiddenStride;
  const float w = blk >= 3 ? W[k * kWidth + row] : W[row * kWidth + k];
  const uint32_t hi = tc::to_tf32(w);
  const uint32_t lo = tc::to_tf32(w - __uint_as_float(hi));
  wsplit[blk * 8192 + e] = __uint_as_float(hi);
  wsplit[blk * 8192 + 4096 + e] = __uint_as_float(lo);
}

template <bool kPoisson>
__global__ void __launch_bounds__(kThreads, 1)
    backward_tc_kernel(const float* __restrict__ coords, const float* __restrict__ params,
                       const float* __restrict__ wsplit, const float* __restrict__ grad_u,
                       const float* __restrict__ grad_lap, float* __restrict__ grad_coords,
                       float* __restrict__ lap_out, float* __restrict__ partials,
                       float* __restrict__ scratch, int64_t n, int64_t tiles, float inv_total,
                       unsigned int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  float* small = reinterpret_cast<float*>(smem + kSmallOff);
  float* grad = reinterpret_cast<float*>(smem + kGradOff);
  float* red = reinterpret_cast<float*>(smem + kRedOff);
  float* part = reinterpret_cast<float*>(smem + kPartOff);
  float* dwacc = reinterpret_cast<float*>(smem + kAccOff);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  Ctx cx;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // ---- set-up ----
  for (int i = tid; i < 3 * 8 * kThreads; i += kThreads) dwacc[i] = 0.0f;
  for (int i = tid; i < kGradFloats; i += kThreads) grad[i] = 0.0f;
  for (int i = tid; i < kSmallFloats; i += kThreads) {
    float v = 0.0f;
    if (i < kSmB0) v = params[i];                                       // W0
    else if (i < kSmB) v = params[kB0 + (i - kSmB0)];                   // b0
    else if (i < kSmWout) {                                             // b1..b3
      const int l = (i - kSmB) >> 6, o = (i - kSmB) & 63;
      v = params[kHiddenBase + l * kHiddenStride + kWidth * kWidth + o];
    } else if (i < kSmBout) v = params[kOutBase + (i - kSmWout)];       // w_out
    else if (i == kSmBout) v = params[kOutBase + kWidth];               // b_out
    small[i] = v;
  }
  if (tid == 0) {
    for (uint32_t r = 0; r < kRing; ++r) {
      mbar_init(bar_empty(r), 1);
      *ring_count(r) = 0u;
    }
    mbar_init(bar_dfull(), 1);
    mbar_init(bar_red(), kWarps);
    for (int k = 0; k < 3; ++k) mbar_init(bar_wfull(k), 1);
    for (int k = 0; k < 2; ++k) mbar_init(bar_stage(k), 1);
    *abort_flag() = 0u;
    *status_slot() = status;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  cx.tmem = *tmem_base_slot;
  if (tid == 0)
    for (int k = 0; k < 3; ++k) load_weight_slot(cx, k, wsplit + k * (kLayerBytes / 4));

  const int q = warp & 3;   // TMEM lane quadrant
  const int s = warp >> 2;  // neurons 16a + 4s + t
  const uint32_t tmem_warp = cx.tmem + (static_cast<uint32_t>(32 * q) << 16);
  const int row = 32 * q + lane;
  // Scratch addressing: element (component c, neuron 16a+4s+t) of this thread's point is at
  // jet + c * 2 * kPlaneFloats + a * 16 * kRowFloats + toff[t].
  int toff[4];
  {
    const int half = q >> 1, pl = 32 * (q & 1) + lane;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int nn = 4 * s + t;
      toff[t] = half * kPlaneFloats + nn * kRowFloats + pl;
    }
  }
  float* const jets = scratch + static_cast<int64_t>(blockIdx.x) * (kScratchJets * kJetFloats);
  float* const zjet = jets + 3 * kJetFloats;
  // Weight-gradient ownership (dw_round): block o0 + jj, i0 + kk over point slice sl; after
  // the slice reduction this thread holds 8 entries (reduce_scatter_slices).
  const int sl = lane & 7;
  const int o0 = 8 * (warp >> 1);
  const int i0 = 8 * (4 * (warp & 1) + (lane >> 3));
  const bool bias_thread = i0 == 0;
  const int own_o = o0 + 4 * ((sl >> 2) & 1) + 2 * (sl & 1);
  const int own_i = i0 + 4 * ((sl >> 1) & 1);

  uint32_t chunk = 0, mlayer = 0, tile_count = 0;
  uint32_t stage_fill[2] = {0u, 0u};
  bool alive = true;
  float nx0 = 0.0f, nx1 = 0.0f;
  {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kTile + row;
    if (p < n) {
      nx0 = coords[2 * p];
      nx1 = coords[2 * p + 1];
    }
  }
  for (int64_t tile = blockIdx.x; alive && tile < tiles; tile += gridDim.x, ++tile_count) {
    const bool has_next = tile + gridDim.x < tiles;
    const int64_t p = tile * kTile + row;
    const bool active = p < n;
    // This tile's point, loaded during the previous tile, is kept in shared memory so that
    // no register holds it through the weight-gradient rounds.
    float* const xs = reinterpret_cast<float*>(smem + kXsOff);
    xs[tid] = nx0;
    xs[kThreads + tid] = nx1;
    const float x0 = nx0, x1 = nx1;

    // ---- forward recompute: layer 0, then the three hidden GEMMs ----
#pragma unroll
    for (int a = 0; a < kChunks; ++a) {
      float h[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int o = 16 * a + 4 * s + t;
        const float w0 = small[kSmW0 + 2 * o], w1 = small[kSmW0 + 2 * o + 1];
        tanh_jet_fast(fmaf(w0, x0, fmaf(w1, x1, small[kSmB0 + o])), w0, w1, 0.0f, h[0][t],
                      h[1][t], h[2][t], h[3][t]);
#pragma unroll
        for (int c = 0; c < 4; ++c) jets[c * 2 * kPlaneFloats + a * 16 * kRowFloats + toff[t]] = h[c][t];
      }
      produce_chunk(chunk++, h, tmem_warp, s, cx);
    }
    float d[4][16];  // d[c][4a + t]: component c of neuron 16a + 4s + t
#pragma unroll 1
    for (int g = 0; g < 3; ++g) {
      warp_wait(bar_dfull(), mlayer & 1u, cx);
      ++mlayer;
      tc::fence_after_sync();
      // GEMM g is complete: its weight slot now takes W_{g+1}^T for the backward.
      if (tid == 0) load_weight_slot(cx, g, wsplit + (3 + g) * (kLayerBytes / 4));
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tc::ld_x4(tmem_warp + 64u * c + 16u * a + 4u * s,
                    *reinterpret_cast<float(*)[4]>(&d[c][4 * a]));
      tc::wait_ld();
      const float* bias = small + kSmB + 64 * g;
#pragma unroll
      for (int i = 0; i < 16; ++i) d[0][i] += bias[16 * (i >> 2) + 4 * s + (i & 3)];
      if (g < 2) {
        float* hjet = jets + (g + 1) * kJetFloats;
#pragma unroll
        for (int a = 0; a < kChunks; ++a) {
          float h[4][4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int i = 4 * a + t;
            tanh_jet_fast(d[0][i], d[1][i], d[2][i], d[3][i], h[0][t], h[1][t], h[2][t],
                          h[3][t]);
#pragma unroll
            for (int c = 0; c < 4; ++c) hjet[c * 2 * kPlaneFloats + a * 16 * kRowFloats + toff[t]] = h[c][t];
          }
          produce_chunk(chunk++, h, tmem_warp, s, cx);
        }
      }
    }

    // ---- output layer, loss seed, layer-3 adjoint (d becomes h3, then zbar3) ----
    {
      float pu = 0.0f, pl = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        tanh_jet_fast(d[0][i], d[1][i], d[2][i], d[3][i], d[0][i], d[1][i], d[2][i], d[3][i]);
        const float w = small[kSmWout + 16 * (i >> 2) + 4 * s + (i & 3)];
        pu = fmaf(w, d[0][i], pu);
        pl = fmaf(w, d[3][i], pl);
      }
      red[s * kTile + row] = pu;
      red[(4 + s) * kTile + row] = pl;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_red());
      warp_wait(bar_red(), tile_count & 1u, cx);
      float lap = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) lap += red[(4 + k) * kTile + row];
      float gu, gl;
      if (kPoisson) {
        // f = -2 pi^2 sin(pi x) sin(pi y)  (src/fused_hoad/problems/poisson.py:29-39)
        const float pi = 3.14159265358979323846f;
        const float f = -2.0f * pi * pi * (sinf(pi * xs[tid]) * sinf(pi * xs[kThreads + tid]));
        const float r = active ? lap - f : 0.0f;
        gu = 0.0f;
        gl = 2.0f * r * inv_total;
        if (s == 0) {
          if (active && lap_out != nullptr) lap_out[p] = lap;
          const float l2 = warp_sum(r * r);
          if (lane == 0) part[kPLoss + q] = l2;
        }
      } else {
        gu = (active && grad_u != nullptr) ? grad_u[p] : 0.0f;
        gl = active ? grad_lap[p] : 0.0f;
        if (s == 0) {
          const float sg = warp_sum(gu);
          if (lane == 0) part[kPBout + q] = sg;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int o = 16 * (i >> 2) + 4 * s + (i & 3);
        const float w = small[kSmWout + o];
        const float dwo = warp_sum(fmaf(gu, d[0][i], gl * d[3][i]));
        if (lane == 0) part[kPWout + q * 64 + o] = dwo;
        float gv = gu * w, g0 = 0.0f, g1 = 0.0f, gL = gl * w;
        adjoint_h(d[0][i], d[1][i], d[2][i], d[3][i], gv, g0, g1, gL);
        d[0][i] = gv;
        d[1][i] = g0;
        d[2][i] = g1;
        d[3][i] = gL;
      }
    }

    // ---- backward through the hidden layers: d holds zbar_l on entry ----
#pragma unroll 1
    for (int l = 3; l >= 1; --l) {
      const int g = 6 - l;
      const float* hsrc = jets + (l - 1) * kJetFloats;
      // zbar_l -> scratch (weight gradient) and ring (input-adjoint GEMM g)
#pragma unroll
      for (int a = 0; a < kChunks; ++a) {
        float z[4][4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            z[c][t] = d[c][4 * a + t];
            zjet[c * 2 * kPlaneFloats + a * 16 * kRowFloats + toff[t]] = z[c][t];
          }
        produce_chunk(chunk++, z, tmem_warp, s, cx);
      }
      fence_proxy_async_global();
      if (!(alive = barrier_ok(cx))) break;

      // weight gradient dW_l over this tile, 8 rounds of (component, point half)
      float acc[8][8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[j][k] = 0.0f;
      if (tid == 0) {
        issue_round(cx, 0, zjet, hsrc);
        issue_round(cx, 1, zjet, hsrc);
      }
      // Rounds 0 and 1 (value component) also sum zbar_v for the bias gradient.
      {
        float dbp[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) dbp[j] = 0.0f;
#pragma unroll 1
        for (int r = 0; r < 2; ++r) {
          warp_wait(bar_stage(r), stage_fill[r] & 1u, cx);
          ++stage_fill[r];
          const float* zs = reinterpret_cast<const float*>(smem + kStageOff + r * kStageBytes);
          if (bias_thread) dw_round<true>(zs, zs + kPlaneFloats, o0, i0, sl, acc, dbp);
          else dw_round<false>(zs, zs + kPlaneFloats, o0, i0, sl, acc, dbp);
          if (!(alive = barrier_ok(cx))) break;
          if (tid == 0) issue_round(cx, r + 2, zjet, hsrc);
        }
        if (bias_thread) {  // lanes 0..7 of the even warps: sum the slices of db in lane 0
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float v = dbp[j];
            v += __shfl_xor_sync(0x000000ffu, v, 4);
            v += __shfl_xor_sync(0x000000ffu, v, 2);
            v += __shfl_xor_sync(0x000000ffu, v, 1);
            dbp[j] = v;
          }
          if (sl == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) grad[kGBias + l * 64 + o0 + j] += dbp[j];
          }
        }
      }
      if (!alive) break;
#pragma unroll 1
      for (int r = 2; r < 8; ++r) {
        const int b = r & 1;
        warp_wait(bar_stage(b), stage_fill[b] & 1u, cx);
        ++stage_fill[b];
        const float* zs = reinterpret_cast<const float*>(smem + kStageOff + b * kStageBytes);
        float unused[8];
        dw_round<false>(zs, zs + kPlaneFloats, o0, i0, sl, acc, unused);
        if (!(alive = barrier_ok(cx))) break;
        if (tid == 0 && r + 2 < 8) issue_round(cx, r + 2, zjet, hsrc);
      }
      if (!alive) break;
      {
        float sums[8];
        reduce_scatter_slices(acc, sl, sums);
#pragma unroll
        for (int v = 0; v < 8; ++v) dwacc[((l - 1) * 8 + v) * kThreads + tid] += sums[v];
      }

      // input adjoint hbar_{l-1} = zbar_l W_l (GEMM g), then zbar_{l-1}
      float hn[4][4];  // h_{l-1} of the next neuron group, loaded ahead of use
      if (l > 1) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int c = 0; c < 4; ++c) hn[c][t] = hsrc[c * 2 * kPlaneFloats + toff[t]];
      }
      warp_wait(bar_dfull(), mlayer & 1u, cx);
      ++mlayer;
      tc::fence_after_sync();
      // GEMM g is complete: its slot takes W_l again for the next tile's forward.
      if (tid == 0 && has_next)
        load_weight_slot(cx, weight_slot(g), wsplit + (l - 1) * (kLayerBytes / 4));
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tc::ld_x4(tmem_warp + 64u * c + 16u * a + 4u * s,
                    *reinterpret_cast<float(*)[4]>(&d[c][4 * a]));
      tc::wait_ld();
      if (l > 1) {
#pragma unroll
        for (int a = 0; a < kChunks; ++a) {
          float h[4][4];
#pragma unroll
          for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int c = 0; c < 4; ++c) h[c][t] = hn[c][t];
          if (a + 1 < kChunks) {
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
              for (int c = 0; c < 4; ++c)
                hn[c][t] = hsrc[c * 2 * kPlaneFloats + (a + 1) * 16 * kRowFloats + toff[t]];
          }
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int i = 4 * a + t;
            adjoint_h(h[0][t], h[1][t], h[2][t], h[3][t], d[0][i], d[1][i], d[2][i], d[3][i]);
          }
        }
      }
    }
    if (!alive) break;

    // The next tile's point: loaded now, used at the next tile's start.
    {
      const int64_t pn = p + static_cast<int64_t>(gridDim.x) * kTile;
      if (pn < n) {
        nx0 = coords[2 * pn];
        nx1 = coords[2 * pn + 1];
      }
    }

    // ---- layer 0: z_v = W0 x + b0, z_J = W0, z_L = 0; d holds hbar_0 ----
    {
      const float x0 = xs[tid], x1 = xs[kThreads + tid];
      float gx0 = 0.0f, gx1 = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int o = 16 * (i >> 2) + 4 * s + (i & 3);
        const float w0 = small[kSmW0 + 2 * o], w1 = small[kSmW0 + 2 * o + 1];
        float a, hj0, hj1, hl;
        tanh_jet_fast(fmaf(w0, x0, fmaf(w1, x1, small[kSmB0 + o])), w0, w1, 0.0f, a, hj0, hj1,
                      hl);
        float gv = d[0][i], g0 = d[1][i], g1 = d[2][i], gL = d[3][i];
        adjoint_h(a, hj0, hj1, hl, gv, g0, g1, gL);
        const float db = warp_sum(gv);
        const float d0 = warp_sum(fmaf(gv, x0, g0));
        const float d1 = warp_sum(fmaf(gv, x1, g1));
        if (lane == 0) {
          part[kPB0 + q * 64 + o] = db;
          part[kPW0x + q * 64 + o] = d0;
          part[kPW0y + q * 64 + o] = d1;
        }
        gx0 = fmaf(w0, gv, gx0);
        gx1 = fmaf(w1, gv, gx1);
      }
      red[s * kTile + row] = gx0;
      red[(4 + s) * kTile + row] = gx1;
    }
    if (!(alive = barrier_ok(cx))) break;
    if (s == 0 && active && grad_coords != nullptr) {
      float sx = 0.0f, sy = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        sx += red[k * kTile + row];
        sy += red[(4 + k) * kTile + row];
      }
      grad_coords[2 * p] = sx;
      grad_coords[2 * p + 1] = sy;
    }
    if (tid < 4 * kWidth) {
      const int kind = tid >> 6, o = tid & 63;
      const int base = kind == 0 ? kPWout : kind == 1 ? kPB0 : kind == 2 ? kPW0x : kPW0y;
      const float v = ((part[base + o] + part[base + 64 + o]) + part[base + 128 + o]) +
                      part[base + 192 + o];
      if (kind == 0) grad[kGWout + o] += v;
      else if (kind == 1) grad[kGBias + o] += v;
      else grad[kGW0 + 2 * o + (kind - 2)] += v;
    } else if (tid == 4 * kWidth) {
      if (kPoisson) {
        grad[kGLoss] += (((part[kPLoss] + part[kPLoss + 1]) + part[kPLoss + 2]) + part[kPLoss + 3]) *
                        inv_total;
      } else {
        grad[kGBout] +=
            ((part[kPBout] + part[kPBout + 1]) + part[kPBout + 2]) + part[kPBout + 3];
      }
    }
    if (!(alive = barrier_ok(cx))) break;
  }

  // ---- teardown: free TMEM (after an abort, let issued MMAs and copies drain first) ----
  const bool aborted = *abort_flag() != 0u;
  tc::fence_before_sync();
  __syncthreads();
  if (aborted) {
    const uint64_t start = global_timer_ns();
    while (global_timer_ns() - start < 2000000ull) {
    }
  }
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(cx.tmem, kTmemCols);
  }
  if (aborted) return;

  // ---- this CTA's partial-gradient row, in the packed ABI layout ----
  float* rowp = partials + static_cast<int64_t>(blockIdx.x) * kRowStride;
#pragma unroll
  for (int l = 0; l < 3; ++l)
#pragma unroll
    for (int v = 0; v < 8; ++v)
      rowp[kHiddenBase + l * kHiddenStride + (own_o + (v >> 2)) * kWidth + own_i + (v & 3)] =
          dwacc[(l * 8 + v) * kThreads + tid];
  for (int k = tid; k < 2 * kWidth; k += kThreads) rowp[k] = grad[kGW0 + k];
  if (tid < kWidth) {
    rowp[kB0 + tid] = grad[kGBias + tid];
#pragma unroll
    for (int l = 1; l < 4; ++l)
      rowp[kHiddenBase + (l - 1) * kHiddenStride + kWidth * kWidth + tid] =
          grad[kGBias + l * kWidth + tid];
    rowp[kOutBase + tid] = grad[kGWout + tid];
  }
  if (tid == 0) {
    rowp[kOutBase + kWidth] = grad[kGBout];
    rowp[kLossColumn] = grad[kGLoss];
  }
}

}  // namespace

cudaError_t prepare_backward_tc() {
  cudaError_t e = cudaFuncSetAttribute(backward_tc_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(backward_tc_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  return e;
}

int backward_tc_grid(int64_t n, const DeviceInfo& dev) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  return static_cast<int>(std::min<int64_t>(tiles, dev.sms));
}

size_t backward_tc_workspace_bytes(int64_t n, const DeviceInfo& dev) {
  const size_t grid = static_cast<size_t>(backward_tc_grid(n, dev));
  return (static_cast<size_t>(kWeightBlocks) * (kLayerBytes / 4) + grid * kRowStride +
          grid * kScratchJets * kJetFloats) *
         sizeof(float);
}

cudaError_t launch_backward_tc(const float* coords, const float* params, const float* grad_u,
                               const float* grad_lap, float* grad_coords, float* lap_out,
                               float* workspace, int64_t n, int64_t n_total, bool poisson,
                               const DeviceInfo& dev, cudaStream_t stream) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int grid = backward_tc_grid(n, dev);
  float* wsplit = workspace;
  float* partials = wsplit + kWeightBlocks * (kLayerBytes / 4);
  float* scratch = partials + static_cast<size_t>(grid) * kRowStride;
  prep_weights_kernel<<<(kWeightBlocks * 4096 + 255) / 256, 256, 0, stream>>>(params, wsplit);
  const float inv_total =
      n_total > 0 ? static_cast<float>(1.0 / static_cast<double>(n_total)) : 0.0f;
  if (poisson) {
    backward_tc_kernel<true><<<grid, kThreads, kSmemBytes, stream>>>(
        coords, params, wsplit, nullptr, nullptr, grad_coords, lap_out, partials, scratch, n,
        tiles, inv_total, dev.status);
  } else {
    backward_tc_kernel<false><<<grid, kThreads, kSmemBytes, stream>>>(
        coords, params, wsplit, grad_u, grad_lap, grad_coords, nullptr, partials, scratch, n,
        tiles, 0.0f, dev.status);
  }
  return cudaGetLastError();
}

float* backward_tc_partials(float* workspace) {
  return workspace + kWeightBlocks * (kLayerBytes / 4);
}

}  // namespace fhb
