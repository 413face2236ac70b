// Tensor-core adjoint-jet backward and fused Poisson step (backward version 6).
//
// Math: the reverse pass of the reference backward (csrc/fused_backward.cu:15-33 adjoint
// formulas, :208-233 output seed, :262-321 weight gradient and input adjoint, :324-359 layer
// 0), on 128-point tiles with all three per-layer contractions on the tensor cores, as f16
// hi/lo operand pairs (x = hi + lo with power-of-2 range scales; the products keep ~22
// significant bits):
//   * forward recompute  Z_l[128 x 64] = H_{l-1} W_l^T   (3xFP16 as the forward kernel's
//     version 3: A = sigma-scaled H in TMEM, B = tau-scaled W_l in shared memory, M = 128
//     points, N = 64, K = 64 per component in chunks of 16);
//   * input adjoint      Hbar_{l-1} = Zbar_l W_l           (3xFP16: A = Zbar scaled per point
//     half and component, in TMEM; B = tau-scaled W_l^T);
//   * weight gradient    dW_l[64 x 64] = sum over points and components of zbar h^T, as
//     M = 128 rows (zbar_hi rows 0..63, zbar_lo rows 64..127) x N = 128 columns (h_hi,
//     h_lo) x K = points: one f16 MMA per 16 points gives all four hi/lo products in four
//     quadrants of the accumulator, summed when it is emptied. A and B are written by the
//     threads straight from registers into two shared-memory staging buffers (MN-major: a
//     thread's 8 neuron rows of one point are one 16-byte store), one per point half, one jet
//     component at a time. The halves run independently (named barriers, one commit barrier
//     each), so one half stages its next component while the tensor core works through the
//     other half's MMAs.
//
// Where the data lives (one CTA per SM, persistent over tiles, clusters of 2 CTAs):
//   * TMEM: accumulators D_c at columns 64c..64c+63 and a ring of four A-operand chunks at
//     [256, 512) (a GEMM's whole A operand). The two weight-gradient accumulators (one per
//     point half) borrow the ring while it is idle (after the input-adjoint GEMM of the
//     layer has completed, before the next layer's chunks) and are emptied every layer;
//   * shared memory: two weight slots (f16 hi + lo, 16 KB each), the six operands of a
//     tile's GEMMs (W1, W2, W3, then W3^T, W2^T, W1^T; all K-major) taking turns: a one-thread
//     bulk copy reloads a slot from a pre-split global copy as soon as the GEMM that used it
//     has completed, two GEMMs before the slot is needed again; the staging buffers; the
//     CTA's hidden-layer weight gradients (48 KB), summed over the cluster at the end through
//     distributed shared memory into one partial row per cluster;
//   * per-CTA scratch in global memory, 256 KB per CTA so it stays in L2: h_1 and h_2 of the
//     tile, written during the forward recompute in a thread-private coalesced layout and
//     read back by the same thread for the adjoint and the weight-gradient staging (h_0 is
//     recomputed from the point);
//   * registers: per thread one point (TMEM lane) and the 16 neurons 16a+4s+t.
// Warps: 16 epilogue warps (all of the elementwise work above; warp w serves TMEM lane
// quadrant w%4 and, with s = w/4, neurons 16a+4s+t) and an MMA warpgroup (warps 16-19) whose
// warp 16 issues the 12 MMAs of every chunk in order once the chunk's 16 arrivals are in.
// The weight-gradient rounds stay with one epilogue warp per point half, which issues right
// after its half's barrier (handing them to the MMA warpgroup serialised them behind two
// mbarrier wake-ups per round). The MMA warpgroup gives its registers to the epilogue with
// setmaxnreg (launch 640 x 96, MMA warpgroup 32, epilogue 112); the host refuses a build
// whose launch register count is not the 96 the split assumes.
// The adjoint is written in terms of the stored activation h = (a, s z_J, s z_L - 2as|z_J|^2)
// with s = 1 - a^2, the quantities the forward produced, so no pre-activation is stored.
// Gradients are accumulated in a fixed order (warp butterflies, quadrants and tiles in
// index order, the tensor core's own order for the weight gradient, the cluster's CTAs in
// rank order, one partial row per cluster summed in row order), so results are bitwise
// reproducible for a given grid. Every wait is bounded; a wait that gives up sets the CTA
// abort flag, the epilogue warps leave together at their next barrier, the MMA warp at its
// next wait, TMEM is freed and every CTA still takes the cluster barriers.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace fhb {
namespace {

constexpr int kTile = 128;
// CTAs per cluster: the partial-gradient rows are summed over a cluster through distributed
// shared memory before they reach global memory (one row per cluster).
constexpr int kCluster = 2;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;          // epilogue threads
constexpr int kMmaWarp = kWarps;                 // warp 16: first warp of the MMA warpgroup
constexpr int kBlockThreads = kThreads + 128;
// Registers per thread: at launch (__launch_bounds__(640, 1) caps ptxas at 96), the MMA
// warpgroup after setmaxnreg.dec, the epilogue warpgroups after setmaxnreg.inc.
constexpr int kLaunchRegs = 96, kMmaRegs = 32, kEpiRegs = 112;
static_assert((kLaunchRegs - kMmaRegs) * 128 >= (kEpiRegs - kLaunchRegs) * kThreads,
              "register split exceeds the launch's registers");
constexpr int kChunks = 4;                       // 16-neuron chunks per 64-wide GEMM
constexpr int kGemmsPerTile = 6;                 // forward W1..W3, backward W3^T, W2^T, W1^T
// The ring holds the four chunks of a GEMM's A operand (f16 hi/lo pairs): every chunk's slot
// was last read by the previous GEMM, whose completion the producing warp has waited for.
constexpr int kRing = 4;
constexpr uint32_t kSlotCols = 64;               // 4 components x {hi, lo} x 8 columns of pairs
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kRingCol = 256;
constexpr uint32_t kDwCol = kRingCol;            // weight-gradient accumulators (borrowed)
constexpr uint32_t kIdesc = tc::idesc_f16(128, 64);
constexpr uint32_t kLbo = 128, kSbo = 1024;      // K-major no-swizzle canonical f16 operand

constexpr int kOperandBytes = kWidth * kWidth * 2;   // 8 KB
constexpr int kLayerBytes = 2 * kOperandBytes;       // hi + lo
constexpr int kWeightBlocks = 6;                     // W1, W2, W3, W1^T, W2^T, W3^T
constexpr int kWeightSlots = 2;

// Per-CTA scratch (floats): h_1 and h_2 as [jet 2][component 4][neuron slot 16][thread 512];
// neuron slot 4a + t of thread (warp 4s + q, lane) is neuron 16a + 4s + t of its point.
constexpr int kScratchFloats = 2 * 4 * 16 * kThreads;

// Weight-gradient staging buffer (one per point half): A = [zbar_hi; zbar_lo] and
// B = [h_hi; h_lo] as f16, 128 rows x 64 points each, MN-major without swizzle: element
// (row r, point k) at byte (r % 8) * 2 + (k % 8) * 16 + (r / 8) * kDwSbo + (k / 8) * kDwLbo,
// so the 8 rows of a 16-byte group are one thread's 8 neurons of one point. Rows 0..63 are
// the hi parts and 64..127 the lo parts of the neurons in accumulator-column order
// (neuron_of_column): row 16s + i is neuron slot i of the warps of block s.
constexpr uint32_t kDwLbo = 128, kDwSbo = 1024;
constexpr int kStageA = 0, kStageB = 16384;
constexpr int kStageBytes = 32768;
constexpr int kFlushStride = 65;                 // [64 rows][65] floats: the z_hi rows when emptying TMEM

// Shared memory (bytes).
constexpr int kWOff = 0;                                      // 2 weight slots
constexpr int kStageOff = kWeightSlots * kLayerBytes;         // 2 staging buffers
constexpr int kSmallOff = kStageOff + 2 * kStageBytes;        // parameters (elementwise)
constexpr int kSmW0 = 0, kSmB0 = 128, kSmB = 192, kSmWout = 384, kSmBout = 448;
constexpr int kSmallFloats = 512;
constexpr int kGradOff = kSmallOff + kSmallFloats * 4;        // small-gradient accumulators
constexpr int kGW0 = 0, kGBias = 128, kGWout = 384, kGBout = 448, kGLoss = 449;
constexpr int kGradFloats = 512;
constexpr int kRedOff = kGradOff + kGradFloats * 4;           // [8][128]: output sums, dx
constexpr int kPartOff = kRedOff + 8 * kTile * 4;             // per-quadrant partials [q][64]
// kinds: 0 w_out, 1 b0, 2 W0[:,0], 3 W0[:,1], 4..6 b1..b3
constexpr int kPartKinds = 7;
constexpr int kPLoss = kPartKinds * 256, kPBout = kPLoss + 4;
constexpr int kPartFloats = kPBout + 4;
constexpr int kXsOff = kPartOff + kPartFloats * 4;            // the tile's points x[512], y[512]
constexpr int kXnOff = kXsOff + 2 * kThreads * 4;             // the next tile's, same layout
// f16 operand scales: per epilogue warp its copy of the h scales sigma[3][4] (h_0, h_1, h_2;
// v, d/dx, d/dy, L) at kSig, their inverses at kInvSig, the weight scales tau[3] (W1..W3)
// at kTau and their inverses at kInvTau; then per warp the maxima of its zbar components
// (kZmaxFloats: |zbar_c| for c = 0..3, and max_c |zbar_c| / sigma_c for the weight gradient)
constexpr int kDwScaleOff = kXnOff + 2 * kThreads * 4;
constexpr int kSig = 0, kInvSig = 12, kTau = 24, kInvTau = 28;
// per layer of a tile: the weight-gradient staging scales zs / (sigma_c S_c) of the zbar_c
// already multiplied by S_c, and 1 / (S_c tau) for the input adjoint's accumulators
constexpr int kStg = 32, kIsc = 36;
constexpr int kSigFloats = 40;
constexpr int kZmaxOff = kDwScaleOff + kWarps * kSigFloats * 4;
constexpr int kZmaxFloats = 8;
// This CTA's hidden-layer weight gradients (3 x 4096; layer l's entry for accumulator
// column c and row r at 4096 l + 64 c + r), summed over its tiles; reduced over the cluster
// at the end.
constexpr int kHiddenGrads = 3 * kWidth * kWidth;
constexpr int kRowsOff = kZmaxOff + kWarps * kZmaxFloats * 4;
constexpr int kBarOff = kRowsOff + kHiddenGrads * 4;         // mbarriers
constexpr int kNumBars = 10;   // dfull red wfull[2] dwdone[2] full[4]
constexpr int kMiscOff = kBarOff + kNumBars * 8;              // TMEM base, abort flag, status
constexpr int kSmemBytes = kMiscOff + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory layout overflow");
static_assert(kStageOff % 1024 == 0 && kBarOff % 8 == 0 && (kMiscOff + 8) % 8 == 0,
              "alignment");
static_assert(64 * kFlushStride * 4 <= kStageBytes, "flush buffer fits a staging buffer");

// Shared-memory objects are addressed as constant offsets of the dynamic shared-memory base
// (no pointers kept in registers across the tile loop).
__device__ __forceinline__ uint8_t* dsmem() {
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  return smem_dyn;
}
__device__ __forceinline__ uint64_t* bar_at(int k) {
  return reinterpret_cast<uint64_t*>(dsmem() + kBarOff) + k;
}
__device__ __forceinline__ uint64_t* bar_dfull() { return bar_at(0); }
__device__ __forceinline__ uint64_t* bar_red() { return bar_at(1); }
__device__ __forceinline__ uint64_t* bar_wfull(int k) { return bar_at(2 + k); }
__device__ __forceinline__ uint64_t* bar_dwdone(int half) { return bar_at(4 + half); }
// A ring slot written by the 16 epilogue warps.
__device__ __forceinline__ uint64_t* bar_full(uint32_t r) {
  return bar_at(6 + static_cast<int>(r));
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

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_for(bar, parity, kSuspendHintNs)) return true;
    if (*abort_flag()) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      *abort_flag() = 1u;
      report_status(*status_slot(), FHB_STATUS_MMA_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform bounded wait (the tcgen05 ld/st and elect.sync after it need the whole warp).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait_or_abort(bar, parity) ? 1 : 0) != 0;
}



// Barrier 3 over the 16 epilogue warps that also tells every one of them whether any warp
// has aborted.
__device__ __forceinline__ bool barrier_ok() {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, 3, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(*abort_flag()), "n"(kThreads)
      : "memory");
  return any == 0;
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


// GEMM g of a tile (0..2: forward with W1..W3, 3..5: input adjoint with W3^T, W2^T, W1^T)
// reads weight slot g % 2. A slot serves GEMMs g, g+2, g+4 of every tile, so GEMM g of the
// tile with index t (counted per CTA) needs the slot's load number 3t + g/2.
__device__ __forceinline__ int weight_block(int g) { return g < 3 ? g : 8 - g; }
__device__ __forceinline__ uint32_t weight_parity(uint32_t tile_index, int g) {
  return (3u * tile_index + static_cast<uint32_t>(g >> 1)) & 1u;
}

__device__ __forceinline__ void load_weight_slot(int slot, const float* wsplit, int block) {
  mbar_arrive_expect_tx(bar_wfull(slot), kLayerBytes);
  bulk_copy_g2s(dsmem() + kWOff + slot * kLayerBytes, wsplit + block * (kLayerBytes / 4),
                kLayerBytes, bar_wfull(slot));
}

// The 12 MMAs of chunk j of GEMM g (A from ring slot `slot`: 4 components x (A_hi B_hi +
// A_lo B_hi + A_hi B_lo), K = 16, the component's hi block at column 16c of the slot and its
// lo block 8 columns on), issued by one elected lane in one block; the first chunk of a GEMM
// first waits for its weight slot. False if that wait gave up (nothing is issued). Not
// inlined: one copy instead of twenty-four keeps the kernel small for the instruction cache.
__device__ __noinline__ bool issue_chunk_mmas(const Ctx& cx, uint32_t tile_index, int g,
                                                 int j, uint32_t slot) {
  const int ws = g & 1;
  if (j == 0 && !warp_wait(bar_wfull(ws), weight_parity(tile_index, g))) return false;
  tc::fence_after_sync();
  const uint32_t w_hi = smem_u32(dsmem() + kWOff + ws * kLayerBytes + 256 * j);
  const uint64_t bhi = tc::smem_desc_kmajor(w_hi, kLbo, kSbo);
  const uint64_t blo = tc::smem_desc_kmajor(w_hi + kOperandBytes, kLbo, kSbo);
  tc::mma_f16_ts_chunk_warp(cx.tmem, cx.tmem + kRingCol + kSlotCols * slot, bhi, blo, kIdesc,
                            j > 0 ? 1u : 0u);
  if (j == kChunks - 1) tc::commit_warp(bar_dfull());
  return true;
}

// Write chunk `n` (this warp's 4 neurons x 4 components, already multiplied by their f16
// scales) into ring slot n % 4 as f16 hi/lo pairs: neuron 4s + t of the chunk is K index
// 4s + t, so the thread's pairs (t = 0, 1) and (t = 2, 3) are columns 2s and 2s + 1 of the
// component's hi block (16c) and lo block (16c + 8).
__device__ __forceinline__ void produce_chunk(uint32_t n, const float (&h)[4][4],
                                              uint32_t tmem_warp, int s) {
  const uint32_t slot = n % kRing;
  const uint32_t base = tmem_warp + kRingCol + kSlotCols * slot + 2u * s;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hi0, lo0, hi1, lo1;
    split_f16_pair_fast(h[c][0], h[c][1], hi0, lo0);
    split_f16_pair_fast(h[c][2], h[c][3], hi1, lo1);
    tc::st_x2(base + 16u * c, hi0, hi1);
    tc::st_x2(base + 16u * c + 8u, lo0, lo1);
  }
  tc::wait_st();
  tc::fence_before_sync();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar_full(slot));
}

// Layer 0 of the forward recompute for the point (x0, x1): z = W0 x + b0, z_J = the row of
// W0, z_L = 0, through the tanh jet, times the f16 scales sg[c] of h_0, into the four chunks
// of GEMM 0's A operand.
__device__ __forceinline__ void produce_layer0(float x0, float x1, const float* small,
                                               const float* sg, uint32_t& chunk,
                                               uint32_t tmem_warp, int s) {
  const float s0 = sg[0], s1 = sg[1], s3 = sg[3];
#pragma unroll
  for (int a = 0; a < kChunks; ++a) {
    float h[4][4];
#pragma unroll
    for (int t = 0; t < 4; t += 2) {
      const int o = 16 * a + 4 * s + t;
      const float w0a = small[kSmW0 + 2 * o], w1a = small[kSmW0 + 2 * o + 1];
      const float w0b = small[kSmW0 + 2 * o + 2], w1b = small[kSmW0 + 2 * o + 3];
      float za, zb;
      fma2o(za, zb, w1a, w1b, x1, x1, small[kSmB0 + o], small[kSmB0 + o + 1]);
      fma2o(za, zb, w0a, w0b, x0, x0, za, zb);
      tanh_jet_fast2(za, zb, w0a, w0b, w1a, w1b, 0.0f, 0.0f, h[0][t], h[0][t + 1], h[1][t],
                     h[1][t + 1], h[2][t], h[2][t + 1], h[3][t], h[3][t + 1]);
    }
#pragma unroll
    for (int t = 0; t < 4; t += 2) {
      mul2(h[0][t], h[0][t + 1], s0, s0);
      mul2(h[1][t], h[1][t + 1], s1, s1);
      mul2(h[2][t], h[2][t + 1], s1, s1);
      mul2(h[3][t], h[3][t + 1], s3, s3);
    }
    produce_chunk(chunk++, h, tmem_warp, s);
  }
}

// Asynchronous copy of point `row` of tile `tile` into shared memory (x at dst[0], y at
// dst[kThreads]): cp.async with a zero source size past the end of the point set, which
// writes zeros. No register holds the point while the copy is in flight.
__device__ __forceinline__ void prefetch_point(const PointSets& ps, int64_t tile, int row,
                                               float* dst) {
  const bool b = tile >= ps.tiles;
  const int64_t p = (b ? tile - ps.tiles : tile) * kTile + row;
  const float* set = b ? ps.boundary : ps.interior;
  const bool in = p < (b ? ps.nb : ps.n);
  const float* src = in ? set + 2 * p : set;  // a valid address even when nothing is read
  const uint32_t bytes = in ? 4u : 0u;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst + kThreads)),
               "l"(src + (in ? 1 : 0)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void prefetch_wait() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Adjoint of the tanh jet in terms of the activation it produced. With h = (a, h_J0, h_J1,
// h_L), s = 1 - a^2 and the upstream adjoint (gv, g0, g1, gl) of h, the pre-activation
// adjoint is (tanh_jet_adjoint's formulas after substituting h_J = s z_J and
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

// adjoint_h of two neurons in packed pair arithmetic: bitwise the results of two adjoint_h
// calls (the same roundings in the same order; the negated products -2 (.) and -f h_Jd are
// formed as (-2) (.) and (-4 a) gl h_Jd, which round to the same magnitudes).
__device__ __forceinline__ void adjoint_h2(float a0, float a1, float hj00, float hj01,
                                           float hj10, float hj11, float hl0, float hl1,
                                           float& gv0, float& gv1, float& g00, float& g01,
                                           float& g10, float& g11, float& gl0, float& gl1) {
  float s0, s1, u0, u1, gj0, gj1, t0, t1, w0, w1, f0, f1, m0, m1;
  fma2o(s0, s1, -a0, -a1, a0, a1, 1.0f, 1.0f);
  mul2o(u0, u1, g10, g11, hj10, hj11);
  fma2o(gj0, gj1, g00, g01, hj00, hj01, u0, u1);
  mul2o(u0, u1, hj10, hj11, hj10, hj11);
  fma2o(u0, u1, hj00, hj01, hj00, hj01, u0, u1);
  fma2o(t0, t1, a0, a1, hl0, hl1, u0, u1);
  mul2o(w0, w1, gl0, gl1, t0, t1);
  fma2o(w0, w1, a0, a1, gj0, gj1, w0, w1);
  mul2o(w0, w1, -2.0f, -2.0f, w0, w1);
  fma2o(gv0, gv1, gv0, gv1, s0, s1, w0, w1);
  mul2o(f0, f1, -4.0f, -4.0f, a0, a1);
  mul2o(f0, f1, f0, f1, gl0, gl1);
  mul2o(m0, m1, f0, f1, hj00, hj01);
  fma2o(g00, g01, g00, g01, s0, s1, m0, m1);
  mul2o(m0, m1, f0, f1, hj10, hj11);
  fma2o(g10, g11, g10, g11, s0, s1, m0, m1);
  mul2o(gl0, gl1, gl0, gl1, s0, s1);
}

// Component c of h_{l-1} for this thread's 16 neuron slots: from the scratch (l >= 2) or,
// for h_0, recomputed from the point.
__device__ __forceinline__ void h_component(float (&hv)[16], int l, int c, const float* hsrc,
                                            const float* small, const float* xs, int tid,
                                            int s) {
  if (l > 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) hv[i] = hsrc[(c * 16 + i) * kThreads];
  } else {
    const float x0 = xs[tid], x1 = xs[kThreads + tid];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {  // neuron pairs, packed pair arithmetic
      const int o = 16 * (i >> 2) + 4 * s + (i & 3);
      const float w0a = small[kSmW0 + 2 * o], w1a = small[kSmW0 + 2 * o + 1];
      const float w0b = small[kSmW0 + 2 * o + 2], w1b = small[kSmW0 + 2 * o + 3];
      float za, zb, va, vb, j0a, j0b, j1a, j1b, la, lb;
      fma2o(za, zb, w1a, w1b, x1, x1, small[kSmB0 + o], small[kSmB0 + o + 1]);
      fma2o(za, zb, w0a, w0b, x0, x0, za, zb);
      tanh_jet_fast2(za, zb, w0a, w0b, w1a, w1b, 0.0f, 0.0f, va, vb, j0a, j0b, j1a, j1b, la,
                     lb);
      hv[i] = c == 0 ? va : c == 1 ? j0a : c == 2 ? j1a : la;
      hv[i + 1] = c == 0 ? vb : c == 1 ? j0b : c == 2 ? j1b : lb;
    }
  }
}

// The 4 weight-gradient MMAs of one jet component for one point half (M = 128, N = 128,
// K = 16 points each, f16, both operands MN-major) into that half's accumulator. Issued by
// one converged warp of the half, then committed to the half's barrier.
__device__ __forceinline__ void issue_dw_mmas(const Ctx& cx, int half, bool first) {
  constexpr uint32_t kIdescDw =
      tc::idesc_f16(128, 128) | tc::kIdescAMnMajor | tc::kIdescBMnMajor;
  const uint32_t base = smem_u32(dsmem() + kStageOff + half * kStageBytes);
  const uint32_t d = cx.tmem + kDwCol + 128u * static_cast<uint32_t>(half);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {  // points 16 ks .. 16 ks + 15: two 8-point K groups
    const uint32_t k0 = static_cast<uint32_t>(ks) * 2u * kDwLbo;
    const uint64_t a = tc::smem_desc_kmajor(base + kStageA + k0, kDwLbo, kDwSbo);
    const uint64_t bb = tc::smem_desc_kmajor(base + kStageB + k0, kDwLbo, kDwSbo);
    tc::mma_f16_ss_warp(d, a, bb, kIdescDw, (first && ks == 0) ? 0u : 1u);
  }
  tc::commit_warp(bar_dwdone(half));
}

// 16-byte shared-memory store.
__device__ __forceinline__ void st_shared_v4(uint8_t* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

// Stages one operand's 16 values of this thread (neuron slots i = 0..15, times `scale`) as f16
// hi/lo pairs: slots 8g..8g+7 are one 16-byte group, hi at row group 2s + g, lo 8 groups on.
__device__ __forceinline__ void stage_f16_rows(uint8_t* at, int s, const float (&v)[16],
                                               float scale) {
  uint32_t hi[8], lo[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    float a = v[2 * p], b = v[2 * p + 1];
    mul2(a, b, scale, scale);
    split_f16_pair_fast(a, b, hi[p], lo[p]);
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    st_shared_v4(at + (2 * s + g) * kDwSbo, hi[4 * g], hi[4 * g + 1], hi[4 * g + 2], hi[4 * g + 3]);
    st_shared_v4(at + (8 + 2 * s + g) * kDwSbo, lo[4 * g], lo[4 * g + 1], lo[4 * g + 2],
                 lo[4 * g + 3]);
  }
}

// Barrier over the 8 warps (256 threads) of one point half; ids 1 and 2 (0 is __syncthreads,
// 3 the epilogue barrier).
__device__ __forceinline__ void half_barrier(int half) {
  asm volatile("bar.sync %0, 256;" ::"r"(1 + half) : "memory");
}

// The MMA warp: issues, in the epilogue warps' order, the MMAs of every chunk of this CTA's
// tiles (GEMMs 0..5 of each tile). Returns early when a wait gives up.
__device__ __forceinline__ void mma_warp(const Ctx& cx, int64_t tiles) {
  uint32_t n = 0, tile_count = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tile_count) {
#pragma unroll 1
    for (int g = 0; g < kGemmsPerTile; ++g) {
#pragma unroll 1
      for (int j = 0; j < kChunks; ++j, ++n) {
        const uint32_t slot = n % kRing;
        if (!warp_wait(bar_full(slot), (n / kRing) & 1u)) return;
        tc::fence_after_sync();
        if (!issue_chunk_mmas(cx, tile_count, g, j, slot)) return;
        __syncwarp();
      }
    }
  }
}

// Sums v[i] over the 32 lanes of the warp for every i < 16 with a fixed butterfly that
// halves the values held per lane at each step (16 shuffles instead of 80); lane l returns
// the total for i = l >> 1.
__device__ __forceinline__ float warp_sum16(const float (&v)[16]) {
  const int lane = threadIdx.x & 31;
  float u8[8], u4[4], u2[2];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool hi = (lane & 16) != 0;
    const float keep = hi ? v[8 + j] : v[j], send = hi ? v[j] : v[8 + j];
    u8[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool hi = (lane & 8) != 0;
    const float keep = hi ? u8[4 + j] : u8[j], send = hi ? u8[j] : u8[4 + j];
    u4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool hi = (lane & 4) != 0;
    const float keep = hi ? u4[2 + j] : u4[j], send = hi ? u4[j] : u4[2 + j];
    u2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  const bool hi = (lane & 2) != 0;
  float r = (hi ? u2[1] : u2[0]) + __shfl_xor_sync(0xffffffffu, hi ? u2[0] : u2[1], 2);
  return r + __shfl_xor_sync(0xffffffffu, r, 1);
}

// Sums v[k] over the 32 lanes for every k < 8 with the same halving butterfly as
// warp_sum16; lane l returns the total for k = (l >> 2) & 7.
__device__ __forceinline__ float warp_sum8(const float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  float u4[4], u2[2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool hi = (lane & 16) != 0;
    const float keep = hi ? v[4 + j] : v[j], send = hi ? v[j] : v[4 + j];
    u4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool hi = (lane & 8) != 0;
    const float keep = hi ? u4[2 + j] : u4[j], send = hi ? u4[j] : u4[2 + j];
    u2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const bool hi = (lane & 4) != 0;
  float r = (hi ? u2[1] : u2[0]) + __shfl_xor_sync(0xffffffffu, hi ? u2[0] : u2[1], 4);
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  return r + __shfl_xor_sync(0xffffffffu, r, 1);
}

// Writes half `h` (neuron slots 8h..8h+7) of a warp_sum8 result to the per-quadrant partials.
__device__ __forceinline__ void store_part8(float* part, int kind, int q, int s, int h, float r) {
  const int lane = threadIdx.x & 31;
  if ((lane & 3) == 0) {
    const int i = 8 * h + (lane >> 2);
    part[kind * 256 + q * 64 + 16 * (i >> 2) + 4 * s + (i & 3)] = r;
  }
}

// Writes this warp's per-neuron sums (warp_sum16 output) to the per-quadrant partials.
__device__ __forceinline__ void store_part16(float* part, int kind, int q, int s, float r) {
  const int lane = threadIdx.x & 31;
  if ((lane & 1) == 0) {
    const int i = lane >> 1;
    part[kind * 256 + q * 64 + 16 * (i >> 2) + 4 * s + (i & 3)] = r;
  }
}

// Cluster helpers: this CTA's rank, a barrier over every thread of the cluster (release /
// acquire: shared-memory writes before it are visible to the cluster's reads after it), the
// shared::cluster address of a shared::cta address in CTA `rank`, and a load through it.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Pre-split weights for the tensor-core backward: six K-major canonical f16 operands, hi then
// lo, of W1, W2, W3 ([out][in], forward GEMMs) and W1^T, W2^T, W3^T ([in][out], input-adjoint
// GEMMs), each times tau_l (the power of 2 that maps max |W_l| to <= 16; the step kernel
// derives the same tau from the same maximum). One block per operand; pair (row, kk..kk+1)
// of an operand is word (row / 8) 256 + (kk / 8) 32 + (row % 8) 4 + (kk % 8) / 2, the layout
// of the forward kernel's f16 weight operands, and row r holds neuron neuron_of_column(r).
__global__ void __launch_bounds__(512) prep_weights_kernel(const float* __restrict__ params,
                                                           float* __restrict__ wsplit) {
  __shared__ float wmax[16];
  // The step kernel after this one starts its set-up now (it waits for these operands
  // before its first weight-slot copy).
  allow_dependents();
  const int blk = blockIdx.x, tid = threadIdx.x;
  const float* W = params + kHiddenBase + (blk % 3) * kHiddenStride;
  // The block's 2048 pairs cover every element of W_l once: their maximum is tau's input,
  // so all loads are issued at once (one memory round trip).
  float a[4], b[4];
  int word[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int w = tid + 512 * k;
    const int n = neuron_of_column(((w >> 8) << 3) | ((w >> 2) & 7));
    const int kk = (((w >> 5) & 7) << 3) | ((w & 3) << 1);
    a[k] = blk >= 3 ? W[kk * kWidth + n] : W[n * kWidth + kk];
    b[k] = blk >= 3 ? W[(kk + 1) * kWidth + n] : W[n * kWidth + kk + 1];
    word[k] = w;
  }
  float m = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) m = fmaxf(m, fmaxf(fabsf(a[k]), fabsf(b[k])));
  m = warp_max_nonneg(m);
  if ((tid & 31) == 0) wmax[tid >> 5] = m;
  __syncthreads();
  float mx = 0.0f;
#pragma unroll
  for (int w = 0; w < 16; ++w) mx = fmaxf(mx, wmax[w]);
  const float tau = pow2_floor_ratio(4, mx);
  uint32_t* out = reinterpret_cast<uint32_t*>(wsplit) + blk * (kLayerBytes / 4);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t hi, lo;
    split_f16_pair_fast(a[k] * tau, b[k] * tau, hi, lo);
    out[word[k]] = hi;
    out[kOperandBytes / 4 + word[k]] = lo;
  }
}

template <bool kPoisson>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kBlockThreads, 1)
    backward_tc_kernel(const PointSets ps, const float* __restrict__ params,
                       const float* __restrict__ wsplit, const float* __restrict__ grad_u,
                       const float* __restrict__ grad_lap, float* __restrict__ grad_coords,
                       float* __restrict__ lap_out, float* __restrict__ partials,
                       float* __restrict__ scratch, int64_t tiles, unsigned int* status) {
  uint8_t* const smem = dsmem();
  float* small = reinterpret_cast<float*>(smem + kSmallOff);
  float* grad = reinterpret_cast<float*>(smem + kGradOff);
  float* red = reinterpret_cast<float*>(smem + kRedOff);
  float* part = reinterpret_cast<float*>(smem + kPartOff);
  float* xs = reinterpret_cast<float*>(smem + kXsOff);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  Ctx cx;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // The training step's update kernel may be scheduled onto SMs as this grid's CTAs exit
  // (it waits for the whole grid before it reads the partial rows).
  allow_dependents();

  // ---- set-up ----
  // The first tile's point, requested first: its latency overlaps the set-up below.
  float x0 = 0.0f, x1 = 0.0f;
  if (warp < kWarps) load_point(ps, blockIdx.x, kTile, 32 * (warp & 3) + lane, x0, x1);
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
  // The hidden-layer weight gradients are accumulated in shared memory, each entry by the
  // one thread that owns it, so the order is fixed.
  float* const hgrad = reinterpret_cast<float*>(smem + kRowsOff);
  for (int i = tid; i < kHiddenGrads; i += kBlockThreads) hgrad[i] = 0.0f;
  if (tid == 0) {
    for (uint32_t r = 0; r < kRing; ++r) mbar_init(bar_full(r), kWarps);

    mbar_init(bar_dfull(), 1);
    mbar_init(bar_red(), kWarps);
    for (int k = 0; k < kWeightSlots; ++k) mbar_init(bar_wfull(k), 1);
    mbar_init(bar_dwdone(0), 1);
    mbar_init(bar_dwdone(1), 1);
    *abort_flag() = 0u;
    *status_slot() = status;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  if (warp < kWarps) {
    // Rows warp + 16 i of W1, W2, W3: the absolute row sums of W1 and W2 (fixed-order warp
    // sums), the norms that bound the activations h_1, h_2 and so their f16 scales, and this
    // warp's maximum |w| of each layer (its weight scale tau).
    float rs[12][2];
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const int r = warp + kWarps * i;
      const float* wr = params + kHiddenBase + (r >> 6) * kHiddenStride + (r & 63) * kWidth;
      rs[i][0] = wr[lane];
      rs[i][1] = wr[lane + 32];
    }
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = fabsf(rs[i][0]) + fabsf(rs[i][1]);
    const float sum = warp_sum8(v);  // lane l: the sum of row warp + 16 ((l >> 2) & 7)
    if ((lane & 3) == 0) red[warp + kWarps * ((lane >> 2) & 7)] = sum;
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      float m = 0.0f;
#pragma unroll
      for (int i = 4 * l; i < 4 * l + 4; ++i) m = fmaxf(m, fmaxf(fabsf(rs[i][0]), fabsf(rs[i][1])));
      m = warp_max_nonneg(m);
      if (lane == 0) red[128 + kWarps * l + warp] = m;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  cx.tmem = *tmem_base_slot;
  if (tid == 0) {
    // This kernel may start while prep_weights_kernel still runs; everything above reads
    // only what was complete before that kernel started. Thread 0 makes every read of the
    // pre-split weights (these copies and the later slot reloads), so it alone waits.
    wait_for_prerequisites();
    for (int k = 0; k < kWeightSlots; ++k) load_weight_slot(k, wsplit, weight_block(k));
  }

  if (warp >= kWarps) {
    // ---- MMA warpgroup: warp 16 issues the chunks, 17-19 wait at the final barrier ----
    regs_dec<kMmaRegs>();
    if (warp == kMmaWarp) mma_warp(cx, tiles);
  } else {
    // ---- epilogue warpgroups ----
    regs_inc<kEpiRegs>();
    const int q = warp & 3;   // TMEM lane quadrant
    const int s = warp >> 2;  // neurons 16a + 4s + t
    const uint32_t tmem_warp = cx.tmem + (static_cast<uint32_t>(32 * q) << 16);
    const int row = 32 * q + lane;
    float* const hscratch = scratch + static_cast<int64_t>(blockIdx.x) * kScratchFloats + tid;
    // Weight-gradient staging: this thread's point is K index kpt = 32 (q & 1) + lane of the
    // staging buffer of its point half q >> 1.
    const int half = q >> 1;
    const int kpt = 32 * (q & 1) + lane;
    uint8_t* const stage_at =
        smem + kStageOff + half * kStageBytes + (kpt % 8) * 16 + (kpt / 8) * kDwLbo;
    float* const zmax = reinterpret_cast<float*>(smem + kZmaxOff);
    float* const sigw = reinterpret_cast<float*>(smem + kDwScaleOff) + warp * kSigFloats;
    {
      // The f16 scales of the weight gradient's h operands, this warp's own copy: the bounds
      // of the 3xFP16 forward (|v| <= 1; |d/dx|, |d/dy| <= B_J grow by the norm N_l of W_l,
      // |L| <= B_L becomes N_l B_L + 2 (N_l B_J)^2), each mapped to <= 2^14 by a power of 2.
      const float n1 = warp_max_nonneg(fmaxf(red[lane], red[lane + 32]));
      const float n2 = warp_max_nonneg(fmaxf(red[64 + lane], red[96 + lane]));
      const float w0x = small[kSmW0 + 2 * lane], w0y = small[kSmW0 + 2 * lane + 1];
      const float w1x = small[kSmW0 + 2 * (lane + 32)], w1y = small[kSmW0 + 2 * (lane + 32) + 1];
      float bj = warp_max_nonneg(
          fmaxf(fmaxf(fabsf(w0x), fabsf(w1x)), fmaxf(fabsf(w0y), fabsf(w1y))));
      float bl = warp_max_nonneg(fmaxf(fmaf(w0x, w0x, w0y * w0y), fmaf(w1x, w1x, w1y * w1y)));
      // lane 4l + c writes sigma of component c of h_l and its inverse (exact: a power of 2)
      const float nrm[2] = {n1, n2};
      float sl[3][2];  // h_l: sigma of d/dx and d/dy, of L
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        sl[l][0] = pow2_floor_ratio(14, bj);
        sl[l][1] = pow2_floor_ratio(14, bl);
        if (l < 2) {
          const float nj = nrm[l] * bj;
          bl = fmaf(nrm[l], bl, 2.0f * nj * nj);
          bj = nj;
        }
      }
      if (lane < 12) {
        const int l = lane >> 2, c = lane & 3;
        const float j = l == 0 ? sl[0][0] : l == 1 ? sl[1][0] : sl[2][0];
        const float lv = l == 0 ? sl[0][1] : l == 1 ? sl[1][1] : sl[2][1];
        const float sg = c == 0 ? 16384.0f : c == 3 ? lv : j;
        sigw[kSig + lane] = sg;
        sigw[kInvSig + lane] = inv_pow2(sg);
      }
      // tau_l maps max |W_l| to <= 16 (the same scale the pre-split weights carry)
      float tl[3];
#pragma unroll
      for (int l = 0; l < 3; ++l)
        tl[l] = pow2_floor_ratio(4, warp_max_nonneg(red[128 + kWarps * l + (lane & 15)]));
      if (lane < 3) {
        const float t = lane == 0 ? tl[0] : lane == 1 ? tl[1] : tl[2];
        sigw[kTau + lane] = t;
        sigw[kInvTau + lane] = inv_pow2(t);
      }
      __syncwarp();
    }

    uint32_t chunk = 0, mlayer = 0, tile_count = 0, dw_issued = 0;
    bool alive = true;
    // The tile's point lives in shared memory (xs), so no register holds it through the
    // backward sweep. Layer 0 of a tile is produced at the end of the previous tile (right
    // after the last input-adjoint GEMM's accumulators are read, before that tile's layer-0
    // adjoint), so GEMM 0 of the next tile runs under it; the first tile's layer 0 runs here.
    {
      xs[tid] = x0;
      xs[kThreads + tid] = x1;
      if (static_cast<int64_t>(blockIdx.x) < tiles)
        produce_layer0(x0, x1, small, sigw + kSig, chunk, tmem_warp, s);
    }
    float* const xn = reinterpret_cast<float*>(smem + kXnOff);  // the next tile's points
    for (int64_t tile = blockIdx.x; alive && tile < tiles; tile += gridDim.x, ++tile_count) {
      const bool has_next = tile + gridDim.x < tiles;
      const bool btile = tile >= ps.tiles;  // a tile of the boundary set (PINN step)
      const int64_t p = (btile ? tile - ps.tiles : tile) * kTile + row;
      const bool active = p < (btile ? ps.nb : ps.n);
      if (has_next) prefetch_point(ps, tile + gridDim.x, row, xn + tid);

      // ---- forward recompute: the three hidden GEMMs (layer 0 is already in the ring) ----
      float d[4][16];  // d[c][4a + t]: component c of neuron 16a + 4s + t
#pragma unroll 1
      for (int g = 0; g < 3; ++g) {
        warp_wait(bar_dfull(), mlayer & 1u);
        ++mlayer;
        tc::fence_after_sync();
        // GEMM g is complete: its weight slot takes the operand of GEMM g + 2.
        if (tid == 0) load_weight_slot(g & 1, wsplit, weight_block(g + 2));
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::ld_x16(tmem_warp + 64u * c + 16u * s, d[c]);
        tc::wait_ld();
        {
          // D carries sigma_c of h_g times tau_g of W_{g+1}: both powers of 2, undone exactly
          const float* bias = small + kSmB + 64 * g;
          const float it = sigw[kInvTau + g];
          const float uv = sigw[kInvSig + 4 * g] * it, uj = sigw[kInvSig + 4 * g + 1] * it;
          const float ul = sigw[kInvSig + 4 * g + 3] * it;
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int o = 16 * (i >> 2) + 4 * s + (i & 3);  // neuron slots i, i + 1: o, o + 1
            fma2o(d[0][i], d[0][i + 1], d[0][i], d[0][i + 1], uv, uv, bias[o], bias[o + 1]);
          }
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            mul2(d[1][i], d[1][i + 1], uj, uj);
            mul2(d[2][i], d[2][i + 1], uj, uj);
            mul2(d[3][i], d[3][i + 1], ul, ul);
          }
        }
        if (g < 2) {
          float* hj = hscratch + g * (4 * 16 * kThreads);  // h_{g+1}
          const float* sg = sigw + kSig + 4 * (g + 1);     // its f16 scales
#pragma unroll
          for (int a = 0; a < kChunks; ++a) {
            float h[4][4];
#pragma unroll
            for (int t = 0; t < 4; t += 2) {
              const int i = 4 * a + t;
              tanh_jet_fast2(d[0][i], d[0][i + 1], d[1][i], d[1][i + 1], d[2][i], d[2][i + 1],
                             d[3][i], d[3][i + 1], h[0][t], h[0][t + 1], h[1][t], h[1][t + 1],
                             h[2][t], h[2][t + 1], h[3][t], h[3][t + 1]);
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                hj[(c * 16 + i) * kThreads] = h[c][t];
                hj[(c * 16 + i + 1) * kThreads] = h[c][t + 1];
              }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float g2 = sg[c];
              mul2(h[c][0], h[c][1], g2, g2);
              mul2(h[c][2], h[c][3], g2, g2);
            }
            produce_chunk(chunk++, h, tmem_warp, s);
          }
        }
      }

      // ---- output layer, loss seed, layer-3 adjoint (d becomes h3, then zbar3) ----
      {
        float pu = 0.0f, pl = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          tanh_jet_fast2(d[0][i], d[0][i + 1], d[1][i], d[1][i + 1], d[2][i], d[2][i + 1],
                         d[3][i], d[3][i + 1], d[0][i], d[0][i + 1], d[1][i], d[1][i + 1],
                         d[2][i], d[2][i + 1], d[3][i], d[3][i + 1]);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float w = small[kSmWout + 16 * ((i + k) >> 2) + 4 * s + ((i + k) & 3)];
            pu = fmaf(w, d[0][i + k], pu);
            pl = fmaf(w, d[3][i + k], pl);
          }
        }
        red[s * kTile + row] = pu;
        red[(4 + s) * kTile + row] = pl;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_red());
        warp_wait(bar_red(), tile_count & 1u);
        float lap = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) lap += red[(4 + k) * kTile + row];
        float gu, gl;
        if (kPoisson) {
          float term;  // this point's loss term
          if (!btile) {
            // f = -2 pi^2 sin(pi x) sin(pi y)  (src/fused_hoad/problems/poisson.py:29-39); sinpif
            // needs no large-argument reduction (no local-memory path)
            const float pi = 3.14159265358979323846f;
            const float f =
                -2.0f * pi * pi * (sinpif(xs[tid]) * sinpif(xs[kThreads + tid]));
            const float r = active ? lap - f : 0.0f;
            gu = 0.0f;
            gl = 2.0f * r * ps.inv_total;
            term = r * r * ps.inv_total;
            if (s == 0 && active && lap_out != nullptr) lap_out[p] = lap;
          } else {
            // boundary term weight * u^2 / boundary_total (src/fused_hoad/training.py:90-92)
            float u = small[kSmBout];
#pragma unroll
            for (int k = 0; k < 4; ++k) u += red[k * kTile + row];
            u = active ? u : 0.0f;
            gu = 2.0f * ps.bweight * u * ps.inv_btotal;
            gl = 0.0f;
            term = ps.bweight * u * u * ps.inv_btotal;
          }
          if (s == 0) {
            const float l2 = warp_sum(term);
            const float sg = btile ? warp_sum(gu) : 0.0f;  // b_out gradient (boundary term)
            if (lane == 0) {
              part[kPLoss + q] = l2;
              part[kPBout + q] = sg;
            }
          }
        } else {
          gu = (active && grad_u != nullptr) ? grad_u[p] : 0.0f;
          gl = active ? grad_lap[p] : 0.0f;
          if (s == 0) {
            const float sg = warp_sum(gu);
            if (lane == 0) part[kPBout + q] = sg;
          }
        }
        // w_out gradient terms, reduced eight neurons at a time (fewer live registers)
#pragma unroll
        for (int half8 = 0; half8 < 2; ++half8) {
          float dwo[8];
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            const int i = 8 * half8 + k;
            mul2o(dwo[k], dwo[k + 1], gl, gl, d[3][i], d[3][i + 1]);
            fma2o(dwo[k], dwo[k + 1], gu, gu, d[0][i], d[0][i + 1], dwo[k], dwo[k + 1]);
          }
          store_part8(part, 0, q, s, half8, warp_sum8(dwo));
        }
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const int o = 16 * (i >> 2) + 4 * s + (i & 3);  // o + 1 is neuron slot i + 1
          const float wa = small[kSmWout + o], wb = small[kSmWout + o + 1];
          float gva, gvb, g0a = 0.0f, g0b = 0.0f, g1a = 0.0f, g1b = 0.0f, gLa, gLb;
          mul2o(gva, gvb, gu, gu, wa, wb);
          mul2o(gLa, gLb, gl, gl, wa, wb);
          adjoint_h2(d[0][i], d[0][i + 1], d[1][i], d[1][i + 1], d[2][i], d[2][i + 1], d[3][i],
                     d[3][i + 1], gva, gvb, g0a, g0b, g1a, g1b, gLa, gLb);
          d[0][i] = gva;
          d[0][i + 1] = gvb;
          d[1][i] = g0a;
          d[1][i + 1] = g0b;
          d[2][i] = g1a;
          d[2][i + 1] = g1b;
          d[3][i] = gLa;
          d[3][i + 1] = gLb;
        }
        store_part16(part, 6, q, s, warp_sum16(d[0]));  // b3
      }

      // ---- backward through the hidden layers: d holds zbar_l on entry ----
#pragma unroll 1
      for (int l = 3; l >= 1; --l) {
        const int g = 6 - l;
        // f16 scales of zbar_l, per tile and point half (a point's row of either GEMM stays in
        // its half): S_c maps the half's max |zbar_c| to <= 2^14 for the input adjoint (one
        // GEMM per component), and zs maps max_c |zbar_c| / sigma_c to <= 2^14 for the weight
        // gradient, whose operands z~_c = zbar_c zs / sigma_c pair with h~_c = h_c sigma_c, so
        // that every component's product carries the same factor zs. This warp's maxima first.
        const float* sg = sigw + kSig + 4 * (l - 1);      // sigma of h_{l-1}: v, d/dx, d/dy, L
        const float* isg = sigw + kInvSig + 4 * (l - 1);  // 1 / sigma
        const float* hsrc = hscratch + (l == 3 ? 4 * 16 * kThreads : 0);  // h_{l-1} (l >= 2)
        {
          float* zw = zmax + kZmaxFloats * warp;
          float zm = 0.0f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float mc = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; i += 2) mc = fmax3(mc, fabsf(d[c][i]), fabsf(d[c][i + 1]));
            mc = warp_max_nonneg(mc);
            zm = fmaxf(zm, mc * isg[c]);
            if (lane == 0) zw[c] = mc;
          }
          if (lane == 0) zw[4] = zm;
        }
        half_barrier(half);
        {
          // lane k < 8 reads warp k of the half; the maxima over the lanes by redux
          float hm[5];
          {
            const float* zw =
                zmax + kZmaxFloats * (2 * half + (lane & 1) + 4 * ((lane >> 1) & 3));
#pragma unroll
            for (int k = 0; k < 5; ++k) hm[k] = warp_max_nonneg(lane < 8 ? zw[k] : 0.0f);
          }
          const float zs = pow2_floor_ratio(14, hm[4]);
          const float itau = sigw[kInvTau + (l - 1)];
          // d becomes zbar_l times S_c (exact: powers of 2) -> ring (input-adjoint GEMM g)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float sc = pow2_floor_ratio(14, hm[c]), isc = inv_pow2(sc);
            if (lane == 0) {
              sigw[kStg + c] = zs * isg[c] * isc;
              sigw[kIsc + c] = isc * itau;
            }
#pragma unroll
            for (int i = 0; i < 16; i += 2) mul2(d[c][i], d[c][i + 1], sc, sc);
          }
          __syncwarp();
#pragma unroll
          for (int a = 0; a < kChunks; ++a) {
            float z[4][4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
              for (int c = 0; c < 4; ++c) z[c][t] = d[c][4 * a + t];
            produce_chunk(chunk++, z, tmem_warp, s);
          }
        }
        // weight gradient dW_l: per jet component, stage zbar_l and h_{l-1} (f16 hi/lo, scaled)
        // for the tile's 128 points and let one warp issue the MMAs. Unrolled, so that the
        // registers of component c of zbar_l are free once its round is staged; component
        // c + 1 of h_{l-1} is read right after component c is staged, so its latency overlaps
        // the round's barrier, issue and commit wait.
        float hv[16];
        h_component(hv, l, 0, hsrc, small, xs, tid, s);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c > 0) warp_wait(bar_dwdone(half), (dw_issued - 1u) & 1u);  // buffer free again
          stage_f16_rows(stage_at + kStageA, s, d[c], sigw[kStg + c]);
          stage_f16_rows(stage_at + kStageB, s, hv, sg[c]);
          if (c < 3) h_component(hv, l, c + 1, hsrc, small, xs, tid, s);
          tc::fence_proxy_async_smem();
          half_barrier(half);
          if (s == 0 && (q & 1) == 0) {  // warp 2 * half issues for its half
            if (c == 0) {
              // the input-adjoint GEMM g has finished with the ring columns the weight-gradient
              // accumulators borrow, and with its weight slot
              warp_wait(bar_dfull(), mlayer & 1u);
              tc::fence_after_sync();
              if (half == 0 && lane == 0 && (g + 2 < kGemmsPerTile || has_next))
                load_weight_slot(g & 1, wsplit, weight_block((g + 2) % kGemmsPerTile));
            }
            tc::fence_after_sync();
            issue_dw_mmas(cx, half, c == 0);
          }
          ++dw_issued;
        }

        // Empty the accumulators into the gradient block. A thread holds row r of the
        // accumulator, columns 16s..16s+15, each the sum over the h_hi and h_lo columns of both
        // halves' accumulators, each half divided by its scale (exact powers of 2). Row r < 64
        // is z_hi times h; row r + 64 is z_lo times h of the same neuron. The rows < 64 go
        // through shared memory (half 1's staging buffer) to the thread of row r + 64, which adds
        // hi + lo into the entry it owns: column-major in accumulator order,
        // hgrad[4096 (l - 1) + 64 c + r] for column c and row r.
        // Both halves first pass this barrier: each half has then waited for its round-2
        // commit, so the parity wait below can only mean round 3 (without it, a half that is
        // two rounds behind would satisfy the wait with its round-1 phase).
        if (!(alive = barrier_ok())) break;
        warp_wait(bar_dwdone(0), (dw_issued - 1u) & 1u);
        warp_wait(bar_dwdone(1), (dw_issued - 1u) & 1u);
        tc::fence_after_sync();
        {
          float* fb = reinterpret_cast<float*>(smem + kStageOff + kStageBytes);  // [64][65]
          float inv[2];  // lane k < 16 reads warp k's maximum
          {
            const float m = lane < 16 ? zmax[kZmaxFloats * lane + 4] : 0.0f;
            const bool h1 = (lane & 2) != 0;  // warp k is in half (k & 3) >> 1
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              inv[hh] = inv_pow2(pow2_floor_ratio(14, warp_max_nonneg(h1 == (hh == 1) ? m : 0.0f)));
          }

          float v[16], w[16];
          tc::ld_x16(tmem_warp + kDwCol + 16u * s, v);
          tc::ld_x16(tmem_warp + kDwCol + 64u + 16u * s, w);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = (v[k] + w[k]) * inv[0];
          tc::ld_x16(tmem_warp + kDwCol + 128u + 16u * s, w);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = fmaf(w[k], inv[1], v[k]);
          tc::ld_x16(tmem_warp + kDwCol + 192u + 16u * s, w);
          tc::wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] = fmaf(w[k], inv[1], v[k]);
          if (row < 64) {
#pragma unroll
            for (int k = 0; k < 16; ++k) fb[row * kFlushStride + 16 * s + k] = v[k];
          }
          // Every warp's accumulator loads are complete past this barrier (the ring's columns
          // take chunks again afterwards); half 1 reads its staging buffer before its next
          // half barrier, after which it stages there again.
          tc::fence_before_sync();
          if (!(alive = barrier_ok())) break;
          if (row >= 64) {
            float* wcol = hgrad + (l - 1) * (kWidth * kWidth) + (row - 64);
            const float* src = fb + (row - 64) * kFlushStride + 16 * s;
#pragma unroll
            for (int k = 0; k < 16; ++k) wcol[(16 * s + k) * kWidth] += src[k] + v[k];
          }
        }

        // input adjoint hbar_{l-1} = zbar_l W_l (GEMM g; D carries S_c tau), then zbar_{l-1}
        warp_wait(bar_dfull(), mlayer & 1u);
        ++mlayer;
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::ld_x16(tmem_warp + 64u * c + 16u * s, d[c]);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float isc = sigw[kIsc + c];
#pragma unroll
          for (int i = 0; i < 16; i += 2) mul2(d[c][i], d[c][i + 1], isc, isc);
        }
        if (l == 1 && has_next) {  // GEMM 0 of the next tile may now overwrite D
          prefetch_wait();
          produce_layer0(xn[tid], xn[kThreads + tid], small, sigw + kSig, chunk, tmem_warp, s);
        }
        if (l > 1) {
#pragma unroll
          for (int a = 0; a < kChunks; ++a) {
            float h[4][4];
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
for (int c = 0; c < 4; ++c) h[c][t] = hsrc[(c * 16 + 4 * a + t) * kThreads];
#pragma unroll
            for (int t = 0; t < 4; t += 2) {
              const int i = 4 * a + t;
              adjoint_h2(h[0][t], h[0][t + 1], h[1][t], h[1][t + 1], h[2][t], h[2][t + 1],
                         h[3][t], h[3][t + 1], d[0][i], d[0][i + 1], d[1][i], d[1][i + 1],
                         d[2][i], d[2][i + 1], d[3][i], d[3][i + 1]);
            }
          }
          store_part16(part, 2 + l, q, s, warp_sum16(d[0]));  // b_{l-1}
        }
      }
      if (!alive) break;


      // ---- layer 0: z_v = W0 x + b0, z_J = W0, z_L = 0; d holds hbar_0 ----
      {
        const float x0 = xs[tid], x1 = xs[kThreads + tid];
        float gx0 = 0.0f, gx1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const int o = 16 * (i >> 2) + 4 * s + (i & 3);  // o + 1 is neuron slot i + 1
          const float w0a = small[kSmW0 + 2 * o], w1a = small[kSmW0 + 2 * o + 1];
          const float w0b = small[kSmW0 + 2 * o + 2], w1b = small[kSmW0 + 2 * o + 3];
          float za, zb, aa, ab, j0a, j0b, j1a, j1b, la, lb;
          fma2o(za, zb, w1a, w1b, x1, x1, small[kSmB0 + o], small[kSmB0 + o + 1]);
          fma2o(za, zb, w0a, w0b, x0, x0, za, zb);
          tanh_jet_fast2(za, zb, w0a, w0b, w1a, w1b, 0.0f, 0.0f, aa, ab, j0a, j0b, j1a, j1b, la,
                         lb);
          adjoint_h2(aa, ab, j0a, j0b, j1a, j1b, la, lb, d[0][i], d[0][i + 1], d[1][i],
                     d[1][i + 1], d[2][i], d[2][i + 1], d[3][i], d[3][i + 1]);
          fma2o(d[1][i], d[1][i + 1], d[0][i], d[0][i + 1], x0, x0, d[1][i], d[1][i + 1]);
          fma2o(d[2][i], d[2][i + 1], d[0][i], d[0][i + 1], x1, x1, d[2][i], d[2][i + 1]);
          // d[0] holds the db0 terms, d[1] and d[2] the dW0[:, 0] and dW0[:, 1] terms
          gx0 = fmaf(w0a, d[0][i], gx0);
          gx1 = fmaf(w1a, d[0][i], gx1);
          gx0 = fmaf(w0b, d[0][i + 1], gx0);
          gx1 = fmaf(w1b, d[0][i + 1], gx1);
        }
        store_part16(part, 1, q, s, warp_sum16(d[0]));
        store_part16(part, 2, q, s, warp_sum16(d[1]));
        store_part16(part, 3, q, s, warp_sum16(d[2]));
        red[s * kTile + row] = gx0;
        red[(4 + s) * kTile + row] = gx1;
      }
      if (!(alive = barrier_ok())) break;
      if (s == 0 && active && !btile && grad_coords != nullptr) {
        float sx = 0.0f, sy = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          sx += red[k * kTile + row];
          sy += red[(4 + k) * kTile + row];
        }
        grad_coords[2 * p] = sx;
        grad_coords[2 * p + 1] = sy;
      }
      // per-quadrant partials -> accumulators, quadrants in index order
      if (tid < kPartKinds * kWidth) {
        const int kind = tid >> 6, o = tid & 63;
        const float* src = part + kind * 256 + o;
        const float v = ((src[0] + src[64]) + src[128]) + src[192];
        if (kind == 0) grad[kGWout + o] += v;
        else if (kind == 1) grad[kGBias + o] += v;
        else if (kind <= 3) grad[kGW0 + 2 * o + (kind - 2)] += v;
        else grad[kGBias + (kind - 3) * kWidth + o] += v;
      } else if (tid == kPartKinds * kWidth) {
        if (kPoisson)
          grad[kGLoss] += ((part[kPLoss] + part[kPLoss + 1]) + part[kPLoss + 2]) + part[kPLoss + 3];
        grad[kGBout] += ((part[kPBout] + part[kPBout + 1]) + part[kPBout + 2]) + part[kPBout + 3];
      }
      // No barrier before the next tile: its first writes of `part`, `red` and `grad` come
      // after its GEMM 2, whose chunks every warp produces only after finishing the reads
      // above; xs is this thread's own.
      if (has_next) {  // this thread's own entries: no other thread reads them
        xs[tid] = xn[tid];
        xs[kThreads + tid] = xn[kThreads + tid];
      }
    }

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
  // ---- the cluster's partial-gradient row ----
  // Every CTA of the cluster takes both cluster barriers, aborted or not (a peer's abort
  // shows in the status word). CTA rank k writes its share of the columns, each the sum over
  // the cluster's CTAs in rank order, read through distributed shared memory.
  cluster_sync();  // the cluster's gradients are complete and visible
  if (!aborted) {
    const uint32_t rank = cluster_ctarank();
    float* const crow = partials + static_cast<int64_t>(blockIdx.x / kCluster) * kRowStride;
    uint32_t hg[kCluster], gr[kCluster];
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      hg[r] = mapa_shared(smem_u32(hgrad), static_cast<uint32_t>(r));
      gr[r] = mapa_shared(smem_u32(grad), static_cast<uint32_t>(r));
    }
    // gradient-block entry e = 4096 l + 64 c + r: accumulator column c (input neuron
    // neuron_of_column(c)) and row r (output neuron neuron_of_column(r)) of layer l + 1
    constexpr int kShare = kHiddenGrads / kCluster;
    for (int i = tid; i < kShare; i += kBlockThreads) {
      const int e = static_cast<int>(rank) * kShare + i;
      float v = ld_dsmem_f32(hg[0] + 4u * e);
#pragma unroll
      for (int r = 1; r < kCluster; ++r) v += ld_dsmem_f32(hg[r] + 4u * e);
      const int o = neuron_of_column(e & 63), n = neuron_of_column((e >> 6) & 63);
      crow[kHiddenBase + (e >> 12) * kHiddenStride + o * kWidth + n] = v;
    }
    if (rank == 0) {  // W0, b0, b1..b3, w_out, b_out and the loss
      int gi = -1, col = 0;
      if (tid < 2 * kWidth) {
        gi = kGW0 + tid;
        col = tid;
      } else if (tid < 3 * kWidth) {
        gi = kGBias + (tid - 2 * kWidth);
        col = kB0 + (tid - 2 * kWidth);
      } else if (tid < 6 * kWidth) {
        const int l = (tid - 3 * kWidth) >> 6, o = (tid - 3 * kWidth) & 63;
        gi = kGBias + (l + 1) * kWidth + o;
        col = kHiddenBase + l * kHiddenStride + kWidth * kWidth + o;
      } else if (tid < 7 * kWidth) {
        gi = kGWout + (tid - 6 * kWidth);
        col = kOutBase + (tid - 6 * kWidth);
      } else if (tid == 7 * kWidth) {
        gi = kGBout;
        col = kOutBase + kWidth;
      } else if (tid == 7 * kWidth + 1) {
        gi = kGLoss;
        col = kLossColumn;
      }
      if (gi >= 0) {
        float v = ld_dsmem_f32(gr[0] + 4u * gi);
#pragma unroll
        for (int r = 1; r < kCluster; ++r) v += ld_dsmem_f32(gr[r] + 4u * gi);
        crow[col] = v;
      }
    }
  }
  cluster_sync();  // no CTA leaves while a peer still reads its shared memory
}

template <bool kPoisson>
cudaError_t set_attributes() {
  // The setmaxnreg split assumes kLaunchRegs per thread at launch; a build with fewer would
  // leave the epilogue's register raise waiting forever, so it is refused here.
  cudaFuncAttributes attr;
  const cudaError_t e = cudaFuncGetAttributes(&attr, backward_tc_kernel<kPoisson>);
  if (e != cudaSuccess) return e;
  if (attr.numRegs != kLaunchRegs) return cudaErrorInvalidKernelImage;
  return cudaFuncSetAttribute(backward_tc_kernel<kPoisson>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

}  // namespace

cudaError_t prepare_backward_tc() {
  const cudaError_t e = set_attributes<false>();
  return e == cudaSuccess ? set_attributes<true>() : e;
}

int backward_tc_grid(int64_t n, int64_t nb, const DeviceInfo& dev) {
  const int64_t tiles = (n + kTile - 1) / kTile + (nb + kTile - 1) / kTile;
  const int64_t whole = (tiles + kCluster - 1) / kCluster * kCluster;  // whole clusters
  return static_cast<int>(std::min<int64_t>(whole, dev.sms / kCluster * kCluster));
}

int backward_tc_rows(int64_t n, int64_t nb, const DeviceInfo& dev) {
  return backward_tc_grid(n, nb, dev) / kCluster;
}

size_t backward_tc_workspace_bytes(int64_t n, int64_t nb, const DeviceInfo& dev) {
  const size_t grid = static_cast<size_t>(backward_tc_grid(n, nb, dev));
  return (static_cast<size_t>(kWeightBlocks) * (kLayerBytes / 4) + grid * kRowStride +
          grid * kScratchFloats) *
         sizeof(float);
}

cudaError_t launch_backward_tc(const PointSets& points, const float* params,
                               const float* grad_u, const float* grad_lap, float* grad_coords,
                               float* lap_out, float* workspace, bool poisson,
                               const DeviceInfo& dev, cudaStream_t stream) {
  PointSets ps = points;
  ps.tiles = (ps.n + kTile - 1) / kTile;
  const int64_t tiles = ps.tiles + (ps.nb + kTile - 1) / kTile;
  const int grid = backward_tc_grid(ps.n, ps.nb, dev);
  float* wsplit = workspace;
  float* partials = wsplit + kWeightBlocks * (kLayerBytes / 4);
  float* scratch = partials + static_cast<size_t>(grid) * kRowStride;
  prep_weights_kernel<<<kWeightBlocks, 512, 0, stream>>>(params, wsplit);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // The step kernel's set-up (parameter staging, scales, the first tile's layer 0) overlaps
  // the pre-split; its first read of the split weights waits for it.
  if (poisson) {
    e = launch_dependent(backward_tc_kernel<true>, dim3(grid), dim3(kBlockThreads), kSmemBytes,
                         stream, ps, params, wsplit, nullptr, nullptr, grad_coords, lap_out,
                         partials, scratch, tiles, dev.status);
  } else {
    e = launch_dependent(backward_tc_kernel<false>, dim3(grid), dim3(kBlockThreads),
                         kSmemBytes, stream, ps, params, wsplit, grad_u, grad_lap,
                         grad_coords, nullptr, partials, scratch, tiles, dev.status);
  }
  return e;
}

float* backward_tc_partials(float* workspace) {
  return workspace + kWeightBlocks * (kLayerBytes / 4);
}

}  // namespace fhb
