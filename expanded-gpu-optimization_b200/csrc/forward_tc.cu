// 3xTF32 tcgen05/TMEM forward-Laplacian kernel (forward versions 3, 4, 5).
//
// Same math as the FP32 kernel and the reference (csrc/fused_residual.cu:16-23), with the
// three hidden 64x64 jet GEMMs on the 5th-generation tensor cores. Each hidden layer is,
// per tile of 128 points and per jet component c in {v, d/dx, d/dy, L},
//     Z_c[128 x 64] = H_c[128 x 64] . W^T,
// run as tcgen05.mma kind::tf32 with M = 128 points, N = 64 output neurons, K = 8 per
// instruction. FP32 accuracy is kept by the 3xTF32 split (x = x_hi + x_lo, both rounded to
// TF32): Z += H_hi W_hi + H_lo W_hi + H_hi W_lo, accumulated in FP32 in tensor memory.
//
// Where the data lives (per CTA, one CTA per SM, persistent over tiles):
//   * weights: all three hidden layers, hi and lo, pre-split once per CTA into the K-major
//     no-swizzle canonical layout in shared memory (96 KB) -- the MMA's B operand;
//   * TMEM (512 columns x 128 lanes, lane = point):
//       [0, 256)   accumulators D_c, component c at columns 64c..64c+63;
//       [256, 512) a ring of 2 A-operand chunks; a chunk is two K steps (16 input
//                  neurons) of the next layer's activations: (component, hi/lo) blocks of
//                  16 columns.
//     The A operand lives in TMEM, not shared memory: with N = 64 an A tile read from
//     shared memory would need ~1.5x the shared-memory bandwidth an SM has.
//   * 16 warps: warp w serves TMEM lanes 32(w%4)..+31 (its quadrant) and, with s = w/4,
//     neurons 16a+4s+t. Per layer it loads its 4 x 16 accumulators (16 x tcgen05.ld.x4),
//     applies the tanh jet in registers and writes TF32 hi/lo activations chunk by chunk
//     into the ring (tcgen05.st) for the next layer. Warp s owns the strided neurons
//     16a+4s+{0..3} (a = 0..3), so chunk j (neurons 16j..16j+15, natural K order) gets 4
//     neurons from every warp and all 16 warps contribute to every chunk;
//   * the warp that completes a chunk last (an acq_rel counter per ring slot) issues its
//     MMAs as a converged warp (elect.sync picks the issuing lane; issued from a divergent
//     lane these small MMAs cost ~4x their execution time): 2 K steps x 4 components x 3
//     products, then tcgen05.commit to free the slot, and after a layer's 4th chunk a
//     commit that marks D complete. A warp contributes to
//     chunk 0 of layer l+1 only after it has read D of layer l, so when the last
//     contribution arrives D may be overwritten -- no separate "D free" barrier.
//   So the MMAs of layer l+1 consume chunk j while the epilogue of layer l produces chunk
//   j+1. (No dedicated MMA warp: a 17th warp would put 5 warps on one SM sub-partition and
//   cap registers at 96; with 16 warps each thread gets 128.)
// Layer 0 (2 inputs) and the output layer (1 output) are elementwise/epilogue work. The
// epilogue, not the tensor core, bounds this kernel, so it is kept lean: tanh_fast (SFU
// exp2 + reciprocal), a 2-instruction TF32 split (hi = cvt.rna, lo = x - hi, which the
// tensor core truncates to TF32) and 16-neuron chunks to halve the synchronisation.
// Every mbarrier wait is bounded; a wait that gives up raises FHB_STATUS_MMA_TIMEOUT, sets
// a CTA abort flag that stops the other warps, and the kernel frees TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace fhb {
namespace {

constexpr int kTile = 128;            // points per tile = MMA M = TMEM lanes
constexpr int kWarps = 16;            // 4 per TMEM lane quadrant
constexpr int kThreads = kWarps * 32;
constexpr int kChunks = 4;            // chunks of 16 neurons (2 K steps) per 64-wide layer
constexpr int kChunksPerTile = kHiddenGemms * kChunks;
constexpr int kRing = 2;
constexpr uint32_t kSlotCols = 128;   // 4 components x {hi, lo} x 16 K positions
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kRingCol = 256;
constexpr uint32_t kIdesc = tc::idesc_tf32(128, 64);

// Shared memory layout (bytes).
constexpr int kOperandBytes = kWidth * kWidth * 4;  // one [64 x 64] tf32 operand: 16 KB
constexpr int kSmallOff = 6 * kOperandBytes;        // W0[128] b0[64] b1..b3[192] wout[64] bout
constexpr int kSmW0 = 0, kSmB0 = 128, kSmB = 192, kSmWout = 384, kSmBout = 448;
constexpr int kSmallFloats = 512;
constexpr int kRedOff = kSmallOff + kSmallFloats * 4;  // [8][128] partial sums
constexpr int kBarOff = kRedOff + 8 * kTile * 4;       // mbarriers: empty[2], dfull, red
constexpr int kCountOff = kBarOff + 8 * 8;             // per-slot contribution counters
constexpr int kMiscOff = kCountOff + 4 * 4;            // TMEM base, abort flag
constexpr int kSmemUsed = kMiscOff + 16;
// Padded so two CTAs never share an SM (each allocates all 512 TMEM columns).
constexpr int kSmemBytes = 120 * 1024;
static_assert(kSmemUsed <= kSmemBytes, "shared memory layout overflow");

// Canonical K-major no-swizzle layout of a [64 rows x 64 K] tf32 operand: 8x4 core
// matrices of 128 B; K chunks of 4 at LBO = 128 B, 8-row groups at SBO = 2048 B.
constexpr uint32_t kLbo = 128, kSbo = 2048;

struct Ctx {
  uint8_t* smem;
  uint64_t* empty;            // [kRing] ring slot consumed by its MMAs (tcgen05.commit)
  uint64_t* dfull;            // accumulators complete (tcgen05.commit)
  uint64_t* red;              // output-layer partial sums written (16 warps arrive)
  uint32_t* count;            // [kRing] contributions to each slot, monotonic
  volatile uint32_t* abort_flag;
  unsigned int* status;
  uint32_t tmem;
};

// Bounded wait that also gives up when another warp has aborted the CTA.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Ctx& cx) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
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



// The 24 MMAs of one chunk: K steps 2j, 2j+1 of hidden GEMM `layer`, A from ring slot
// `slot` (component c, hi/lo sp, K step kk at columns 32c + 16sp + 8kk of the slot).
__device__ __forceinline__ void issue_chunk_mmas(const Ctx& cx, int layer, int j,
                                                 uint32_t slot) {
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const uint32_t w_hi = smem_u32(cx.smem + (2 * layer) * kOperandBytes + 256 * (2 * j + kk));
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
  tc::commit_warp(&cx.empty[slot]);
  if (j == kChunks - 1) tc::commit_warp(cx.dfull);
}


// Write chunk `n` (this warp's 4 neurons x 4 components, TF32 hi and lo) into ring slot
// n % kRing; the warp completing the chunk last issues its MMAs. False if aborted.
__device__ __forceinline__ bool produce_chunk(uint32_t n, const float (&h)[4][4],
                                              uint32_t tmem_warp, int s, const Ctx& cx) {
  const uint32_t slot = n % kRing;
  if (!warp_wait(&cx.empty[slot], ((n / kRing) & 1u) ^ 1u, cx)) return false;
  tc::fence_after_sync();
  const uint32_t base = tmem_warp + kRingCol + kSlotCols * slot + 4u * s;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) tc::split_tf32(h[c][t], hi[t], lo[t]);
    tc::st_x4(base + 32u * c, hi[0], hi[1], hi[2], hi[3]);
    tc::st_x4(base + 32u * c + 16u, lo[0], lo[1], lo[2], lo[3]);
  }
  tc::wait_st();
  tc::fence_before_sync();
  __syncwarp();
  uint32_t last = 0;
  if ((threadIdx.x & 31) == 0) last = (count_contribution(&cx.count[slot]) % kWarps) == kWarps - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {  // warp-uniform: the whole converged warp issues, elect.sync picks a lane
    tc::fence_after_sync();
    const uint32_t in_tile = n % kChunksPerTile;
    issue_chunk_mmas(cx, static_cast<int>(in_tile / kChunks), static_cast<int>(in_tile % kChunks),
                     slot);
    __syncwarp();
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    forward_tc_kernel(const float* __restrict__ coords, const float* __restrict__ params,
                      float* __restrict__ u_out, float* __restrict__ lap_out, int64_t n,
                      int64_t tiles, unsigned int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  float* small = reinterpret_cast<float*>(smem + kSmallOff);
  float* red = reinterpret_cast<float*>(smem + kRedOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  Ctx cx;
  cx.smem = smem;
  cx.empty = bars;
  cx.dfull = bars + kRing;
  cx.red = bars + kRing + 1;
  cx.count = reinterpret_cast<uint32_t*>(smem + kCountOff);
  cx.abort_flag = reinterpret_cast<volatile uint32_t*>(smem + kMiscOff + 4);
  cx.status = status;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The first tile's point, requested first: its latency overlaps the set-up below.
  const int row0 = 32 * (warp & 3) + lane;
  float nx0 = 0.0f, nx1 = 0.0f;
  {
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kTile + row0;
    if (p < n) {
      nx0 = coords[2 * p];
      nx1 = coords[2 * p + 1];
    }
  }

  // ---- set-up: split weights to TF32 hi/lo in the canonical layout, small params ----
  // Element e of an operand, enumerated as (row group, K chunk, row in group, K in chunk),
  // sits at byte 4e of the canonical layout: consecutive threads store consecutive words.
  // All 25 loads of a thread (24 weights, one small parameter) are issued before any is used.
  static_assert(kSmallFloats == kThreads, "one small parameter per thread");
  {
    float sv = 0.0f;
    {
      const int i = threadIdx.x;
      if (i < kSmB0) sv = params[i];                                       // W0
      else if (i < kSmB) sv = params[kB0 + (i - kSmB0)];                   // b0
      else if (i < kSmWout) {                                              // b1..b3
        const int l = (i - kSmB) >> 6, o = (i - kSmB) & 63;
        sv = params[kHiddenBase + l * kHiddenStride + kWidth * kWidth + o];
      } else if (i < kSmBout) sv = params[kOutBase + (i - kSmWout)];       // w_out
      else if (i == kSmBout) sv = params[kOutBase + kWidth];               // b_out
    }
    constexpr int kPerThread = kHiddenGemms * kWidth * kWidth / kThreads;  // 24
    float w[kPerThread];
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) {
      const int idx = threadIdx.x + r * kThreads;
      const int layer = idx >> 12, e = idx & 4095;
      const int row = ((e >> 9) << 3) | ((e >> 2) & 7);
      const int k = (((e >> 5) & 15) << 2) | (e & 3);
      w[r] = params[kHiddenBase + layer * kHiddenStride + row * kWidth + k];
    }
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) {
      const int idx = threadIdx.x + r * kThreads;
      const int layer = idx >> 12, e = idx & 4095;
      const uint32_t hi = tc::to_tf32(w[r]);
      const uint32_t lo = tc::to_tf32(w[r] - __uint_as_float(hi));
      reinterpret_cast<uint32_t*>(smem + (2 * layer) * kOperandBytes)[e] = hi;
      reinterpret_cast<uint32_t*>(smem + (2 * layer + 1) * kOperandBytes)[e] = lo;
    }
    small[threadIdx.x] = sv;
  }
  if (threadIdx.x == 0) {
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&cx.empty[r], 1);
      cx.count[r] = 0u;
    }
    mbar_init(cx.dfull, 1);
    mbar_init(cx.red, kWarps);
    *cx.abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_base_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_proxy_async_smem();  // weight operands visible to the tensor core
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  cx.tmem = *tmem_base_slot;

  const int q = warp & 3;   // TMEM lane quadrant
  const int s = warp >> 2;  // neuron block 16s..16s+15
  const uint32_t tmem_warp = cx.tmem + (static_cast<uint32_t>(32 * q) << 16);
  const int row = 32 * q + lane;
  uint32_t chunk = 0, mlayer = 0, tile_count = 0;
  bool ok = true;
  // Points of the next tile are loaded one tile ahead, so the load latency (long when the
  // points sit in pinned host memory read over the host link) overlaps a tile of work.
  for (int64_t tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++tile_count) {
    const int64_t p = tile * kTile + row;
    const bool active = p < n;
    const float x0 = nx0, x1 = nx1;
    {
      const int64_t pn = p + static_cast<int64_t>(gridDim.x) * kTile;
      if (pn < n) {
        nx0 = coords[2 * pn];
        nx1 = coords[2 * pn + 1];
      }
    }

    // layer 0: z = W0 x + b0, z_J = W0 columns, z_L = 0
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      float h[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int o = 16 * j + 4 * s + t;
        const float w0 = small[kSmW0 + 2 * o], w1 = small[kSmW0 + 2 * o + 1];
        tanh_jet_fast(fmaf(w0, x0, fmaf(w1, x1, small[kSmB0 + o])), w0, w1, 0.0f, h[0][t],
                      h[1][t], h[2][t], h[3][t]);
      }
      if (!(ok = produce_chunk(chunk++, h, tmem_warp, s, cx))) break;
    }

    for (int l = 0; ok && l < kHiddenGemms; ++l, ++mlayer) {
      if (!(ok = warp_wait(cx.dfull, mlayer & 1u, cx))) break;
      tc::fence_after_sync();
      // d[c][4a + t] = component c of neuron 16a + 4s + t
      float d[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tc::ld_x4(tmem_warp + 64u * c + 16u * a + 4u * s,
                    *reinterpret_cast<float(*)[4]>(&d[c][4 * a]));
      tc::wait_ld();
      const float* bias = small + kSmB + 64 * l;
#pragma unroll
      for (int i = 0; i < 16; ++i) d[0][i] += bias[16 * (i >> 2) + 4 * s + (i & 3)];

      if (l + 1 < kHiddenGemms) {
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
          float h[4][4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int i = 4 * j + t;
            tanh_jet_fast(d[0][i], d[1][i], d[2][i], d[3][i], h[0][t], h[1][t], h[2][t],
                          h[3][t]);
          }
          if (!(ok = produce_chunk(chunk++, h, tmem_warp, s, cx))) break;
        }
      } else {
        // output layer: u = w.v + b, lap = w.L, over this warp's 16 neurons
        float pu = 0.0f, pl = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v, j0, j1, lv;
          tanh_jet_fast(d[0][i], d[1][i], d[2][i], d[3][i], v, j0, j1, lv);
          const float w = small[kSmWout + 16 * (i >> 2) + 4 * s + (i & 3)];
          pu = fmaf(w, v, pu);
          pl = fmaf(w, lv, pl);
        }
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

cudaError_t prepare_forward_tc() {
  return cudaFuncSetAttribute(forward_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes);
}

cudaError_t launch_forward_tc(const float* coords, const float* params, float* u, float* lap,
                              int64_t n, const DeviceInfo& dev, cudaStream_t stream) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sms));
  forward_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(coords, params, u, lap, n, tiles,
                                                            dev.status);
  return cudaGetLastError();
}

}  // namespace fhb
