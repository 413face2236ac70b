// 3xFP16 tcgen05/TMEM forward-Laplacian kernel (forward version 3, the default tensor-core
// path; versions 4 and 5 run the 3xTF32 kernel of forward_tc.cu).
//
// Same math, tiling and warp roles as forward_tc.cu -- per tile of 128 points and hidden
// layer, Z_c[128 x 64] = H_c[128 x 64] . W^T for the four jet components c, with the A
// operand (activations) in TMEM and B (weights) in shared memory -- but the operands are
// f16 pairs (tcgen05.mma kind::f16, K = 16 per instruction) instead of tf32:
//   x = hi + lo with hi = f16(x), lo' = f16(2^11 (x - hi))  (11 + 11 significant bits, the
//   precision of the 3xTF32 split), and
//   D = A_hi (2^11 W_hi) + A_lo' W_hi + A_hi W_lo' = 2^11 A W   (FP32 accumulation),
// so a 16-neuron chunk is 12 MMAs instead of 24 and writes half the bytes into TMEM. Both
// halves matter: the tf32 kernel spends its layer time on the MMAs, on the chunk stores and
// on the TMEM traffic between them (a chunk's 24 MMAs take 0.57-0.74 us instead of 0.39 us
// while 16 warps store the next chunk).
// Range: f16 holds magnitudes below 65,504. Each launch derives power-of-2 scales from the
// weights -- tau_l maps max|W_l| to <= 16 (so 2^11 W_hi stays finite), sigma_{l,c} maps an
// upper bound of component c of GEMM l's A operand to <= 2^14 -- applies them before the
// split and removes them exactly from the accumulators (D * 1 / (2^11 sigma tau), a power of
// 2). The bounds: |v| <= 1; |dv/dx|, |dv/dy| grow by N_l = max row-abs-sum of W_l per layer;
// |Lv| becomes N_l |Lv| + (N_l Bx)^2 + (N_l By)^2 (tanh' <= 1 and 2 |tanh tanh'| <= 1).
// Values far below their bound keep full relative precision until they are 2^28 times
// smaller. The scales depend on the weights only (fixed-order warp reductions), so every CTA
// and every shard of a batch uses the same ones.
// TMEM (512 columns): accumulators D_c at columns 64c.. (256) and a ring of 4 chunks of 64
// columns (component c, hi/lo: 8 columns of f16 pairs, K positions 2j and 2j+1 in column j),
// i.e. a whole layer's A operand. Every mbarrier wait is bounded, as in forward_tc.cu.
#include <algorithm>

#include <cuda_fp16.h>

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
constexpr int kRing = 4;
constexpr uint32_t kSlotCols = 64;    // 4 components x {hi, lo} x 8 columns (16 f16 K positions)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kRingCol = 256;
constexpr uint32_t kIdesc = tc::idesc_f16(128, 64);
constexpr float kLoScale = 2048.0f;  // lo' = 2^11 (x - hi)

// Shared memory layout (bytes).
constexpr int kOperandBytes = kWidth * kWidth * 2;  // one [64 x 64] f16 operand: 8 KB
constexpr int kSmallOff = 9 * kOperandBytes;        // W0[128] b0[64] b1..b3[192] wout[64] bout
constexpr int kSmW0 = 0, kSmB0 = 128, kSmB = 192, kSmWout = 384, kSmBout = 448;
constexpr int kSmallFloats = 512;
constexpr int kRedOff = kSmallOff + kSmallFloats * 4;  // [8][128] partial sums
constexpr int kBarOff = kRedOff + 8 * kTile * 4;       // mbarriers: empty[4], dfull, red
constexpr int kCountOff = kBarOff + 8 * 8;             // per-slot contribution counters
constexpr int kMiscOff = kCountOff + 4 * 4;            // TMEM base, abort flag
constexpr int kScaleOff = kMiscOff + 16;               // sigma[3][4], unscale[3][4], tau[3]
constexpr int kSmemUsed = kScaleOff + 32 * 4;
// Padded so two CTAs never share an SM (each allocates all 512 TMEM columns).
constexpr int kSmemBytes = 120 * 1024;
static_assert(kSmemUsed <= kSmemBytes, "shared memory layout overflow");

// Canonical K-major no-swizzle layout of a [64 rows x 64 K] f16 operand: core matrices of
// 8 rows x 8 elements (128 B); K chunks of 8 at LBO = 128 B, 8-row groups at SBO = 1024 B.
constexpr uint32_t kLbo = 128, kSbo = 1024;

struct Ctx {
  uint8_t* smem;
  uint64_t* empty;            // [kRing] ring slot consumed by its MMAs (tcgen05.commit)
  uint64_t* dfull;            // accumulators complete (tcgen05.commit)
  uint64_t* red;              // output-layer partial sums written (16 warps arrive)
  uint32_t* count;            // [kRing] contributions to each slot, monotonic
  volatile uint32_t* abort_flag;
  unsigned int* status;
  uint32_t tmem;
  const float* sigma;         // [3][4] A-operand scale of GEMM l, component c (power of 2)
  const float* unscale;       // [3][4] 1 / (2048 sigma tau) for the accumulators of GEMM l
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



// The 12 MMAs of one chunk (K = 16 input neurons) of hidden GEMM `layer`, A from ring slot
// `slot`: per component, A_hi (2^11 W_hi) + A_lo' W_hi + A_hi W_lo'.
__device__ __forceinline__ void issue_chunk_mmas(const Ctx& cx, int layer, int j, uint32_t slot) {
  const uint32_t w0 = smem_u32(cx.smem + (3 * layer) * kOperandBytes + 256 * j);
  const uint64_t b_hs = tc::smem_desc_kmajor(w0, kLbo, kSbo);
  const uint64_t b_hi = tc::smem_desc_kmajor(w0 + kOperandBytes, kLbo, kSbo);
  const uint64_t b_lo = tc::smem_desc_kmajor(w0 + 2 * kOperandBytes, kLbo, kSbo);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t d = cx.tmem + 64u * c;
    const uint32_t a_hi = cx.tmem + kRingCol + kSlotCols * slot + 16u * c;
    const uint32_t a_lo = a_hi + 8u;
    tc::mma_f16_ts_warp(d, a_hi, b_hs, kIdesc, j > 0 ? 1u : 0u);
    tc::mma_f16_ts_warp(d, a_lo, b_hi, kIdesc, 1u);
    tc::mma_f16_ts_warp(d, a_hi, b_lo, kIdesc, 1u);
  }
  tc::commit_warp(&cx.empty[slot]);
  if (j == kChunks - 1) tc::commit_warp(cx.dfull);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
// Largest power of 2 <= x for x in [2^-126, 2^127]; clamped to that range otherwise.
__device__ __forceinline__ float pow2_floor(float x) {
  x = fminf(fmaxf(x, 1.17549435e-38f), 1.7e38f);
  return __uint_as_float(__float_as_uint(x) & 0x7F800000u);
}

// f16 pairs for the A operand: hi = f16(x) and lo' = f16(2^11 (x - hi)), elements a (even K)
// in the low half.
__device__ __forceinline__ uint32_t pack_hi(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_lo(float a, float b) {
  const float ha = __half2float(__float2half_rn(a)), hb = __half2float(__float2half_rn(b));
  const __half2 h = __floats2half2_rn((a - ha) * kLoScale, (b - hb) * kLoScale);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Write chunk `n` (this warp's 4 neurons x 4 components, scaled by sigma of their GEMM, as f16
// hi and lo' pairs) into ring slot n % kRing; the warp completing the chunk last issues its
// MMAs. False if aborted.
__device__ __forceinline__ bool produce_chunk(uint32_t n, const float (&h)[4][4],
                                              uint32_t tmem_warp, int s, const Ctx& cx) {
  const uint32_t slot = n % kRing;
  if (!warp_wait(&cx.empty[slot], ((n / kRing) & 1u) ^ 1u, cx)) return false;
  tc::fence_after_sync();
  const uint32_t base = tmem_warp + kRingCol + kSlotCols * slot + 2u * s;
  const float* sig = cx.sigma + 4 * ((n % kChunksPerTile) / kChunks);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float g = sig[c];
    const float a0 = h[c][0] * g, a1 = h[c][1] * g, a2 = h[c][2] * g, a3 = h[c][3] * g;
    tc::st_x2(base + 16u * c, pack_hi(a0, a1), pack_hi(a2, a3));
    tc::st_x2(base + 16u * c + 8u, pack_lo(a0, a1), pack_lo(a2, a3));
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
    forward_f16_kernel(const float* __restrict__ coords, const float* __restrict__ params,
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

  // ---- set-up: small params, the f16 operand scales, then the split weights ----
  // Every load of the set-up is issued before any is used (one memory round trip): the small
  // parameter, 24 values for the weight-row statistics and 12 pairs for the operand split.
  static_assert(kSmallFloats == kThreads, "one small parameter per thread");
  constexpr int kStatRows = 3 * kWidth / kWarps;                   // 12 rows per warp
  constexpr int kPairs = kHiddenGemms * kWidth * kWidth / 2;       // 6144
  constexpr int kPairsPerThread = kPairs / kThreads;               // 12
  static_assert(kPairs % kThreads == 0, "whole pairs per thread");
  float* scales = reinterpret_cast<float*>(smem + kScaleOff);
  float wp[kPairsPerThread][2];
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
    float rs[kStatRows][2];
#pragma unroll
    for (int i = 0; i < kStatRows; ++i) {  // row warp + 16 i of the 192 hidden-weight rows
      const int r = warp + kWarps * i;
      const float* wr = params + kHiddenBase + (r >> 6) * kHiddenStride + (r & 63) * kWidth;
      rs[i][0] = wr[lane];
      rs[i][1] = wr[lane + 32];
    }
#pragma unroll
    for (int k = 0; k < kPairsPerThread; ++k) {
      const int idx = threadIdx.x + k * kThreads;
      const int layer = idx >> 11, e = (idx & 2047) * 2;
      const int row = ((e >> 9) << 3) | ((e >> 3) & 7);
      const int kk = (((e >> 6) & 7) << 3) | (e & 7);
      const float* wr = params + kHiddenBase + layer * kHiddenStride + row * kWidth + kk;
      wp[k][0] = wr[0];
      wp[k][1] = wr[1];
    }
    // Row statistics: fixed-order warp reductions, so every CTA derives the same scales.
#pragma unroll
    for (int i = 0; i < kStatRows; ++i) {
      const float a = fabsf(rs[i][0]), b = fabsf(rs[i][1]);
      const float sum = warp_sum(a + b), mx = warp_max(fmaxf(a, b));
      if (lane == 0) {
        red[warp + kWarps * i] = sum;  // the output-layer buffer is free during set-up
        red[256 + warp + kWarps * i] = mx;
      }
    }
    small[threadIdx.x] = sv;
  }
  __syncthreads();
  // Power-of-2 scales that keep every f16 operand in range: tau_l maps max|W_l| to <= 16 (so
  // 2^11 W_hi stays finite); sigma_{l,c} maps a bound of component c of the A operand of
  // GEMM l to <= 2^14. Bounds: |v| <= 1; |d/dx|, |d/dy| grow by N_l (max row-abs-sum of W_l)
  // per layer; |L| becomes N_l |L| + (N_l Bx)^2 + (N_l By)^2 (tanh' <= 1, 2 |tanh tanh'| <= 1).
  if (warp == 0) {
    float nrm[3], wmax[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      nrm[l] = warp_max(fmaxf(red[64 * l + lane], red[64 * l + lane + 32]));
      wmax[l] = warp_max(fmaxf(red[256 + 64 * l + lane], red[256 + 64 * l + lane + 32]));
    }
    const float w0x = small[kSmW0 + 2 * lane], w0y = small[kSmW0 + 2 * lane + 1];
    const float w0x2 = small[kSmW0 + 2 * (lane + 32)], w0y2 = small[kSmW0 + 2 * (lane + 32) + 1];
    float bx = warp_max(fmaxf(fabsf(w0x), fabsf(w0x2)));
    float by = warp_max(fmaxf(fabsf(w0y), fabsf(w0y2)));
    float bl = warp_max(fmaxf(fmaf(w0x, w0x, w0y * w0y), fmaf(w0x2, w0x2, w0y2 * w0y2)));
    if (lane == 0) {
      for (int l = 0; l < 3; ++l) {
        const float tau = pow2_floor(16.0f / fmaxf(wmax[l], 1e-30f));
        const float bnd[4] = {1.0f, bx, by, bl};
        for (int c = 0; c < 4; ++c) {
          const float sig = pow2_floor(16384.0f / fmaxf(bnd[c], 1e-30f));
          scales[4 * l + c] = sig;
          scales[12 + 4 * l + c] = 1.0f / (kLoScale * sig * tau);
        }
        scales[24 + l] = tau;
        const float nx = nrm[l] * bx, ny = nrm[l] * by;
        bl = fmaf(nrm[l], bl, fmaf(nx, nx, ny * ny));
        bx = nx;
        by = ny;
      }
    }
  }
  __syncthreads();
  // The split: pairs of adjacent K elements, enumerated (row group, K chunk of 8, row in
  // group, K pair) so consecutive threads store consecutive words of the canonical layout.
#pragma unroll
  for (int k = 0; k < kPairsPerThread; ++k) {
    const int idx = threadIdx.x + k * kThreads;
    const int layer = idx >> 11, e = (idx & 2047) * 2;
    const float tau = scales[24 + layer];
    const float a = wp[k][0] * tau, b = wp[k][1] * tau;
    const __half2 hi = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(hi);
    const __half2 hs = __floats2half2_rn(hf.x * kLoScale, hf.y * kLoScale);
    const __half2 lo = __floats2half2_rn((a - hf.x) * kLoScale, (b - hf.y) * kLoScale);
    uint8_t* base = smem + (3 * layer) * kOperandBytes + 2 * e;
    *reinterpret_cast<__half2*>(base) = hs;
    *reinterpret_cast<__half2*>(base + kOperandBytes) = hi;
    *reinterpret_cast<__half2*>(base + 2 * kOperandBytes) = lo;
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
  cx.sigma = reinterpret_cast<const float*>(smem + kScaleOff);
  cx.unscale = cx.sigma + 12;

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
      for (int c = 0; c < 4; ++c) {
        const float us = cx.unscale[4 * l + c];
#pragma unroll
        for (int i = 0; i < 16; ++i) d[c][i] *= us;
      }
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

cudaError_t prepare_forward_f16() {
  return cudaFuncSetAttribute(forward_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes);
}

cudaError_t launch_forward_f16(const float* coords, const float* params, float* u, float* lap,
                               int64_t n, const DeviceInfo& dev, cudaStream_t stream) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sms));
  forward_f16_kernel<<<grid, kThreads, kSmemBytes, stream>>>(coords, params, u, lap, n, tiles,
                                                            dev.status);
  return cudaGetLastError();
}

}  // namespace fhb
