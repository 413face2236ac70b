// Launchers shared between the kernel translation units and the C ABI layer (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/fused_hoad_b200.h"

namespace fhb {

// Floats per partial-gradient row of the backward workspace: 12,737 gradients, one loss
// partial (fused step only), padded to a 16-byte multiple.
constexpr int kRowStride = 12740;
constexpr int kLossColumn = 12737;

// The points of one backward launch: the interior set (the VJP's points, or the collocation
// points of the Poisson residual) and, for the PINN step, a boundary set whose loss term is
// bweight * u^2 / nb_total. Tiles of the interior set come first, then the boundary's.
struct PointSets {
  const float* interior = nullptr;  // [n][2]
  int64_t n = 0;
  int64_t tiles = 0;                // tiles of the interior set (set by the launcher)
  const float* boundary = nullptr;  // [nb][2]
  int64_t nb = 0;
  float inv_total = 0.0f;           // 1 / n_total: the residual term's normaliser
  float inv_btotal = 0.0f;          // 1 / nb_total
  float bweight = 0.0f;             // boundary term weight
};

// The training step's update: the partial rows are summed per block of kUpdateCols columns
// (kUpdateGroups row groups each), one CTA per block.
constexpr int kUpdateCols = 32;
constexpr int kUpdateGroups = 8;
constexpr int kUpdateBlocks = (kLossColumn + 1 + kUpdateCols - 1) / kUpdateCols;  // 399

// Data-parallel exchange through peer memory (collective.cu). Each rank owns one buffer of
// 64-bit words, words[2][kMaxRanks][kRowStride]: slot = epoch % 2, row = source rank, word =
// (epoch << 32) | bits of the source rank's column sum for that epoch. Every rank stores its
// words into row `rank` of every rank's buffer, so a rank reads only its own memory.
constexpr int kMaxRanks = 8;
constexpr size_t kExchangeWords = 2ull * kMaxRanks * kRowStride;
constexpr size_t kExchangeBytes = kExchangeWords * sizeof(uint64_t);
static_assert(kMaxRanks == FHB_EXCHANGE_MAX_RANKS, "exchange ABI drifted");
static_assert(kRowStride == FHB_EXCHANGE_ROW_WORDS, "exchange ABI drifted");

// Device-resident state of one exchange (one per rank and trainer).
struct ExchangeState {
  uint64_t* peers[kMaxRanks];  // every rank's buffer as mapped in this process (own included)
  uint32_t epoch;              // exchanges completed
  uint32_t done;               // CTAs of the running update that have finished (0 between)
};

struct AdamArgs {
  float* params;
  float* exp_avg;
  float* exp_avg_sq;
  int64_t* step;
  float lr, beta1, beta2, eps;
};

#ifdef __CUDACC__
// Sum of column `col` over the partial rows grp, grp + kUpdateGroups, ... in row order, eight
// loads in flight per batch (the last batch predicated: skipped rows add nothing, so the sum
// is the plain in-order sum bit for bit). Adding the kUpdateGroups results in group order
// gives the column's total; the order is fixed, so every kernel doing this gets the same bits.
__device__ __forceinline__ float column_group_sum(const float* __restrict__ partials, int rows,
                                                  int col, int grp) {
  constexpr int kBatch = 8;
  float acc = 0.0f;
  for (int r = grp; r < rows; r += kBatch * kUpdateGroups) {
    float v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int rr = r + k * kUpdateGroups;
      v[k] = rr < rows ? partials[static_cast<int64_t>(rr) * kRowStride + col] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
      if (r + k * kUpdateGroups < rows) acc += v[k];
  }
  return acc;
}

// torch.optim.Adam's single-tensor update (no weight decay, no amsgrad) for step t:
//   m = lerp(m, g, 1 - beta1); v = beta2 v + (1 - beta2) g^2
//   p -= lr / (1 - beta1^t) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
struct AdamScalars {
  float step_size;
  float bias2_sqrt;
};
__device__ __forceinline__ AdamScalars adam_scalars(int64_t t, float lr, float beta1,
                                                    float beta2) {
  const double bias1 = 1.0 - pow(static_cast<double>(beta1), static_cast<double>(t));
  const double bias2 = 1.0 - pow(static_cast<double>(beta2), static_cast<double>(t));
  return {static_cast<float>(static_cast<double>(lr) / bias1),
          static_cast<float>(sqrt(bias2))};
}
__device__ __forceinline__ void adam_element(float g, float& p, float& m, float& v,
                                             const AdamScalars& s, float beta1, float beta2,
                                             float eps) {
  m = fmaf(1.0f - beta1, g - m, m);
  v = fmaf(beta2, v, (1.0f - beta2) * g * g);
  const float denom = sqrtf(v) / s.bias2_sqrt + eps;
  p = p - s.step_size * (m / denom);
}

// Coordinates of point `row` of tile `tile` (tiles of `tile_points` points), (0, 0) past the
// end of its set.
__device__ __forceinline__ void load_point(const PointSets& ps, int64_t tile, int tile_points,
                                           int row, float& x0, float& x1) {
  const bool b = tile >= ps.tiles;
  const int64_t p = (b ? tile - ps.tiles : tile) * tile_points + row;
  const float* src = b ? ps.boundary : ps.interior;
  x0 = 0.0f;
  x1 = 0.0f;
  if (p < (b ? ps.nb : ps.n)) {
    x0 = src[2 * p];
    x1 = src[2 * p + 1];
  }
}
#endif

struct DeviceInfo {
  int sms = 0;
  int cc_major = 0;
  int cc_minor = 0;
  unsigned int* status = nullptr;  // device address of this device's status word
};

// ---- capi.cu ----
// The current device's one-time set-up (kernel attributes, SM count, the address of its
// status word) and its DeviceInfo: FHB_OK, or the FHB_ERR_* code of the set-up.
int current_device_info(const DeviceInfo** info);
// FHB_OK for cudaSuccess; otherwise remembers `e` for fhb_last_cuda_error and returns
// FHB_ERR_CUDA.
int record_cuda_error(cudaError_t e);

// ---- forward_fp32.cu ----
cudaError_t prepare_forward_fp32();
// tile: 0 -> 32-point tiles, 1 -> 128-point tiles, 2 -> 64-point tiles
// activation: FHB_ACTIVATION_TANH or FHB_ACTIVATION_SILU
cudaError_t launch_forward_fp32(int tile, const float* coords, const float* params, float* u,
                                float* lap, int64_t n, int activation, const DeviceInfo& dev,
                                cudaStream_t stream);

// ---- forward_tc.cu ----
cudaError_t prepare_forward_tc();
// f16: the 3xFP16 operand format (forward version 3), else 3xTF32 (versions 4, 5). SiLU
// always runs the 3xTF32 format (its activations are unbounded, so no weight-derived f16
// range scale exists).
cudaError_t launch_forward_tc(const float* coords, const float* params, float* u, float* lap,
                              int64_t n, bool f16, int activation, const DeviceInfo& dev,
                              cudaStream_t stream);

// ---- biharmonic.cu ----
cudaError_t prepare_biharmonic();
// (u, Laplacian, biharmonic) of the tanh MLP, FP32 CUDA cores.
cudaError_t launch_forward_biharmonic(const float* coords, const float* params, float* u,
                                      float* lap, float* bilap, int64_t n,
                                      const DeviceInfo& dev, cudaStream_t stream);

// ---- backward_fp32.cu ----
cudaError_t prepare_backward_fp32();
int backward_grid(int64_t n, int64_t nb, const DeviceInfo& dev);
// poisson: fused Poisson / PINN step (loss gradient formed in the kernel); otherwise the
// plain VJP of the interior set with caller-supplied grad_u / grad_lap.
cudaError_t launch_backward_fp32(const PointSets& points, const float* params,
                                 const float* grad_u, const float* grad_lap,
                                 float* grad_coords, float* lap_out, float* partials,
                                 bool poisson, int activation, const DeviceInfo& dev,
                                 cudaStream_t stream);
cudaError_t launch_reduce_rows(const float* partials, int rows, float* grad_params,
                               float* loss, cudaStream_t stream);

// ---- backward_tc.cu ----
cudaError_t prepare_backward_tc();
int backward_tc_grid(int64_t n, int64_t nb, const DeviceInfo& dev);
// Partial-gradient rows the tensor-core backward leaves (one per cluster of CTAs).
int backward_tc_rows(int64_t n, int64_t nb, const DeviceInfo& dev);
// Workspace: pre-split weights, one partial-gradient row per CTA, per-CTA L2 scratch.
size_t backward_tc_workspace_bytes(int64_t n, int64_t nb, const DeviceInfo& dev);
float* backward_tc_partials(float* workspace);
// poisson: the loss gradient is formed in the kernel (residual term for the interior set,
// boundary term for the boundary set); otherwise grad_u / grad_lap of the interior set.
cudaError_t launch_backward_tc(const PointSets& points, const float* params,
                               const float* grad_u, const float* grad_lap, float* grad_coords,
                               float* lap_out, float* workspace, bool poisson,
                               const DeviceInfo& dev, cudaStream_t stream);

// Launches `kernel` with programmatic stream serialization: it may start while the kernel
// before it in `stream` is still running, once every CTA of that kernel has called
// allow_dependents() (common.cuh) or exited, and it orders its reads of that kernel's
// results with wait_for_prerequisites(). Stream capture records the same dependency.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- adam.cu ----
cudaError_t launch_adam(float* params, const float* grad, float* exp_avg, float* exp_avg_sq,
                        int64_t count, int64_t* step, float lr, float beta1, float beta2,
                        float eps, cudaStream_t stream);
// ---- collective.cu ----
// The training step's tail in one launch: the column sums of the backward's partial rows,
// with world > 1 the sum over ranks through the peer buffers of `state`, then Adam on the
// parameters; grad_out (kLossColumn + 1 floats, may be null) receives the summed gradient and
// loss, loss_out (may be null) the loss. A peer wait that exceeds wait_limit_ns sets
// FHB_STATUS_PEER_TIMEOUT and leaves that column's parameter unchanged.
cudaError_t launch_step_update(const float* partials, int rows, ExchangeState* state, int world,
                               int rank, uint64_t wait_limit_ns, const AdamArgs& adam,
                               float* grad_out, float* loss_out, unsigned int* status,
                               cudaStream_t stream);
cudaError_t launch_debug_tanh(const float* x, float* out, int64_t n, int fast,
                              cudaStream_t stream);
cudaError_t launch_bounded_wait_selftest(uint64_t limit_ns, unsigned int* status,
                                         cudaStream_t stream);

}  // namespace fhb
