// Launchers shared between the kernel translation units and the C ABI layer (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

#ifdef __CUDACC__
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

// ---- forward_fp32.cu ----
cudaError_t prepare_forward_fp32();
// tile: 0 -> 32-point tiles, 1 -> 128-point tiles, 2 -> 64-point tiles
cudaError_t launch_forward_fp32(int tile, const float* coords, const float* params, float* u,
                                float* lap, int64_t n, const DeviceInfo& dev,
                                cudaStream_t stream);

// ---- forward_tc.cu ----
cudaError_t prepare_forward_tc();
cudaError_t launch_forward_tc(const float* coords, const float* params, float* u, float* lap,
                              int64_t n, const DeviceInfo& dev, cudaStream_t stream);

// ---- backward_fp32.cu ----
cudaError_t prepare_backward_fp32();
int backward_grid(int64_t n, int64_t nb, const DeviceInfo& dev);
// poisson: fused Poisson / PINN step (loss gradient formed in the kernel); otherwise the
// plain VJP of the interior set with caller-supplied grad_u / grad_lap.
cudaError_t launch_backward_fp32(const PointSets& points, const float* params,
                                 const float* grad_u, const float* grad_lap,
                                 float* grad_coords, float* lap_out, float* partials,
                                 bool poisson, const DeviceInfo& dev, cudaStream_t stream);
cudaError_t launch_reduce_rows(const float* partials, int rows, float* grad_params,
                               float* loss, cudaStream_t stream);

// ---- backward_tc.cu ----
cudaError_t prepare_backward_tc();
int backward_tc_grid(int64_t n, int64_t nb, const DeviceInfo& dev);
// Workspace: pre-split weights, one partial-gradient row per CTA, per-CTA L2 scratch.
size_t backward_tc_workspace_bytes(int64_t n, int64_t nb, const DeviceInfo& dev);
float* backward_tc_partials(float* workspace);
// poisson: the loss gradient is formed in the kernel (residual term for the interior set,
// boundary term for the boundary set); otherwise grad_u / grad_lap of the interior set.
cudaError_t launch_backward_tc(const PointSets& points, const float* params,
                               const float* grad_u, const float* grad_lap, float* grad_coords,
                               float* lap_out, float* workspace, bool poisson,
                               const DeviceInfo& dev, cudaStream_t stream);

// ---- adam.cu ----
cudaError_t launch_adam(float* params, const float* grad, float* exp_avg, float* exp_avg_sq,
                        int64_t count, int64_t* step, float lr, float beta1, float beta2,
                        float eps, cudaStream_t stream);
cudaError_t launch_debug_tanh(const float* x, float* out, int64_t n, int fast,
                              cudaStream_t stream);
cudaError_t launch_bounded_wait_selftest(uint64_t limit_ns, unsigned int* status,
                                         cudaStream_t stream);

}  // namespace fhb
