// Launchers shared between the kernel translation units and the C ABI layer (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fhb {

// Floats per partial-gradient row of the backward workspace: 12,737 gradients, one loss
// partial (fused step only), padded to a 16-byte multiple.
constexpr int kRowStride = 12740;
constexpr int kLossColumn = 12737;

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
int backward_grid(int64_t n, const DeviceInfo& dev);
// mode 0: plain VJP with caller-supplied grad_u/grad_lap; mode 1: fused Poisson step.
cudaError_t launch_backward_fp32(const float* coords, const float* params,
                                 const float* grad_u, const float* grad_lap,
                                 float* grad_coords, float* lap_out, float* partials,
                                 int64_t n, int64_t n_total, bool poisson,
                                 const DeviceInfo& dev, cudaStream_t stream);
cudaError_t launch_reduce_rows(const float* partials, int rows, float* grad_params,
                               float* loss, cudaStream_t stream);

// ---- backward_tc.cu ----
cudaError_t prepare_backward_tc();
int backward_tc_grid(int64_t n, const DeviceInfo& dev);
// Workspace: pre-split weights, one partial-gradient row per CTA, per-CTA L2 scratch.
size_t backward_tc_workspace_bytes(int64_t n, const DeviceInfo& dev);
float* backward_tc_partials(float* workspace);
cudaError_t launch_backward_tc(const float* coords, const float* params, const float* grad_u,
                               const float* grad_lap, float* grad_coords, float* lap_out,
                               float* workspace, int64_t n, int64_t n_total, bool poisson,
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
