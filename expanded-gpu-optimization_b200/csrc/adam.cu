// Fused Adam over the flat 12,737-float parameter buffer, and the bounded-wait self-test.
//
// Adam follows torch.optim.Adam's single-tensor update (the optimizer of reference
// benchmarks/benchmark_training.py:41), with no weight decay and no amsgrad (adam_element).
// The step counter t lives in device memory so a captured CUDA graph can replay the step.
#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kAdamThreads = 1024;

// One CTA: every thread reads the counter before thread 0 stores the incremented value.
// The elements are processed in blocks of kAdamUnroll per thread with all loads of a block
// issued before any is used, so a 12,737-element buffer takes two round trips to memory.
constexpr int kAdamUnroll = 7;
__global__ void __launch_bounds__(kAdamThreads)
    adam_kernel(float* __restrict__ params, const float* __restrict__ grad,
                float* __restrict__ exp_avg, float* __restrict__ exp_avg_sq, int64_t count,
                int64_t* __restrict__ step, float lr, float beta1, float beta2, float eps) {
  const int64_t t = *step + 1;
  const AdamScalars s = adam_scalars(t, lr, beta1, beta2);
  for (int64_t base = 0; base < count; base += static_cast<int64_t>(kAdamThreads) * kAdamUnroll) {
    float g[kAdamUnroll], m[kAdamUnroll], v[kAdamUnroll], p[kAdamUnroll];
#pragma unroll
    for (int k = 0; k < kAdamUnroll; ++k) {
      const int64_t i = base + threadIdx.x + static_cast<int64_t>(k) * kAdamThreads;
      const bool in = i < count;
      g[k] = in ? grad[i] : 0.0f;
      m[k] = in ? exp_avg[i] : 0.0f;
      v[k] = in ? exp_avg_sq[i] : 0.0f;
      p[k] = in ? params[i] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kAdamUnroll; ++k) {
      const int64_t i = base + threadIdx.x + static_cast<int64_t>(k) * kAdamThreads;
      if (i >= count) continue;
      adam_element(g[k], p[k], m[k], v[k], s, beta1, beta2, eps);
      exp_avg[i] = m[k];
      exp_avg_sq[i] = v[k];
      params[i] = p[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = t;
}

// Waits on an mbarrier that nothing arrives at; the bounded wait gives up after limit_ns,
// records FHB_STATUS_SELFTEST and returns. Exercises the timeout path without a fault.
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, unsigned int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t start = global_timer_ns();
  bool done = false;
  while (!done) {
    done = mbar_try_wait(&bar, 0);
    if (!done && global_timer_ns() - start > limit_ns) break;
  }
  if (!done && threadIdx.x == 0) report_status(status, FHB_STATUS_SELFTEST);
}

// out[i] = tanh_fast(x[i]) (fast != 0) or tanhf(x[i]): lets the tests bound tanh_fast
// against CUDA's tanhf on the device.
__global__ void debug_tanh_kernel(const float* __restrict__ x, float* __restrict__ out,
                                  int64_t n, int fast) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = fast ? tanh_fast(x[i]) : tanhf(x[i]);
}

}  // namespace

cudaError_t launch_debug_tanh(const float* x, float* out, int64_t n, int fast,
                              cudaStream_t stream) {
  const int64_t blocks = (n + 255) / 256;
  debug_tanh_kernel<<<static_cast<int>(blocks < 1024 ? blocks : 1024), 256, 0, stream>>>(x, out, n,
                                                                                        fast);
  return cudaGetLastError();
}

cudaError_t launch_adam(float* params, const float* grad, float* exp_avg, float* exp_avg_sq,
                        int64_t count, int64_t* step, float lr, float beta1, float beta2,
                        float eps, cudaStream_t stream) {
  adam_kernel<<<1, kAdamThreads, 0, stream>>>(params, grad, exp_avg, exp_avg_sq, count, step,
                                              lr, beta1, beta2, eps);
  return cudaGetLastError();
}

cudaError_t launch_bounded_wait_selftest(uint64_t limit_ns, unsigned int* status,
                                         cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, status);
  return cudaGetLastError();
}

}  // namespace fhb
