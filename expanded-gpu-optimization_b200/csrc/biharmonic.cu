// FP32 CUDA-core forward of the biharmonic (u, Laplacian u, Laplacian of the Laplacian u) of
// the fixed 2->64x4->1 tanh MLP. The reference has no kernel for it; its README names the
// biharmonic as the next operator to test its kernel design on, and its own tool for it is
// nested autograd (src/fused_hoad/autodiff.py:39-41 applied twice).
//
// The jet: per neuron nine components [v, g_x, g_y, H_xx, H_xy, H_yy, T_x, T_y, B] --
// value, gradient, Hessian, T = grad(Laplacian), B = biharmonic -- of each pre-activation.
// A linear layer maps all nine linearly (the bias only the value), so each hidden layer is a
// 64x64 GEMM over 9 components (2.25x the Laplacian's 4). tanh maps them by the chain rule
// with d1..d4 its first four derivatives at z (d1 = 1 - a^2, d2 = -2 a d1,
// d3 = -2 d1 (1 - 3a^2), d4 = 8 a d1 (2 - 3a^2), a = tanh z):
//   H'_ij = d2 g_i g_j + d1 H_ij,
//   T'_k  = (d3 |g|^2 + d2 tr H) g_k + 2 d2 (H g)_k + d1 T_k,
//   B'    = d4 |g|^4 + d3 (2 tr H |g|^2 + 4 g.H.g) + d2 (2 |H|_F^2 + 4 g.T + (tr H)^2) + d1 B.
// Layer 0 starts from the input jet of (x, y): g = the row of W0 and H = T = B = 0.
//
// Layout (the FP32 Laplacian kernel's design, forward_fp32.cu): persistent grid, one CTA per
// SM with two independent 256-thread tile groups; the parameter buffer staged once per CTA
// by one bulk copy; a tile is 32 points, warp w of a group owns neurons 8w..8w+7 and lane l
// point l, so a layer is a register-tiled GEMM with 9 x 8 accumulators per thread, weights
// read as broadcast float2 and the jet as [component][neuron][point] in shared memory (72 KB
// per group); the last hidden layer folds in the output layer with a fixed-order sum of the
// 8 warps' partials. Bound: FP32 FMA issue, ~2.25x the Laplacian kernel's FLOPs per point;
// the GEMM's fmas run as packed pairs over the components of one neuron (fma.rn.f32x2), with
// the weights read two K at a time (float2) to leave the registers for them.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kComps = 9;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kNeuronsPerWarp = kWidth / kWarps;  // 8
constexpr int kTile = 32;                         // one point per lane
constexpr int kPlane = kWidth * kTile;            // one component, [neuron][point]
constexpr int kJetFloats = kComps * kPlane;
constexpr int kRedFloats = 3 * kWarps * kTile;    // per-warp partials of u, lap, bilap
constexpr int kGroups = 2;
constexpr int kBlock = kGroups * kThreads;
constexpr size_t kSmem =
    static_cast<size_t>(kParamSmemFloats + kGroups * (kJetFloats + kRedFloats)) * 4 + 16;
static_assert(kSmem <= 227 * 1024, "shared memory");

__device__ __forceinline__ void group_sync(int group) {
  asm volatile("bar.sync %0, 256;" ::"r"(1 + group) : "memory");
}

// The tanh map of one neuron's nine components, in place (the formulas above).
__device__ __forceinline__ void tanh_biharmonic(float (&c)[kComps]) {
  const float gx = c[1], gy = c[2], hxx = c[3], hxy = c[4], hyy = c[5];
  const float a = tanhf(c[0]);
  const float a2 = a * a;
  const float d1 = fmaf(-a, a, 1.0f);
  const float d2 = -2.0f * a * d1;
  const float d3 = -2.0f * d1 * fmaf(-3.0f, a2, 1.0f);
  const float d4 = 8.0f * a * d1 * fmaf(-3.0f, a2, 2.0f);
  const float g2 = fmaf(gx, gx, gy * gy);
  const float tr = hxx + hyy;
  const float hgx = fmaf(hxx, gx, hxy * gy);
  const float hgy = fmaf(hxy, gx, hyy * gy);
  const float ghg = fmaf(gx, hgx, gy * hgy);
  const float hf2 = fmaf(hxx, hxx, fmaf(2.0f * hxy, hxy, hyy * hyy));
  const float gt = fmaf(gx, c[6], gy * c[7]);
  const float kt = fmaf(d3, g2, d2 * tr);
  const float b = fmaf(d4 * g2, g2,
                       fmaf(d3, fmaf(2.0f * tr, g2, 4.0f * ghg),
                            fmaf(d2, fmaf(2.0f, hf2, fmaf(4.0f, gt, tr * tr)), d1 * c[8])));
  c[0] = a;
  c[1] = d1 * gx;
  c[2] = d1 * gy;
  c[3] = fmaf(d2 * gx, gx, d1 * hxx);
  c[4] = fmaf(d2 * gx, gy, d1 * hxy);
  c[5] = fmaf(d2 * gy, gy, d1 * hyy);
  c[6] = fmaf(kt, gx, fmaf(2.0f * d2, hgx, d1 * c[6]));
  c[7] = fmaf(kt, gy, fmaf(2.0f * d2, hgy, d1 * c[7]));
  c[8] = b;
}

__global__ void __launch_bounds__(kBlock, 1)
    forward_biharmonic_kernel(const float* __restrict__ coords, const float* __restrict__ params,
                              float* __restrict__ u_out, float* __restrict__ lap_out,
                              float* __restrict__ bilap_out, int64_t n, int64_t tiles,
                              int params_aligned, unsigned int* status) {
  extern __shared__ __align__(16) float smem[];
  float* sp = smem;  // staged parameters, ABI layout
  uint64_t* bar =
      reinterpret_cast<uint64_t*>(smem + kParamSmemFloats + kGroups * (kJetFloats + kRedFloats));
  if (!stage_parameters(sp, params, bar, params_aligned != 0, status)) return;

  const int group = threadIdx.x / kThreads;
  const int gt = threadIdx.x % kThreads;
  float* jet = smem + kParamSmemFloats + group * (kJetFloats + kRedFloats);
  float* red = jet + kJetFloats;  // [3][kWarps][kTile]
  const int warp = gt >> 5;
  const int lane = gt & 31;
  const int o0 = warp * kNeuronsPerWarp;

  for (int64_t tile = blockIdx.x + static_cast<int64_t>(group) * gridDim.x; tile < tiles;
       tile += static_cast<int64_t>(gridDim.x) * kGroups) {
    const int64_t p = tile * kTile + lane;
    const bool in = p < n;
    const float x0 = in ? coords[2 * p] : 0.0f;
    const float x1 = in ? coords[2 * p + 1] : 0.0f;

    // Layer 0: z = W0 x + b0 with g = (W0[o][0], W0[o][1]) and H = T = B = 0.
#pragma unroll
    for (int k = 0; k < kNeuronsPerWarp; ++k) {
      const int o = o0 + k;
      const float w0 = sp[2 * o], w1 = sp[2 * o + 1];
      float c[kComps] = {fmaf(w0, x0, fmaf(w1, x1, sp[kB0 + o])), w0, w1, 0.0f, 0.0f,
                         0.0f, 0.0f, 0.0f, 0.0f};
      tanh_biharmonic(c);
      float* dst = jet + o * kTile + lane;
#pragma unroll
      for (int m = 0; m < kComps; ++m) dst[m * kPlane] = c[m];
    }

#pragma unroll 1
    for (int layer = 0; layer < kHiddenGemms; ++layer) {
      const float* W = sp + kHiddenBase + layer * kHiddenStride;  // [out][in]
      const float* bias = W + kWidth * kWidth;
      group_sync(group);  // the input jet of this layer is complete

      float acc[kComps][kNeuronsPerWarp];
#pragma unroll
      for (int k = 0; k < kNeuronsPerWarp; ++k) {
        acc[0][k] = bias[o0 + k];
#pragma unroll
        for (int m = 1; m < kComps; ++m) acc[m][k] = 0.0f;
      }
#pragma unroll 1
      for (int i = 0; i < kWidth; i += 2) {
        float2 w[kNeuronsPerWarp];
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k)
          w[k] = *reinterpret_cast<const float2*>(W + (o0 + k) * kWidth + i);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float h[kComps];
          const float* src = jet + (i + j) * kTile + lane;
#pragma unroll
          for (int m = 0; m < kComps; ++m) h[m] = src[m * kPlane];
          // component pairs (m, m + 1) of one neuron in packed fmas (fma.rn.f32x2, each lane
          // rounded as fmaf: bitwise the scalar loop); the ninth component alone
#pragma unroll
          for (int k = 0; k < kNeuronsPerWarp; ++k) {
            const float wk = j == 0 ? w[k].x : w[k].y;
#pragma unroll
            for (int m = 0; m + 1 < kComps; m += 2)
              fma2(acc[m][k], acc[m + 1][k], wk, wk, h[m], h[m + 1]);
            acc[kComps - 1][k] = fmaf(wk, h[kComps - 1], acc[kComps - 1][k]);
          }
        }
      }
      group_sync(group);  // every read of this layer's input jet is done

      if (layer + 1 < kHiddenGemms) {
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k) {
          float c[kComps];
#pragma unroll
          for (int m = 0; m < kComps; ++m) c[m] = acc[m][k];
          tanh_biharmonic(c);
          float* dst = jet + (o0 + k) * kTile + lane;
#pragma unroll
          for (int m = 0; m < kComps; ++m) dst[m * kPlane] = c[m];
        }
      } else {
        // Output layer folded in: u = w.v + b, lap = w.(H_xx + H_yy), bilap = w.B.
        float pu = 0.0f, pl = 0.0f, pb = 0.0f;
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k) {
          float c[kComps];
#pragma unroll
          for (int m = 0; m < kComps; ++m) c[m] = acc[m][k];
          tanh_biharmonic(c);
          const float wo = sp[kOutBase + o0 + k];
          pu = fmaf(wo, c[0], pu);
          pl = fmaf(wo, c[3] + c[5], pl);
          pb = fmaf(wo, c[8], pb);
        }
        red[warp * kTile + lane] = pu;
        red[(kWarps + warp) * kTile + lane] = pl;
        red[(2 * kWarps + warp) * kTile + lane] = pb;
      }
    }
    group_sync(group);  // partial sums complete

    if (gt < kTile) {
      const int64_t q = tile * kTile + gt;
      if (q < n) {
        float uu = 0.0f, ll = 0.0f, bb = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          uu += red[w * kTile + gt];
          ll += red[(kWarps + w) * kTile + gt];
          bb += red[(2 * kWarps + w) * kTile + gt];
        }
        u_out[q] = uu + sp[kOutBase + kWidth];
        lap_out[q] = ll;
        bilap_out[q] = bb;
      }
    }
  }
}

}  // namespace

cudaError_t prepare_biharmonic() {
  return cudaFuncSetAttribute(forward_biharmonic_kernel,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSmem));
}

cudaError_t launch_forward_biharmonic(const float* coords, const float* params, float* u,
                                      float* lap, float* bilap, int64_t n,
                                      const DeviceInfo& dev, cudaStream_t stream) {
  const int64_t tiles = (n + kTile - 1) / kTile;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sms));
  const int params_aligned = (reinterpret_cast<uintptr_t>(params) % 16) == 0;
  forward_biharmonic_kernel<<<grid, kBlock, kSmem, stream>>>(
      coords, params, u, lap, bilap, n, tiles, params_aligned, dev.status);
  return cudaGetLastError();
}

}  // namespace fhb
