// FP32 CUDA-core forward-Laplacian kernel (forward versions 0, 1, 2).
//
// Same math as the reference's fwd v0-v2 (csrc/fused_residual.cu:61-279): the jet
// (value, d/dx, d/dy, Laplacian) of every hidden neuron is carried through the 2->64x4->1
// MLP, with tanh (the reference kernels' activation) or SiLU (the other activation of the
// reference's PyTorch forward-Laplacian backend) as the Act template parameter. Design for
// sm_100a:
//   * persistent grid, one CTA per SM; the whole 51 KB parameter buffer is staged into
//     shared memory ONCE per CTA by one bulk (TMA) copy, not once per tile. A CTA holds two
//     independent 256-thread tile groups (32- and 64-point tiles; one group for 128-point
//     tiles, whose 128 accumulators per thread leave no registers for a second), each with
//     its own jet buffer and named barrier, taking the CTA's tiles in turn: 4 warps per
//     scheduler instead of 2 hide the FMA and shared-memory latencies that bounded one group
//     (64-point tiles 174 -> 166 us at 64K points, 32-point tiles 190 -> 169 us);
//   * a tile holds 32*PPL points; warp w of a group owns neurons 8w..8w+7, lane l owns points
//     l*PPL..l*PPL+PPL-1, so every 64x64 layer is a register-tiled GEMM with
//     4 comps x 8 neurons x PPL points = 32*PPL accumulators per thread. Weights are read
//     row-major as float4 (broadcast within a warp: 8 LDS.128 per 4 inputs), jet columns
//     as float2/float4;
//   * the tanh-jet update is applied in registers straight from the accumulators, and the
//     last hidden layer folds the output layer in (no fourth jet write); the 8 per-warp
//     partial sums of u and lap are combined in a fixed order (deterministic).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kNeuronsPerWarp = kWidth / kWarps;  // 8
static_assert(kNeuronsPerWarp == 8, "mapping assumes 8 neurons per warp");

template <int PPL>
struct Cfg {
  static constexpr int kTile = 32 * PPL;
  static constexpr int kPlane = kWidth * kTile;  // one jet component, [neuron][point]
  static constexpr int kJetFloats = 4 * kPlane;
  static constexpr int kRedFloats = 2 * kWarps * kTile;
  // Independent 8-warp tile groups per CTA sharing the staged parameters: two where the
  // accumulators leave room for 512 threads (<= 128 registers), one for 128-point tiles.
  static constexpr int kGroups = PPL == 4 ? 1 : 2;
  static constexpr int kBlock = kGroups * kThreads;
  static constexpr size_t kSmem =
      (size_t)(kParamSmemFloats + kGroups * (kJetFloats + kRedFloats)) * sizeof(float) + 16;
};

// Barrier over the 256 threads of one tile group (ids 1, 2; 0 is __syncthreads).
template <int kGroups>
__device__ __forceinline__ void group_sync(int group) {
  if constexpr (kGroups == 1) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, 256;" ::"r"(1 + group) : "memory");
  }
}

template <int PPL>
__device__ __forceinline__ void ld_pts(const float* p, float (&v)[PPL]) {
  if constexpr (PPL == 1) {
    v[0] = *p;
  } else if constexpr (PPL == 2) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x;
    v[1] = t.y;
  } else {
    static_assert(PPL == 4, "PPL must be 1, 2 or 4");
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  }
}

template <int PPL>
__device__ __forceinline__ void st_pts(float* p, const float (&v)[PPL]) {
  if constexpr (PPL == 1) {
    *p = v[0];
  } else if constexpr (PPL == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

__device__ __forceinline__ float lane_of(const float4& w, int j) {
  return j == 0 ? w.x : j == 1 ? w.y : j == 2 ? w.z : w.w;
}

template <int PPL, class Act>
__global__ void __launch_bounds__(Cfg<PPL>::kBlock, 1)
    forward_fp32_kernel(const float* __restrict__ coords, const float* __restrict__ params,
                        float* __restrict__ u_out, float* __restrict__ lap_out, int64_t n,
                        int64_t tiles, int params_aligned, int coords_aligned,
                        unsigned int* status) {
  using C = Cfg<PPL>;
  extern __shared__ __align__(16) float smem[];
  float* sp = smem;                       // staged parameters, ABI layout
  uint64_t* bar = reinterpret_cast<uint64_t*>(
      smem + kParamSmemFloats + C::kGroups * (C::kJetFloats + C::kRedFloats));
  if (!stage_parameters(sp, params, bar, params_aligned != 0, status)) return;

  const int group = threadIdx.x / kThreads;
  const int gt = threadIdx.x % kThreads;  // thread within the group
  float* jet = smem + kParamSmemFloats + group * (C::kJetFloats + C::kRedFloats);  // [4][64][kTile]
  float* red = jet + C::kJetFloats;       // [2][kWarps][kTile]
  const int warp = gt >> 5;
  const int lane = gt & 31;
  const int o0 = warp * kNeuronsPerWarp;
  const int col = lane * PPL;

  // The CTA's tiles (blockIdx.x + k gridDim.x) alternate between its groups, so the SM's
  // share stays balanced and an odd last tile runs with the SM to itself.
  for (int64_t tile = blockIdx.x + static_cast<int64_t>(group) * gridDim.x; tile < tiles;
       tile += static_cast<int64_t>(gridDim.x) * C::kGroups) {
    const int64_t first = tile * C::kTile + col;
    float x0[PPL], x1[PPL];
    if (coords_aligned && PPL >= 2 && first + PPL <= n) {
      const float4* src = reinterpret_cast<const float4*>(coords + 2 * first);
#pragma unroll
      for (int h = 0; h < PPL / 2; ++h) {
        const float4 t = src[h];
        x0[2 * h] = t.x;
        x1[2 * h] = t.y;
        x0[2 * h + 1] = t.z;
        x1[2 * h + 1] = t.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < PPL; ++q) {
        const bool in = first + q < n;
        x0[q] = in ? coords[2 * (first + q)] : 0.0f;
        x1[q] = in ? coords[2 * (first + q) + 1] : 0.0f;
      }
    }

    // Layer 0: input jet (x, I, 0) gives z_J = W0 columns and z_L = 0.
#pragma unroll
    for (int k = 0; k < kNeuronsPerWarp; ++k) {
      const int o = o0 + k;
      const float w0 = sp[2 * o], w1 = sp[2 * o + 1], b = sp[kB0 + o];
      float hv[PPL], hj0[PPL], hj1[PPL], hl[PPL];
#pragma unroll
      for (int q = 0; q < PPL; ++q)
        Act::jet(fmaf(w0, x0[q], fmaf(w1, x1[q], b)), w0, w1, 0.0f, hv[q], hj0[q], hj1[q],
                 hl[q]);
      float* dst = jet + o * C::kTile + col;
      st_pts<PPL>(dst, hv);
      st_pts<PPL>(dst + C::kPlane, hj0);
      st_pts<PPL>(dst + 2 * C::kPlane, hj1);
      st_pts<PPL>(dst + 3 * C::kPlane, hl);
    }

#pragma unroll 1
    for (int layer = 0; layer < kHiddenGemms; ++layer) {
      const float* W = sp + kHiddenBase + layer * kHiddenStride;  // [out][in]
      const float* bias = W + kWidth * kWidth;
      group_sync<C::kGroups>(group);  // the input jet of this layer is complete

      float acc[4][kNeuronsPerWarp][PPL];
#pragma unroll
      for (int k = 0; k < kNeuronsPerWarp; ++k) {
        const float b = bias[o0 + k];
#pragma unroll
        for (int q = 0; q < PPL; ++q) {
          acc[0][k][q] = b;
          acc[1][k][q] = 0.0f;
          acc[2][k][q] = 0.0f;
          acc[3][k][q] = 0.0f;
        }
      }
#pragma unroll 2
      for (int i = 0; i < kWidth; i += 4) {
        float4 w[kNeuronsPerWarp];
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k)
          w[k] = *reinterpret_cast<const float4*>(W + (o0 + k) * kWidth + i);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float h[4][PPL];
          const float* src = jet + (i + j) * C::kTile + col;
#pragma unroll
          for (int c = 0; c < 4; ++c) ld_pts<PPL>(src + c * C::kPlane, h[c]);
          // packed fmas: pairs of points, or pairs of neurons with one point per lane
          if constexpr (PPL % 2 == 0) {
#pragma unroll
            for (int k = 0; k < kNeuronsPerWarp; ++k) {
              const float wk = lane_of(w[k], j);
#pragma unroll
              for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int q = 0; q < PPL; q += 2)
                  fma2(acc[c][k][q], acc[c][k][q + 1], wk, wk, h[c][q], h[c][q + 1]);
            }
          } else {
#pragma unroll
            for (int k = 0; k < kNeuronsPerWarp; k += 2) {
              const float wa = lane_of(w[k], j), wb = lane_of(w[k + 1], j);
#pragma unroll
              for (int c = 0; c < 4; ++c)
                fma2(acc[c][k][0], acc[c][k + 1][0], wa, wb, h[c][0], h[c][0]);
            }
          }
        }
      }
      group_sync<C::kGroups>(group);  // every read of this layer's input jet is done

      if (layer + 1 < kHiddenGemms) {
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k) {
          float hv[PPL], hj0[PPL], hj1[PPL], hl[PPL];
#pragma unroll
          for (int q = 0; q < PPL; ++q)
            Act::jet(acc[0][k][q], acc[1][k][q], acc[2][k][q], acc[3][k][q], hv[q], hj0[q],
                     hj1[q], hl[q]);
          float* dst = jet + (o0 + k) * C::kTile + col;
          st_pts<PPL>(dst, hv);
          st_pts<PPL>(dst + C::kPlane, hj0);
          st_pts<PPL>(dst + 2 * C::kPlane, hj1);
          st_pts<PPL>(dst + 3 * C::kPlane, hl);
        }
      } else {
        // Output layer folded in: u = w.v + b, lap = w.L; per-warp partial sums.
        float pu[PPL], pl[PPL];
#pragma unroll
        for (int q = 0; q < PPL; ++q) pu[q] = pl[q] = 0.0f;
#pragma unroll
        for (int k = 0; k < kNeuronsPerWarp; ++k) {
          const float wo = sp[kOutBase + o0 + k];
#pragma unroll
          for (int q = 0; q < PPL; ++q) {
            float v, j0, j1, l;
            Act::jet(acc[0][k][q], acc[1][k][q], acc[2][k][q], acc[3][k][q], v, j0, j1, l);
            pu[q] = fmaf(wo, v, pu[q]);
            pl[q] = fmaf(wo, l, pl[q]);
          }
        }
        st_pts<PPL>(red + warp * C::kTile + col, pu);
        st_pts<PPL>(red + (kWarps + warp) * C::kTile + col, pl);
      }
    }
    group_sync<C::kGroups>(group);  // partial sums complete

    if (gt < C::kTile) {
      const int t = gt;
      const int64_t p = tile * C::kTile + t;
      if (p < n) {
        float uu = 0.0f, ll = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          uu += red[w * C::kTile + t];
          ll += red[(kWarps + w) * C::kTile + t];
        }
        u_out[p] = uu + sp[kOutBase + kWidth];
        lap_out[p] = ll;
      }
    }
  }
}

template <int PPL, class Act>
cudaError_t set_attributes() {
  return cudaFuncSetAttribute(forward_fp32_kernel<PPL, Act>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(Cfg<PPL>::kSmem));
}

template <int PPL, class Act>
cudaError_t launch(const float* coords, const float* params, float* u, float* lap, int64_t n,
                   const DeviceInfo& dev, cudaStream_t stream) {
  using C = Cfg<PPL>;
  const int64_t tiles = (n + C::kTile - 1) / C::kTile;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.sms));
  const int params_aligned = (reinterpret_cast<uintptr_t>(params) % 16) == 0;
  const int coords_aligned = (reinterpret_cast<uintptr_t>(coords) % 16) == 0;
  forward_fp32_kernel<PPL, Act><<<grid, C::kBlock, C::kSmem, stream>>>(
      coords, params, u, lap, n, tiles, params_aligned, coords_aligned, dev.status);
  return cudaGetLastError();
}

template <class Act>
cudaError_t launch_act(int tile, const float* coords, const float* params, float* u, float* lap,
                       int64_t n, const DeviceInfo& dev, cudaStream_t stream) {
  switch (tile) {
    case 0: return launch<1, Act>(coords, params, u, lap, n, dev, stream);
    case 1: return launch<4, Act>(coords, params, u, lap, n, dev, stream);
    default: return launch<2, Act>(coords, params, u, lap, n, dev, stream);
  }
}

}  // namespace

cudaError_t prepare_forward_fp32() {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {set_attributes<1, TanhAct>(), set_attributes<2, TanhAct>(),
                        set_attributes<4, TanhAct>(), set_attributes<1, SiluAct>(),
                        set_attributes<2, SiluAct>(), set_attributes<4, SiluAct>()})
    if (e == cudaSuccess) e = r;
  return e;
}

cudaError_t launch_forward_fp32(int tile, const float* coords, const float* params, float* u,
                                float* lap, int64_t n, int activation, const DeviceInfo& dev,
                                cudaStream_t stream) {
  return activation == FHB_ACTIVATION_SILU
             ? launch_act<SiluAct>(tile, coords, params, u, lap, n, dev, stream)
             : launch_act<TanhAct>(tile, coords, params, u, lap, n, dev, stream);
}

}  // namespace fhb
