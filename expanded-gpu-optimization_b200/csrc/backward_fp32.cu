// FP32 CUDA-core adjoint-jet backward (all backward versions) and the fused Poisson step.
//
// Math: the reverse pass through the forward-Laplacian jet of the reference backward
// (csrc/fused_backward.cu:15-33 for the adjoint formulas, :208-233 output seed, :262-321
// weight gradient and input adjoint, :324-359 layer 0). Design for sm_100a:
//   * persistent grid, one 256-thread CTA per SM, 32-point tiles; the parameter buffer is
//     staged into shared memory once per CTA by one bulk (TMA) copy;
//   * the forward is recomputed per tile and its pre-activation jets z1, z2 stay in the
//     registers of the thread that produced them (warp w -> neurons 8w..8w+7, lane ->
//     point), because the same thread later applies the tanh adjoint at the same
//     (neuron, point). z3 is consumed as soon as it is produced and z0 is rebuilt from x.
//     Nothing is spilled to a global scratch area (the reference writes 128 KB per CTA);
//   * per layer: tanh adjoint in registers -> zbar to shared memory -> dW += zbar h^T
//     (each thread owns 16 entries of each of the three 64x64 dW blocks in registers, for
//     the whole persistent loop) and hbar = W^T zbar (register-tiled, weights broadcast);
//   * small gradients (biases, W0, w_out, b_out) are reduced over the tile's points with
//     warp shuffles and accumulated in shared memory by a single writer per entry;
//   * each CTA writes one partial-gradient row; reduce_rows_kernel sums the rows in a
//     fixed order. No atomics anywhere, so gradients are bitwise reproducible for a given
//     grid (grid = min(tiles, SMs)).
// The fused Poisson step (poisson = true) forms dL/dlap = 2 (lap - f) / n_total in the
// tile from the recomputed forward, so a training step needs no separate forward launch.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kTile = 32;                 // points per tile (one per lane)
constexpr int kStride = kTile + 4;        // padded [neuron][point] row (16-byte aligned)
constexpr int kPlane = kWidth * kStride;  // one jet component
constexpr int kJet = 4 * kPlane;

// Small-gradient accumulators in shared memory.
constexpr int kSmallW0 = 0;                        // [64][2]
constexpr int kSmallBias = kSmallW0 + 2 * kWidth;  // [4][64], layers 0..3
constexpr int kSmallWout = kSmallBias + 4 * kWidth;
constexpr int kSmallBout = kSmallWout + kWidth;
constexpr int kSmallLoss = kSmallBout + 1;
constexpr int kSmallCount = 456;  // >= kSmallLoss + 1, multiple of 4

constexpr int kRedFloats = 2 * kWarps * kTile;
constexpr int kPointFloats = 4 * kTile;  // x0, x1, g_u, g_lap
constexpr size_t kSmem =
    (size_t)(kParamSmemFloats + 2 * kJet + kSmallCount + kRedFloats + kPointFloats) *
        sizeof(float) +
    16;

__device__ __forceinline__ float comp4(const float4& w, int j) {
  return j == 0 ? w.x : j == 1 ? w.y : j == 2 ? w.z : w.w;
}

// z[c][k] = sum_i W[o0+k][i] h[c][i][lane] (+ bias for the value component).
__device__ __forceinline__ void gemm_forward(const float* __restrict__ W,
                                             const float* __restrict__ h, int o0, int lane,
                                             float (&z)[4][8]) {
  const float* bias = W + kWidth * kWidth;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    z[0][k] = bias[o0 + k];
    z[1][k] = z[2][k] = z[3][k] = 0.0f;
  }
#pragma unroll 2
  for (int i = 0; i < kWidth; i += 4) {
    float4 w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = *reinterpret_cast<const float4*>(W + (o0 + k) * kWidth + i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float* src = h + (i + j) * kStride + lane;
      const float hv = src[0], hj0 = src[kPlane], hj1 = src[2 * kPlane], hl = src[3 * kPlane];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float wk = comp4(w[k], j);
        z[0][k] = fmaf(wk, hv, z[0][k]);
        z[1][k] = fmaf(wk, hj0, z[1][k]);
        z[2][k] = fmaf(wk, hj1, z[2][k]);
        z[3][k] = fmaf(wk, hl, z[3][k]);
      }
    }
  }
}

// hb[c][k] = sum_o W[o][i0+k] zbar[c][o][lane]  (input adjoint, i = i0 + k).
__device__ __forceinline__ void gemm_input_adjoint(const float* __restrict__ W,
                                                   const float* __restrict__ adj, int i0,
                                                   int lane, float (&hb)[4][8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) hb[0][k] = hb[1][k] = hb[2][k] = hb[3][k] = 0.0f;
#pragma unroll 4
  for (int o = 0; o < kWidth; ++o) {
    const float4 wa = *reinterpret_cast<const float4*>(W + o * kWidth + i0);
    const float4 wb = *reinterpret_cast<const float4*>(W + o * kWidth + i0 + 4);
    const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    const float* src = adj + o * kStride + lane;
    const float av = src[0], aj0 = src[kPlane], aj1 = src[2 * kPlane], al = src[3 * kPlane];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      hb[0][k] = fmaf(w[k], av, hb[0][k]);
      hb[1][k] = fmaf(w[k], aj0, hb[1][k]);
      hb[2][k] = fmaf(w[k], aj1, hb[2][k]);
      hb[3][k] = fmaf(w[k], al, hb[3][k]);
    }
  }
}

// dw[j][k] += sum_c sum_p zbar[c][ob+16j][p] * h[c][ib+16k][p].
__device__ __forceinline__ void gemm_weight_grad(const float* __restrict__ adj,
                                                 const float* __restrict__ h, int ob, int ib,
                                                 float (&dw)[4][4]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
#pragma unroll 2
    for (int p = 0; p < kTile; p += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        a[j] = *reinterpret_cast<const float4*>(adj + c * kPlane + (ob + 16 * j) * kStride + p);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        b[k] = *reinterpret_cast<const float4*>(h + c * kPlane + (ib + 16 * k) * kStride + p);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float s = dw[j][k];
          s = fmaf(a[j].x, b[k].x, s);
          s = fmaf(a[j].y, b[k].y, s);
          s = fmaf(a[j].z, b[k].z, s);
          s = fmaf(a[j].w, b[k].w, s);
          dw[j][k] = s;
        }
    }
  }
}

__device__ __forceinline__ void store_jet(float* buf, int o, int lane, float v, float j0,
                                          float j1, float l) {
  float* dst = buf + o * kStride + lane;
  dst[0] = v;
  dst[kPlane] = j0;
  dst[2 * kPlane] = j1;
  dst[3 * kPlane] = l;
}

template <bool kPoisson, class Act>
__global__ void __launch_bounds__(kThreads, 1)
    backward_fp32_kernel(const PointSets ps, const float* __restrict__ params,
                         const float* __restrict__ grad_u, const float* __restrict__ grad_lap,
                         float* __restrict__ grad_coords, float* __restrict__ lap_out,
                         float* __restrict__ partials, int64_t tiles, int params_aligned,
                         unsigned int* status) {
  extern __shared__ __align__(16) float smem[];
  float* sp = smem;
  float* hbuf = sp + kParamSmemFloats;  // forward jet h, [4][64][kStride]
  float* adj = hbuf + kJet;             // adjoint zbar, [4][64][kStride]
  float* small = adj + kJet;
  float* red = small + kSmallCount;     // [2][kWarps][kTile]
  float* pts = red + kRedFloats;        // x0[32] x1[32] gu[32] gl[32]
  uint64_t* bar = reinterpret_cast<uint64_t*>(pts + kPointFloats);

  for (int k = threadIdx.x; k < kSmallCount; k += kThreads) small[k] = 0.0f;
  if (!stage_parameters(sp, params, bar, params_aligned != 0, status)) return;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int o0 = warp * 8;       // elementwise mapping: neurons o0..o0+7 at point `lane`
  const int ob = tid >> 4;       // weight-gradient mapping: rows ob+16j, cols ib+16k
  const int ib = tid & 15;
  const float* W1 = sp + kHiddenBase;
  const float* W2 = W1 + kHiddenStride;
  const float* W3 = W2 + kHiddenStride;
  const float* wout = sp + kOutBase;

  float dw[3][4][4];
#pragma unroll
  for (int l = 0; l < 3; ++l)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) dw[l][j][k] = 0.0f;

  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const bool btile = tile >= ps.tiles;  // a tile of the boundary set (PINN step)
    const int64_t p = (btile ? tile - ps.tiles : tile) * kTile + lane;
    const bool active = p < (btile ? ps.nb : ps.n);
    if (tid < kTile) {
      load_point(ps, tile, kTile, tid, pts[tid], pts[kTile + tid]);
      if (!kPoisson) {
        pts[2 * kTile + tid] = (active && grad_u != nullptr) ? grad_u[p] : 0.0f;
        pts[3 * kTile + tid] = active ? grad_lap[p] : 0.0f;
      }
    }
    __syncthreads();
    const float x0 = pts[lane], x1 = pts[kTile + lane];

    // ---- forward recompute ----
    float zv0[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int o = o0 + k;
      const float w0 = sp[2 * o], w1 = sp[2 * o + 1];
      zv0[k] = fmaf(w0, x0, fmaf(w1, x1, sp[kB0 + o]));
      float v, j0, j1, l;
      Act::jet(zv0[k], w0, w1, 0.0f, v, j0, j1, l);
      store_jet(hbuf, o, lane, v, j0, j1, l);
    }
    __syncthreads();
    float z1[4][8], z2[4][8];
    gemm_forward(W1, hbuf, o0, lane, z1);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float v, j0, j1, l;
      Act::jet(z1[0][k], z1[1][k], z1[2][k], z1[3][k], v, j0, j1, l);
      store_jet(hbuf, o0 + k, lane, v, j0, j1, l);
    }
    __syncthreads();
    gemm_forward(W2, hbuf, o0, lane, z2);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float v, j0, j1, l;
      Act::jet(z2[0][k], z2[1][k], z2[2][k], z2[3][k], v, j0, j1, l);
      store_jet(hbuf, o0 + k, lane, v, j0, j1, l);
    }
    __syncthreads();  // hbuf = h2, kept until the layer-3 weight gradient
    {
      float z3[4][8];
      gemm_forward(W3, hbuf, o0, lane, z3);

      // ---- output layer: u = w.v + b, lap = w.L ----
      float h3v[8], h3l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float j0, j1;
        Act::jet(z3[0][k], z3[1][k], z3[2][k], z3[3][k], h3v[k], j0, j1, h3l[k]);
      }
      float gu, gl;
      if (kPoisson) {
        float part = 0.0f, partu = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          part = fmaf(wout[o0 + k], h3l[k], part);
          partu = fmaf(wout[o0 + k], h3v[k], partu);
        }
        red[warp * kTile + lane] = part;
        red[(kWarps + warp) * kTile + lane] = partu;
        __syncthreads();
        float term;  // this point's loss term
        if (!btile) {
          float lap = 0.0f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) lap += red[w * kTile + lane];
          // f = -2 pi^2 sin(pi x) sin(pi y)  (src/fused_hoad/problems/poisson.py:29-39); sinpif
          // needs no large-argument reduction (no local-memory path)
          const float pi = 3.14159265358979323846f;
          const float f = -2.0f * pi * pi * (sinpif(x0) * sinpif(x1));
          const float r = active ? lap - f : 0.0f;
          gu = 0.0f;
          gl = 2.0f * r * ps.inv_total;
          term = r * r * ps.inv_total;
          if (warp == 0 && active && lap_out != nullptr) lap_out[p] = lap;
        } else {
          // boundary term weight * u^2 / boundary_total (src/fused_hoad/training.py:90-92)
          float u = sp[kOutBase + kWidth];
#pragma unroll
          for (int w = 0; w < kWarps; ++w) u += red[(kWarps + w) * kTile + lane];
          u = active ? u : 0.0f;
          gu = 2.0f * ps.bweight * u * ps.inv_btotal;
          gl = 0.0f;
          term = ps.bweight * u * u * ps.inv_btotal;
        }
        if (warp == 0) {
          const float l2 = warp_sum(term);
          const float sg = btile ? warp_sum(gu) : 0.0f;  // b_out gradient (boundary term)
          if (lane == 0) {
            small[kSmallLoss] += l2;
            small[kSmallBout] += sg;
          }
        }
      } else {
        gu = pts[2 * kTile + lane];
        gl = pts[3 * kTile + lane];
        if (warp == 0) {
          const float s = warp_sum(gu);
          if (lane == 0) small[kSmallBout] += s;
        }
      }

      // seed the adjoint (vbar = g_u w, Jbar = 0, Lbar = g_lap w), then the layer-3 tanh
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int o = o0 + k;
        const float w = wout[o];
        const float dwo = warp_sum(fmaf(gu, h3v[k], gl * h3l[k]));
        float av = gu * w, aj0 = 0.0f, aj1 = 0.0f, al = gl * w;
        Act::adjoint(z3[0][k], z3[1][k], z3[2][k], z3[3][k], av, aj0, aj1, al);
        const float db = warp_sum(av);
        if (lane == 0) {
          small[kSmallWout + o] += dwo;
          small[kSmallBias + 3 * kWidth + o] += db;
        }
        store_jet(adj, o, lane, av, aj0, aj1, al);
      }
    }
    __syncthreads();  // adj = zbar3, hbuf = h2

    float hb[4][8];
    gemm_weight_grad(adj, hbuf, ob, ib, dw[2]);
    gemm_input_adjoint(W3, adj, o0, lane, hb);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int o = o0 + k;
      Act::adjoint(z2[0][k], z2[1][k], z2[2][k], z2[3][k], hb[0][k], hb[1][k], hb[2][k],
                       hb[3][k]);
      const float db = warp_sum(hb[0][k]);
      if (lane == 0) small[kSmallBias + 2 * kWidth + o] += db;
      store_jet(adj, o, lane, hb[0][k], hb[1][k], hb[2][k], hb[3][k]);
      float v, j0, j1, l;
      Act::jet(z1[0][k], z1[1][k], z1[2][k], z1[3][k], v, j0, j1, l);
      store_jet(hbuf, o, lane, v, j0, j1, l);
    }
    __syncthreads();  // adj = zbar2, hbuf = h1

    gemm_weight_grad(adj, hbuf, ob, ib, dw[1]);
    gemm_input_adjoint(W2, adj, o0, lane, hb);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int o = o0 + k;
      Act::adjoint(z1[0][k], z1[1][k], z1[2][k], z1[3][k], hb[0][k], hb[1][k], hb[2][k],
                       hb[3][k]);
      const float db = warp_sum(hb[0][k]);
      if (lane == 0) small[kSmallBias + 1 * kWidth + o] += db;
      store_jet(adj, o, lane, hb[0][k], hb[1][k], hb[2][k], hb[3][k]);
      const float w0 = sp[2 * o], w1 = sp[2 * o + 1];
      float v, j0, j1, l;
      Act::jet(zv0[k], w0, w1, 0.0f, v, j0, j1, l);
      store_jet(hbuf, o, lane, v, j0, j1, l);
    }
    __syncthreads();  // adj = zbar1, hbuf = h0

    gemm_weight_grad(adj, hbuf, ob, ib, dw[0]);
    gemm_input_adjoint(W1, adj, o0, lane, hb);

    // ---- layer 0: z_v = W0 x + b0, z_J = W0, z_L = 0 ----
    float gx0 = 0.0f, gx1 = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int o = o0 + k;
      const float w0 = sp[2 * o], w1 = sp[2 * o + 1];
      Act::adjoint(zv0[k], w0, w1, 0.0f, hb[0][k], hb[1][k], hb[2][k], hb[3][k]);
      const float zb = active ? hb[0][k] : 0.0f;
      const float db = warp_sum(zb);
      const float d0 = warp_sum(fmaf(zb, x0, active ? hb[1][k] : 0.0f));
      const float d1 = warp_sum(fmaf(zb, x1, active ? hb[2][k] : 0.0f));
      if (lane == 0) {
        small[kSmallBias + o] += db;
        small[kSmallW0 + 2 * o] += d0;
        small[kSmallW0 + 2 * o + 1] += d1;
      }
      gx0 = fmaf(w0, zb, gx0);
      gx1 = fmaf(w1, zb, gx1);
    }
    red[warp * kTile + lane] = gx0;
    red[(kWarps + warp) * kTile + lane] = gx1;
    __syncthreads();  // also: every read of adj/hbuf for this tile is done
    if (warp == 0 && active && !btile && grad_coords != nullptr) {
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        s0 += red[w * kTile + lane];
        s1 += red[(kWarps + w) * kTile + lane];
      }
      grad_coords[2 * p] = s0;
      grad_coords[2 * p + 1] = s1;
    }
  }
  __syncthreads();

  // ---- this CTA's partial-gradient row, in the packed ABI layout ----
  float* row = partials + static_cast<int64_t>(blockIdx.x) * kRowStride;
  for (int k = tid; k < 2 * kWidth; k += kThreads) row[k] = small[kSmallW0 + k];
  if (tid < kWidth) {
    row[kB0 + tid] = small[kSmallBias + tid];
#pragma unroll
    for (int l = 1; l < 4; ++l)
      row[kHiddenBase + (l - 1) * kHiddenStride + kWidth * kWidth + tid] =
          small[kSmallBias + l * kWidth + tid];
    row[kOutBase + tid] = small[kSmallWout + tid];
  }
  if (tid == 0) {
    row[kOutBase + kWidth] = small[kSmallBout];
    row[kLossColumn] = small[kSmallLoss];
  }
#pragma unroll
  for (int l = 0; l < 3; ++l) {
    float* wrow = row + kHiddenBase + l * kHiddenStride;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) wrow[(ob + 16 * j) * kWidth + ib + 16 * k] = dw[l][j][k];
  }
}

// out[col] = sum over the partial rows of partials[r][col] in a fixed order: a block takes 32
// columns; its 8 row groups (rows g, g+8, g+16, ...) are summed in row order by 8 threads
// of a column (column_group_sum), then the 8 group sums are added in group order.
constexpr int kReduceCols = kUpdateCols, kReduceGroups = kUpdateGroups;
__global__ void __launch_bounds__(kReduceCols * kReduceGroups)
    reduce_rows_kernel(const float* __restrict__ partials, int rows,
                       float* __restrict__ grad_params, float* __restrict__ loss) {
  __shared__ float sums[kReduceGroups][kReduceCols];
  const int cx = threadIdx.x % kReduceCols, grp = threadIdx.x / kReduceCols;
  const int col = blockIdx.x * kReduceCols + cx;
  const float acc = col <= kLossColumn ? column_group_sum(partials, rows, col, grp) : 0.0f;
  sums[grp][cx] = acc;
  __syncthreads();
  if (grp != 0 || col > kLossColumn) return;
  float total = sums[0][cx];
#pragma unroll
  for (int k = 1; k < kReduceGroups; ++k) total += sums[k][cx];
  if (col == kLossColumn) {
    if (loss != nullptr) *loss = total;
  } else {
    grad_params[col] = total;
  }
}

template <bool kPoisson, class Act>
cudaError_t set_attributes() {
  return cudaFuncSetAttribute(backward_fp32_kernel<kPoisson, Act>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSmem));
}

template <class Act>
void launch_act(const PointSets& ps, const float* params, const float* grad_u,
                const float* grad_lap, float* grad_coords, float* lap_out, float* partials,
                bool poisson, int grid, int64_t tiles, int aligned, const DeviceInfo& dev,
                cudaStream_t stream) {
  if (poisson) {
    backward_fp32_kernel<true, Act><<<grid, kThreads, kSmem, stream>>>(
        ps, params, nullptr, nullptr, grad_coords, lap_out, partials, tiles, aligned,
        dev.status);
  } else {
    backward_fp32_kernel<false, Act><<<grid, kThreads, kSmem, stream>>>(
        ps, params, grad_u, grad_lap, grad_coords, nullptr, partials, tiles, aligned,
        dev.status);
  }
}

}  // namespace

cudaError_t prepare_backward_fp32() {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {set_attributes<false, TanhAct>(), set_attributes<true, TanhAct>(),
                        set_attributes<false, SiluAct>(), set_attributes<true, SiluAct>()})
    if (e == cudaSuccess) e = r;
  return e;
}

int backward_grid(int64_t n, int64_t nb, const DeviceInfo& dev) {
  const int64_t tiles = (n + kTile - 1) / kTile + (nb + kTile - 1) / kTile;
  return static_cast<int>(std::min<int64_t>(tiles, dev.sms));
}

cudaError_t launch_backward_fp32(const PointSets& points, const float* params,
                                 const float* grad_u, const float* grad_lap,
                                 float* grad_coords, float* lap_out, float* partials,
                                 bool poisson, int activation, const DeviceInfo& dev,
                                 cudaStream_t stream) {
  PointSets ps = points;
  ps.tiles = (ps.n + kTile - 1) / kTile;
  const int64_t tiles = ps.tiles + (ps.nb + kTile - 1) / kTile;
  const int grid = backward_grid(ps.n, ps.nb, dev);
  const int aligned = (reinterpret_cast<uintptr_t>(params) % 16) == 0;
  if (activation == FHB_ACTIVATION_SILU)
    launch_act<SiluAct>(ps, params, grad_u, grad_lap, grad_coords, lap_out, partials, poisson,
                        grid, tiles, aligned, dev, stream);
  else
    launch_act<TanhAct>(ps, params, grad_u, grad_lap, grad_coords, lap_out, partials, poisson,
                        grid, tiles, aligned, dev, stream);
  return cudaGetLastError();
}

cudaError_t launch_reduce_rows(const float* partials, int rows, float* grad_params,
                               float* loss, cudaStream_t stream) {
  const int cols = kLossColumn + 1;
  reduce_rows_kernel<<<(cols + kReduceCols - 1) / kReduceCols, kReduceCols * kReduceGroups, 0,
                       stream>>>(partials, rows, grad_params, loss);
  return cudaGetLastError();
}

}  // namespace fhb
