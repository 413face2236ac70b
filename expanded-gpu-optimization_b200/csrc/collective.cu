// The training step's tail in one kernel: the fixed-order sum of the backward's partial
// rows, the sum over data-parallel ranks through NVLink peer memory, and Adam.
//
// The reference trains on one GPU (autograd + torch.optim.Adam, reference
// benchmarks/benchmark_training.py:51-56), so this exchange is new. A data-parallel step
// would otherwise be three launches after the gradient kernel -- row reduction, an NCCL
// all-reduce of 12,738 floats, Adam -- each a full launch gap for ~51 KB of work. Here one CTA
// owns one block of 32 columns (399 CTAs, all resident at once) and, for epoch e = epoch + 1:
//   1. sums its columns over the partial rows in a fixed order (column_group_sum);
//   2. world > 1: stores the 32 sums into row `rank` of slot e % 2 of EVERY rank's exchange
//      buffer (plain stores over NVLink into CUDA IPC mappings), then, after a system-scope
//      fence, raises flags[block][rank] = e in every rank's buffer;
//   3. waits, bounded by wait_limit_ns, until flags[block][q] has reached e for every q in its
//      own buffer, and sums the rows q = 0, 1, ... of its own slot in that order, so every rank
//      gets bitwise the same totals;
//   4. applies Adam to its columns and writes the loss;
// and the last CTA to finish advances the step counter and the epoch.
// Reuse of a slot needs no second barrier: rank r writes slot e % 2 of rank q again at epoch
// e + 2, which it reaches only after seeing rank q's flag for e + 1, and rank q raises that
// flag only after its epoch-e reads of the block are done. Flags are compared as
// (int32)(flag - e) >= 0 because a fast peer may already have published e + 1.
// Peer memory is touched only by plain stores (no loads, no multicast, no TMA, no library
// kernel). A wait that gives up sets FHB_STATUS_PEER_TIMEOUT; that CTA leaves its parameters
// unchanged and the step counters still advance, so the host sees the error on its next
// status read rather than a hung GPU.
#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kUpdateThreads = kUpdateCols * kUpdateGroups;

__device__ __forceinline__ void store_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* exchange_flag(float* buffer, int block, int source) {
  return reinterpret_cast<uint32_t*>(buffer) + kExchangeFlagOffset + block * kMaxRanks + source;
}

__global__ void __launch_bounds__(kUpdateThreads)
    step_update_kernel(const float* __restrict__ partials, int rows, ExchangeState* state,
                       int world, int rank, uint64_t wait_limit_ns, AdamArgs adam,
                       float* __restrict__ grad_out, float* __restrict__ loss_out,
                       unsigned int* status) {
  __shared__ float sums[kUpdateGroups][kUpdateCols];
  __shared__ int gave_up;
  const int cx = threadIdx.x % kUpdateCols, grp = threadIdx.x / kUpdateCols;
  const int block = blockIdx.x;
  const int col = block * kUpdateCols + cx;
  const bool live = col <= kLossColumn;
  // Read before this CTA counts itself done, so before the last CTA advances them.
  const int64_t t = *adam.step + 1;
  const uint32_t e = state->epoch + 1u;

  sums[grp][cx] = live ? column_group_sum(partials, rows, col, grp) : 0.0f;
  if (threadIdx.x == 0) gave_up = 0;
  __syncthreads();
  float total = 0.0f;
  if (grp == 0) {
    total = sums[0][cx];
#pragma unroll
    for (int k = 1; k < kUpdateGroups; ++k) total += sums[k][cx];
  }

  if (world > 1) {
    const size_t slot = (e & 1u) * kMaxRanks;
    if (grp == 0 && live) {
      for (int q = 0; q < world; ++q) state->peers[q][(slot + rank) * kRowStride + col] = total;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int q = 0; q < world; ++q) store_release_sys(exchange_flag(state->peers[q], block, rank), e);
    }
    if (threadIdx.x < world) {
      const uint32_t* flag = exchange_flag(state->peers[rank], block, threadIdx.x);
      const uint64_t start = global_timer_ns();
      while (static_cast<int32_t>(load_acquire_sys(flag) - e) < 0) {
        if (global_timer_ns() - start > wait_limit_ns) {
          report_status(status, FHB_STATUS_PEER_TIMEOUT);
          gave_up = 1;
          break;
        }
      }
    }
    __syncthreads();
    if (grp == 0 && live && !gave_up) {
      const float* own = state->peers[rank] + slot * kRowStride + col;
      total = __ldcg(own);
      for (int q = 1; q < world; ++q) total += __ldcg(own + static_cast<size_t>(q) * kRowStride);
    }
  }

  if (grp == 0 && live && !gave_up) {
    if (grad_out != nullptr) grad_out[col] = total;
    if (col == kLossColumn) {
      if (loss_out != nullptr) *loss_out = total;
    } else {
      const AdamScalars s = adam_scalars(t, adam.lr, adam.beta1, adam.beta2);
      float p = adam.params[col], m = adam.exp_avg[col], v = adam.exp_avg_sq[col];
      adam_element(total, p, m, v, s, adam.beta1, adam.beta2, adam.eps);
      adam.exp_avg[col] = m;
      adam.exp_avg_sq[col] = v;
      adam.params[col] = p;
    }
  }

  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&state->done, 1u) == gridDim.x - 1) {
      *adam.step = t;
      state->epoch = e;
      state->done = 0;
    }
  }
}

}  // namespace

cudaError_t launch_step_update(const float* partials, int rows, ExchangeState* state, int world,
                               int rank, uint64_t wait_limit_ns, const AdamArgs& adam,
                               float* grad_out, float* loss_out, unsigned int* status,
                               cudaStream_t stream) {
  step_update_kernel<<<kUpdateBlocks, kUpdateThreads, 0, stream>>>(
      partials, rows, state, world, rank, wait_limit_ns, adam, grad_out, loss_out, status);
  return cudaGetLastError();
}

}  // namespace fhb
