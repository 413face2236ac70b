// The training step's tail in one kernel: the fixed-order sum of the backward's partial
// rows, the sum over data-parallel ranks through NVLink peer memory, and Adam.
//
// The reference trains on one GPU (autograd + torch.optim.Adam, reference
// benchmarks/benchmark_training.py:51-56), so this exchange is new. A data-parallel step
// would otherwise be three launches after the gradient kernel -- row reduction, an NCCL
// all-reduce of 12,738 floats, Adam -- for ~51 KB of work. Here one CTA owns a block of 32
// columns (399 CTAs, all resident at once) and one thread of it owns one column. For epoch
// e = epoch + 1 the column's thread:
//   1. sums the column over the partial rows in a fixed order (column_group_sum + the
//      groups in order);
//   2. world > 1: stores the 64-bit word (e << 32 | bits of the sum) into row `rank` of slot
//      e % 2 of EVERY rank's exchange buffer (plain stores over NVLink into the CUDA IPC
//      mappings), then reads the words of rows 0, 1, ... of its own buffer, each until its
//      high half is e (bounded by wait_limit_ns), and adds their low halves in rank order,
//      so every rank gets bitwise the same sum;
//   3. applies Adam to its parameter (or writes the loss).
// The last CTA to finish advances the step counter and the epoch.
//
// Why the words carry the epoch: an aligned 64-bit access is single-copy atomic, so a word
// whose epoch half reads e carries that epoch's value. No flag and no memory fence is needed
// between the data and its signal; a system-scope fence costs microseconds whenever stores
// to a peer are in flight, and a flag-per-block protocol needing one measured 15-30 us per
// step on two GPUs against about 7 us for this one.
// Why two slots suffice: rank r stores into slot e % 2 of rank q again at epoch e + 2, which
// its kernel starts only after its epoch e + 1 read of rank q's word for the same column;
// rank q stored that word in its epoch e + 1 kernel, which starts only after its epoch e
// kernel -- and with it the epoch e read of the slot -- has finished.
// Peer memory is touched only by plain 64-bit stores (no loads, no multicast, no TMA, no
// library kernel). A wait that gives up sets FHB_STATUS_PEER_TIMEOUT; that column keeps
// its parameter and moments and the counters still advance, so the host sees the error at
// its next status read instead of a hung GPU.
#include "common.cuh"
#include "kernels.cuh"

namespace fhb {
namespace {

constexpr int kUpdateThreads = kUpdateCols * kUpdateGroups;

__device__ __forceinline__ void store_word_sys(uint64_t* addr, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t load_word_sys(const uint64_t* addr) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

__global__ void __launch_bounds__(kUpdateThreads)
    step_update_kernel(const float* __restrict__ partials, int rows, ExchangeState* state,
                       int world, int rank, uint64_t wait_limit_ns, AdamArgs adam,
                       float* __restrict__ grad_out, float* __restrict__ loss_out,
                       unsigned int* status) {
  __shared__ float sums[kUpdateGroups][kUpdateCols];
  const int cx = threadIdx.x % kUpdateCols, grp = threadIdx.x / kUpdateCols;
  const int col = blockIdx.x * kUpdateCols + cx;
  const bool live = col <= kLossColumn;
  // Read before this CTA counts itself done, so before the last CTA advances them.
  const int64_t t = *adam.step + 1;
  const uint32_t e = state->epoch + 1u;
  // The column's parameter and moments: the previous step's update kernel wrote them and
  // finished before this step's gradient kernel started, and the gradient kernel does not
  // write them, so they are read before the wait below.
  const bool adam_col = grp == 0 && live && col != kLossColumn;
  float p = 0.0f, m = 0.0f, v = 0.0f;
  if (adam_col) {
    p = adam.params[col];
    m = adam.exp_avg[col];
    v = adam.exp_avg_sq[col];
  }
  // Launched as a dependent of the gradient kernel: its partial rows are complete and
  // visible only after this wait.
  wait_for_prerequisites();

  sums[grp][cx] = live ? column_group_sum(partials, rows, col, grp) : 0.0f;
  __syncthreads();
  if (grp == 0 && live) {
    float total = sums[0][cx];
#pragma unroll
    for (int k = 1; k < kUpdateGroups; ++k) total += sums[k][cx];
    bool ok = true;
    if (world > 1) {
      const size_t slot = (e & 1u) * kMaxRanks;
      const uint64_t word = (static_cast<uint64_t>(e) << 32) | __float_as_uint(total);
      for (int q = 0; q < world; ++q)
        store_word_sys(state->peers[q] + (slot + rank) * kRowStride + col, word);
      const uint64_t* own = state->peers[rank] + slot * kRowStride + col;
      const uint64_t start = global_timer_ns();
      for (int q = 0; q < world && ok; ++q) {
        uint64_t got = load_word_sys(own + static_cast<size_t>(q) * kRowStride);
        while (static_cast<uint32_t>(got >> 32) != e) {
          if (global_timer_ns() - start > wait_limit_ns) {
            report_status(status, FHB_STATUS_PEER_TIMEOUT);
            ok = false;
            break;
          }
          got = load_word_sys(own + static_cast<size_t>(q) * kRowStride);
        }
        const float value = __uint_as_float(static_cast<uint32_t>(got));
        total = q == 0 ? value : total + value;
      }
    }
    if (ok) {
      if (grad_out != nullptr) grad_out[col] = total;
      if (col == kLossColumn) {
        if (loss_out != nullptr) *loss_out = total;
      } else {
        const AdamScalars s = adam_scalars(t, adam.lr, adam.beta1, adam.beta2);
        adam_element(total, p, m, v, s, adam.beta1, adam.beta2, adam.eps);
        adam.exp_avg[col] = m;
        adam.exp_avg_sq[col] = v;
        adam.params[col] = p;
      }
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
  // A dependent launch: its CTAs take the SMs the gradient kernel's CTAs leave, without a
  // launch gap, and wait in wait_for_prerequisites() for the whole gradient grid.
  return launch_dependent(step_update_kernel, dim3(kUpdateBlocks), dim3(kUpdateThreads), 0,
                          stream, partials, rows, state, world, rank, wait_limit_ns, adam,
                          grad_out, loss_out, status);
}

}  // namespace fhb
