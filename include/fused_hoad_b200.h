/*
 * fused_hoad_b200 -- C ABI of the B200-native (sm_100a) forward-Laplacian kernels for the
 * fixed 2 -> 64 -> 64 -> 64 -> 64 -> 1 tanh MLP.
 *
 * Plain pointers, sizes and a CUDA stream; no torch types. Every pointer is a device
 * pointer on the current CUDA device unless stated. All compute calls are asynchronous on
 * `stream`, never synchronise the host and never allocate device memory (callers pass the
 * workspace a call needs), so they can be captured in a CUDA graph once the per-device
 * set-up (fhb_prepare_device, or the first call on that device) has run outside capture.
 * The set-up calls of the data-parallel exchange (fhb_exchange_*) are the exception: they
 * allocate and synchronise, once per trainer.
 *
 * Parameter buffer: the reference's packed ABI (csrc/mlp_abi.cuh:8-17), 12,737 floats:
 * W0[64][2] b0[64] | W1[64][64] b1[64] | W2 b2 | W3 b3 | w_out[64] b_out[1], W row-major
 * [out][in] as nn.Linear stores it.
 *
 * Return value: FHB_OK or one of the FHB_ERR_* codes; fhb_status_string() names them.
 */
#ifndef FUSED_HOAD_B200_H_
#define FUSED_HOAD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as cudaStream_t, so a cudaStream_t converts without a cast. */
typedef struct CUstream_st* fhb_stream_t;

#define FHB_PARAMETER_COUNT 12737

#define FHB_OK 0
#define FHB_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad version */
#define FHB_ERR_MISALIGNED 2       /* a pointer breaks the alignment the call documents */
#define FHB_ERR_WORKSPACE 3        /* workspace missing or smaller than required */
#define FHB_ERR_DEVICE 4           /* current device is not sm_100 (B200) */
#define FHB_ERR_CUDA 5             /* a CUDA runtime call failed; see fhb_last_cuda_error */
#define FHB_ERR_TOO_LARGE 6        /* size beyond what the entry point supports */

/* Bits of the per-device status word a kernel sets when a bounded wait gives up. */
#define FHB_STATUS_STAGE_TIMEOUT 0x1u /* parameter staging copy never completed */
#define FHB_STATUS_MMA_TIMEOUT 0x2u   /* tensor-core pipeline wait gave up */
#define FHB_STATUS_PEER_TIMEOUT 0x4u  /* an exchange wait for a peer rank gave up */
#define FHB_STATUS_SELFTEST 0x80u     /* set by fhb_debug_bounded_wait_selftest */

/* Forward kernel families selected by `version` (reference csrc/bindings.cpp:33). */
#define FHB_FORWARD_VERSION_MIN 0
#define FHB_FORWARD_VERSION_MAX 5
/* Version 3 runs the 3xFP16 tensor-core kernel (f16 operand pairs with power-of-2 range
 * scaling), 4 and 5 the 3xTF32 one; both keep FP32-level accuracy. */
#define FHB_FORWARD_VERSION_F16 3
/* Backward versions accepted for drop-in compatibility (reference csrc/bindings.cpp:45). */
#define FHB_BACKWARD_VERSION_MIN 1
#define FHB_BACKWARD_VERSION_MAX 6
/* Backward versions 1..5 run the FP32 CUDA-core adjoint kernel; 6 (the reference's default)
 * runs the tensor-core one (forward recompute and input adjoint in 3xFP16, weight gradient
 * as scaled f16 hi/lo pairs, all on tcgen05). Both reduce in a fixed order. */
#define FHB_BACKWARD_VERSION_TENSOR_CORE 6

/* Hidden-layer activations (reference src/fused_hoad/specs.py:17, models.py:9-12). The
 * reference's fused CUDA path is tanh only; SiLU is the jet of its PyTorch forward-Laplacian
 * backend (src/fused_hoad/backends/forward_laplacian.py:34-38). */
#define FHB_ACTIVATION_TANH 0
#define FHB_ACTIVATION_SILU 1

const char* fhb_status_string(int code);
/* Last CUDA runtime error seen by this library on the calling thread (cudaError_t). */
int fhb_last_cuda_error(void);
int fhb_parameter_count(void);

/*
 * One-time per-device set-up (kernel attributes, SM count, status word). Called
 * implicitly by the first call of any entry point on a device; call it explicitly before
 * capturing a CUDA graph on a device that has not run a kernel yet. Fails (FHB_ERR_CUDA,
 * no kernel launched) if the tensor-core forward was built with another register count
 * than its warpgroups' register split assumes.
 */
int fhb_prepare_device(int device);

/*
 * Forward Laplacian: u[n], lap[n] for coords[n][2] (row-major, 8 bytes per point).
 * Replaces fused_forward_laplacian_cuda (reference csrc/fused_residual.cu:587-643) behind
 * fused_hoad._C.fused_forward_laplacian (csrc/bindings.cpp:31-36).
 * version 0..2: FP32 CUDA-core kernel (0: 32-point tiles, 1: 128-point tiles,
 *               2: 64-point tiles, the default);
 * version 3:    3xFP16 tcgen05/TMEM tensor-core kernel (kind::f16; hi/lo f16 operand pairs
 *               with per-launch power-of-2 scales derived from the weights, so no operand
 *               leaves the f16 range; FP32-level accuracy), the fastest. The scales come
 *               from FP32 upper bounds of the jets, which overflow for weights around
 *               3e5 times the nn.Linear default init (|W| ~ 4e4); use 4 or 5 beyond that;
 * version 4, 5: 3xTF32 tcgen05/TMEM tensor-core kernel (FP32-level accuracy over the whole
 *               FP32 range).
 * n == 0 is a no-op. The parameter buffer may have any 4-byte alignment.
 */
int fhb_forward(const float* coords, const float* params, float* u, float* lap, int64_t n,
                int version, fhb_stream_t stream);
/*
 * fhb_forward with the hidden activation chosen (FHB_ACTIVATION_*); fhb_forward is this call
 * with FHB_ACTIVATION_TANH. SiLU is the jet of the reference's PyTorch forward-Laplacian
 * backend (src/fused_hoad/backends/forward_laplacian.py:34-38); versions 0..2 run the FP32
 * kernel with it, versions 3..5 the 3xTF32 tensor-core kernel (SiLU's activations are
 * unbounded, so the 3xFP16 operand scales, derived from weights alone, do not apply).
 */
int fhb_forward_ex(const float* coords, const float* params, float* u, float* lap, int64_t n,
                   int version, int activation, fhb_stream_t stream);

/*
 * The biharmonic of the tanh MLP: u[n], lap[n] (the Laplacian) and bilap[n] (the Laplacian
 * of the Laplacian, u_xxxx + 2 u_xxyy + u_yyyy) at coords[n][2], on the FP32 CUDA cores by a
 * nine-component jet (value, gradient, Hessian, gradient of the Laplacian, biharmonic per
 * neuron). No counterpart entry in the reference, which names the biharmonic as the next
 * operator for its kernel design and computes it only by nested autograd
 * (src/fused_hoad/autodiff.py:39-41 applied twice). Tolerance against that FP64 autograd:
 * that of the FP32 forward (atol 1e-5, rtol 1e-4). n == 0 is a no-op.
 */
int fhb_forward_biharmonic(const float* coords, const float* params, float* u, float* lap,
                           float* bilap, int64_t n, fhb_stream_t stream);

/*
 * Workspace the backward needs for n points on the current device, in bytes (0 for n==0),
 * enough for every backward version: one partial-gradient row per CTA of the persistent
 * grid (the tensor-core kernel fills one per cluster of two CTAs), and for the tensor-core
 * kernel also the f16 pre-split weights (96 KB) and 256 KB of per-CTA scratch that stays in
 * L2 (about 45 MB on a 148-SM B200 from 18,944 points up).
 */
size_t fhb_backward_workspace_bytes(int64_t n);

/*
 * Vector-Jacobian product of the forward Laplacian: given grad_u[n] and grad_lap[n]
 * (dLoss/du, dLoss/dlap), writes grad_params[12737] and grad_coords[n][2].
 * Replaces fused_forward_laplacian_backward_cuda (reference csrc/fused_backward.cu:859-934)
 * behind fused_hoad._C.fused_forward_laplacian_backward (csrc/bindings.cpp:42-54).
 * grad_u may be NULL (treated as zeros); grad_coords may be NULL (not written).
 * The reduction over points has a fixed order: results are bitwise reproducible for a
 * given n, version and device. n == 0 writes zeros to grad_params. Versions 1..5 run the
 * FP32 CUDA-core kernel, 6 the tensor-core kernel (FHB_BACKWARD_VERSION_TENSOR_CORE).
 * Workspace: fhb_backward_workspace_bytes(n) bytes, 16-byte aligned.
 */
int fhb_backward(const float* coords, const float* params, const float* grad_u,
                 const float* grad_lap, float* grad_params, float* grad_coords, int64_t n,
                 int version, void* workspace, size_t workspace_bytes, fhb_stream_t stream);
/*
 * fhb_backward with the hidden activation chosen; fhb_backward is this call with
 * FHB_ACTIVATION_TANH. SiLU runs the FP32 CUDA-core adjoint kernel for every version (its
 * adjoint needs the pre-activations, which that kernel keeps in registers).
 */
int fhb_backward_ex(const float* coords, const float* params, const float* grad_u,
                    const float* grad_lap, float* grad_params, float* grad_coords, int64_t n,
                    int version, int activation, void* workspace, size_t workspace_bytes,
                    fhb_stream_t stream);

/*
 * fhb_backward without a workspace argument: no counterpart in the reference (its backward
 * allocates partials and scratch with the ATen allocator on every call).
 * For callers that cannot allocate device memory where they call the backward: hosts
 * behind a thin FFI with no device allocator, processes whose device-memory budget is fixed
 * at start-up, and callers that cannot afford cudaMalloc's device-wide synchronisation.
 * The scratch is a file-scope device array of 148 partial-gradient rows (7.5 MB, one row per
 * SM of a B200) that every GPU loading this library holds until exit; the call returns
 * FHB_ERR_TOO_LARGE when the persistent grid for n would need more rows (only on a GPU with
 * more than 148 SMs). The first call on a device does the set-up (kernel attributes, the
 * array's device address), so make it before any stream capture. All calls share the array:
 * calls that overlap on the GPU race on it -- order them on one stream. Otherwise as
 * fhb_backward: grad_u may be NULL, grad_coords may be NULL, n == 0 zeroes grad_params; a
 * pointer that is not 4-byte aligned returns FHB_ERR_MISALIGNED before anything is
 * launched; a bounded wait in the kernel that gives up sets its bit in the device status
 * word (fhb_read_device_status), and fhb_last_cuda_error reports this call's CUDA errors.
 */
int fhb_backward_noalloc(const float* coords, const float* params, const float* grad_u,
                         const float* grad_lap, float* grad_params, float* grad_coords,
                         int64_t n, fhb_stream_t stream);

/*
 * Fused Poisson training-step gradients for the interior loss
 *     L = sum_p (lap_p - f(x_p))^2 / n_total,  f = -2 pi^2 sin(pi x) sin(pi y)
 * (reference benchmarks/benchmark_training.py:46-48, src/fused_hoad/problems/poisson.py:37-39):
 * one persistent kernel recomputes the forward jet per tile, forms dL/dlap in registers and
 * runs the adjoint sweep, so no separate forward launch is needed. Writes grad_params[12737]
 * (this shard's contribution; n_total >= n lets data-parallel shards sum to the global
 * gradient), *loss (this shard's contribution, device scalar), optionally lap_out[n] and
 * grad_coords[n][2] (either may be NULL). `version` picks the kernel as for fhb_backward
 * (6: tensor cores). Workspace as for fhb_backward.
 */
int fhb_poisson_step_gradients(const float* coords, const float* params, int64_t n,
                               int64_t n_total, float* grad_params, float* grad_coords,
                               float* lap_out, float* loss, int version, void* workspace,
                               size_t workspace_bytes, fhb_stream_t stream);

/*
 * Fused gradients of the full Poisson PINN loss of the reference's training driver
 * (src/fused_hoad/training.py:68-94, benchmarks/train_poisson.py):
 *     L = sum_p (lap_p - f(x_p))^2 / n_total + w * sum_b u(x_b)^2 / n_boundary_total
 * over interior points coords[n][2] and boundary points boundary[n_boundary][2] (w =
 * boundary_weight, the reference's default is 100). One launch walks the interior tiles
 * and then the boundary tiles (the boundary term is the VJP of u alone: grad_u = 2 w u /
 * n_boundary_total, grad_lap = 0), so one reduction gives grad_params[12737] and *loss of
 * both terms (this shard's contributions; the totals >= the local counts let data-parallel
 * shards sum to the global values). No counterpart entry in the reference, whose boundary
 * term is a separate eager forward and autograd backward. `version` as for fhb_backward,
 * `activation` an FHB_ACTIVATION_* (SiLU runs the FP32 kernel).
 * Workspace: fhb_pinn_step_workspace_bytes(n, n_boundary) bytes, 16-byte aligned.
 */
size_t fhb_pinn_step_workspace_bytes(int64_t n, int64_t n_boundary);
int fhb_pinn_step_gradients(const float* coords, int64_t n, int64_t n_total,
                            const float* boundary, int64_t n_boundary,
                            int64_t n_boundary_total, float boundary_weight,
                            const float* params, float* grad_params, float* loss, int version,
                            int activation, void* workspace, size_t workspace_bytes,
                            fhb_stream_t stream);

/*
 * One Adam step on a flat buffer, torch.optim.Adam semantics (no weight decay, no amsgrad),
 * replacing the optimizer of reference benchmarks/benchmark_training.py:41, :54-56.
 * `step` is a device int64 counter holding the number of steps taken so far; the kernel
 * reads it, uses step+1 for the bias corrections and stores step+1, so the call can be
 * replayed from a CUDA graph.
 */
int fhb_adam_step(float* params, const float* grad, float* exp_avg, float* exp_avg_sq,
                  int64_t count, int64_t* step, float lr, float beta1, float beta2, float eps,
                  fhb_stream_t stream);

/*
 * ---- Training step: fused update and the data-parallel gradient exchange ----
 * No counterpart in the reference (single GPU; its step is autograd + torch.optim.Adam,
 * benchmarks/benchmark_training.py:51-56). The step's tail -- the fixed-order sum of the
 * backward's partial rows, the sum over ranks and Adam -- is one kernel. With more than one
 * rank, each rank stores its column sums straight into every peer's exchange buffer over
 * NVLink (CUDA IPC mappings, plain 64-bit stores of value and epoch together) and reads the
 * peers' words from its own buffer, each wait bounded; every rank then sums the ranks in rank
 * order, so all replicas get bitwise the same gradient and update. No NCCL call on the step.
 *
 * An exchange object holds this rank's buffer, the mapped peer buffers and a device epoch
 * counter. Set-up calls (create, handle, connect, destroy) allocate, synchronise and may not
 * be captured; the step itself is asynchronous and capturable. Every rank of a group must run
 * the same number of steps, in order, one process per GPU (never two ranks of a group on one
 * GPU: their kernels wait on one another).
 * Exchange buffer layout (FHB_EXCHANGE_BUFFER_BYTES):
 *   uint64_t words[2][FHB_EXCHANGE_MAX_RANKS][FHB_EXCHANGE_ROW_WORDS]
 *   slot = epoch % 2, row = source rank; word = (epoch << 32) | bits of the float column sum
 *   (columns 0..12736 the gradient, 12737 the loss).
 */
#define FHB_EXCHANGE_MAX_RANKS 8
#define FHB_EXCHANGE_ROW_WORDS 12740
#define FHB_EXCHANGE_HANDLE_BYTES 64
#define FHB_EXCHANGE_BUFFER_BYTES (2 * FHB_EXCHANGE_MAX_RANKS * FHB_EXCHANGE_ROW_WORDS * 8)

typedef struct fhb_exchange fhb_exchange;

/* Bytes of one rank's exchange buffer. */
size_t fhb_exchange_buffer_bytes(void); /* FHB_EXCHANGE_BUFFER_BYTES */
/*
 * New exchange for rank `rank` of `world` (1..FHB_EXCHANGE_MAX_RANKS) on the current device;
 * wait_limit_ns bounds every wait for a peer. world == 1 needs no connect (and no buffer).
 */
int fhb_exchange_create(int world, int rank, uint64_t wait_limit_ns, fhb_exchange** out);
/* CUDA IPC handle of this rank's buffer (FHB_EXCHANGE_HANDLE_BYTES bytes) for the peers. */
int fhb_exchange_handle(const fhb_exchange* exchange, void* handle_out);
/* Maps the peers' buffers: handles = world handles in rank order (own entry ignored). */
int fhb_exchange_connect(fhb_exchange* exchange, const void* handles);
/* This rank's buffer (device pointer), for tests and inspection. */
int fhb_exchange_buffer(const fhb_exchange* exchange, void** buffer_out);
/*
 * Test hook: connect with peer buffers given as device pointers of the current device
 * (peer_buffers[world], own entry ignored) instead of IPC handles, so one process can stand
 * in for the peers of a rank by writing their words itself.
 */
int fhb_debug_exchange_connect_local(fhb_exchange* exchange, void* const* peer_buffers);
/* Unmaps the peers and frees the buffers (synchronises the device). Every rank must have
 * finished its last step first (a host barrier after a device synchronise). */
int fhb_exchange_destroy(fhb_exchange* exchange);

/*
 * One fused training step of the Poisson PINN on this rank's shard: the gradient kernel of
 * fhb_pinn_step_gradients (boundary may be NULL with n_boundary 0: the interior loss of
 * fhb_poisson_step_gradients), then one update kernel that sums the partial rows, sums over
 * the exchange's ranks and applies Adam (as fhb_adam_step) to params / exp_avg / exp_avg_sq /
 * step. grad_out (NULL or 12,738 floats) receives the global gradient and then the global
 * loss; loss_out (NULL or 1 float) the global loss. `activation` is an FHB_ACTIVATION_*
 * (SiLU runs the FP32 gradient kernel). The totals are the global counts. If a
 * peer wait gives up, FHB_STATUS_PEER_TIMEOUT is set, the parameters whose wait gave up are
 * left unchanged and the replicas are no longer consistent: stop or reload a checkpoint.
 * Workspace: fhb_pinn_step_workspace_bytes(n, n_boundary) bytes, 16-byte aligned.
 * With the tensor-core kernel the step is three launches in `stream`: the weight pre-split
 * (an ordinary launch), then the gradient kernel and the update kernel as programmatic
 * dependent launches, each starting while the kernel before it finishes and waiting on the
 * device for that kernel's results.
 */
int fhb_train_step(const float* coords, int64_t n, int64_t n_total, const float* boundary,
                   int64_t n_boundary, int64_t n_boundary_total, float boundary_weight,
                   float* params, float* exp_avg, float* exp_avg_sq, int64_t* step, float lr,
                   float beta1, float beta2, float eps, fhb_exchange* exchange,
                   float* grad_out, float* loss_out, int version, int activation,
                   void* workspace, size_t workspace_bytes, fhb_stream_t stream);

/* Reads and clears the status word of `device` (synchronises that device). */
int fhb_read_device_status(int device, unsigned int* status_out);

/*
 * Test hook for the bounded-wait machinery: launches one CTA that waits on an mbarrier
 * nothing arrives at, with a limit of `limit_ns` nanoseconds; the wait gives up, sets
 * FHB_STATUS_SELFTEST in the device status word and the kernel returns normally.
 */
int fhb_debug_bounded_wait_selftest(uint64_t limit_ns, fhb_stream_t stream);

/*
 * Test hook for the tensor-core kernel's tanh: out[i] = tanh_fast(x[i]) when fast != 0
 * (tanh from 1 - 2/(exp(2x)+1) on the special-function unit), else CUDA's tanhf(x[i]).
 */
int fhb_debug_tanh(const float* x, float* out, int64_t n, int fast, fhb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FUSED_HOAD_B200_H_ */
