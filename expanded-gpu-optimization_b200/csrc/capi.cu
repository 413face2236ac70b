// extern "C" entry points declared in include/fused_hoad_b200.h: argument validation,
// one-time per-device set-up and dispatch onto the sm_100a kernels. No torch types, no
// device allocation, no host synchronisation on the compute entry points.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr int kMaxDevices = 64;

// One status word per device: a file-scope __device__ variable has a separate instance on
// every device that loads this library. Kernels that give up on a bounded wait set bits.
__device__ unsigned int g_status_word;

thread_local int g_last_cuda_error = 0;
fhb::DeviceInfo g_devices[kMaxDevices];
int g_prepare_result[kMaxDevices];
std::once_flag g_prepare_once[kMaxDevices];

int record(cudaError_t e) {
  if (e == cudaSuccess) return FHB_OK;
  g_last_cuda_error = static_cast<int>(e);
  return FHB_ERR_CUDA;
}

int prepare_locked(int device) {
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return record(e);
  if (previous != device && (e = cudaSetDevice(device)) != cudaSuccess) return record(e);
  fhb::DeviceInfo info;
  int code = FHB_OK;
  do {
    if ((e = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess) {
      code = record(e);
      break;
    }
    if (info.cc_major != 10 || info.cc_minor != 0) {
      code = FHB_ERR_DEVICE;  // this library carries sm_100a code only
      break;
    }
    if ((e = cudaGetSymbolAddress(reinterpret_cast<void**>(&info.status), g_status_word)) != cudaSuccess ||
        (e = fhb::prepare_forward_fp32()) != cudaSuccess ||
        (e = fhb::prepare_forward_tc()) != cudaSuccess ||
        (e = fhb::prepare_backward_fp32()) != cudaSuccess ||
        (e = fhb::prepare_backward_tc()) != cudaSuccess ||
        (e = fhb::prepare_biharmonic()) != cudaSuccess) {
      code = record(e);
      break;
    }
    g_devices[device] = info;
  } while (false);
  if (previous != device) cudaSetDevice(previous);
  return code;
}

int prepare(int device) {
  if (device < 0 || device >= kMaxDevices) return FHB_ERR_INVALID_ARGUMENT;
  std::call_once(g_prepare_once[device], [device] { g_prepare_result[device] = prepare_locked(device); });
  return g_prepare_result[device];
}

int current_device(const fhb::DeviceInfo** info) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return record(e);
  const int code = prepare(device);
  if (code != FHB_OK) return code;
  *info = &g_devices[device];
  return FHB_OK;
}

// Enough for either backward kernel: the FP32 one needs one partial row per CTA, the
// tensor-core one also its pre-split weights and per-CTA scratch.
size_t backward_workspace_bytes(int64_t n, int64_t nb, const fhb::DeviceInfo& dev) {
  if (n + nb <= 0) return 0;
  const size_t fp32 =
      static_cast<size_t>(fhb::backward_grid(n, nb, dev)) * fhb::kRowStride * sizeof(float);
  return std::max(fp32, fhb::backward_tc_workspace_bytes(n, nb, dev));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool valid_activation(int activation) {
  return activation == FHB_ACTIVATION_TANH || activation == FHB_ACTIVATION_SILU;
}

bool valid_adam(float lr, float beta1, float beta2, float eps) {
  return lr >= 0.0f && beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f &&
         eps >= 0.0f;
}

// Runs `body` with `device` current, restoring the caller's device afterwards.
template <typename Body>
int on_device(int device, Body body) {
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return record(e);
  if (previous != device && (e = cudaSetDevice(device)) != cudaSuccess) return record(e);
  const int code = body();
  if (previous != device) cudaSetDevice(previous);
  return code;
}

}  // namespace

namespace fhb {
int current_device_info(const DeviceInfo** info) { return current_device(info); }
int record_cuda_error(cudaError_t e) { return record(e); }
}  // namespace fhb

static_assert(sizeof(cudaIpcMemHandle_t) == FHB_EXCHANGE_HANDLE_BYTES, "IPC handle size");
static_assert(fhb::kExchangeBytes == FHB_EXCHANGE_BUFFER_BYTES, "exchange ABI drifted");

// One rank's side of the data-parallel exchange (opaque to callers).
struct fhb_exchange {
  int device = 0;
  int world = 1;
  int rank = 0;
  uint64_t wait_limit_ns = 0;
  uint64_t* buffer = nullptr;            // this rank's exchange buffer (world > 1)
  fhb::ExchangeState* state = nullptr;   // device-resident epoch, done count, peer table
  uint64_t* peers[fhb::kMaxRanks] = {};  // host copy of state->peers
  bool mapped[fhb::kMaxRanks] = {};      // peers[q] is an IPC mapping this object opened
  bool connected = false;
};

namespace {

// Uploads the peer table; the caller has made ex->device current.
int publish_peers(fhb_exchange* ex) {
  fhb::ExchangeState init{};
  for (int q = 0; q < fhb::kMaxRanks; ++q) init.peers[q] = ex->peers[q];
  cudaError_t e = cudaMemcpy(ex->state, &init, sizeof(init), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return record(e);
  ex->connected = true;
  return FHB_OK;
}

void unmap_peers(fhb_exchange* ex) {
  for (int q = 0; q < fhb::kMaxRanks; ++q) {
    if (ex->mapped[q]) cudaIpcCloseMemHandle(ex->peers[q]);
    ex->mapped[q] = false;
    if (q != ex->rank) ex->peers[q] = nullptr;
  }
}

}  // namespace

extern "C" {

const char* fhb_status_string(int code) {
  switch (code) {
    case FHB_OK: return "ok";
    case FHB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FHB_ERR_MISALIGNED: return "misaligned pointer";
    case FHB_ERR_WORKSPACE: return "workspace missing or too small";
    case FHB_ERR_DEVICE: return "current device is not sm_100 (B200); this library holds sm_100a code only";
    case FHB_ERR_CUDA: return "CUDA runtime error";
    case FHB_ERR_TOO_LARGE: return "size beyond the entry point's limit";
    default: return "unknown status";
  }
}

int fhb_last_cuda_error(void) { return g_last_cuda_error; }

int fhb_parameter_count(void) { return fhb::kParamCount; }

int fhb_prepare_device(int device) { return prepare(device); }

int fhb_forward_ex(const float* coords, const float* params, float* u, float* lap, int64_t n,
                   int version, int activation, fhb_stream_t stream) {
  if (version < FHB_FORWARD_VERSION_MIN || version > FHB_FORWARD_VERSION_MAX || n < 0 ||
      !valid_activation(activation))
    return FHB_ERR_INVALID_ARGUMENT;
  if (n == 0) return FHB_OK;
  if (!coords || !params || !u || !lap) return FHB_ERR_INVALID_ARGUMENT;
  if (!aligned(coords, 4) || !aligned(params, 4) || !aligned(u, 4) || !aligned(lap, 4))
    return FHB_ERR_MISALIGNED;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  cudaError_t e;
  if (version <= 2)
    e = fhb::launch_forward_fp32(version, coords, params, u, lap, n, activation, *dev, stream);
  else
    e = fhb::launch_forward_tc(coords, params, u, lap, n, version == FHB_FORWARD_VERSION_F16,
                               activation, *dev, stream);
  return record(e);
}

int fhb_forward(const float* coords, const float* params, float* u, float* lap, int64_t n,
                int version, fhb_stream_t stream) {
  return fhb_forward_ex(coords, params, u, lap, n, version, FHB_ACTIVATION_TANH, stream);
}

int fhb_forward_biharmonic(const float* coords, const float* params, float* u, float* lap,
                           float* bilap, int64_t n, fhb_stream_t stream) {
  if (n < 0) return FHB_ERR_INVALID_ARGUMENT;
  if (n == 0) return FHB_OK;
  if (!coords || !params || !u || !lap || !bilap) return FHB_ERR_INVALID_ARGUMENT;
  if (!aligned(coords, 4) || !aligned(params, 4) || !aligned(u, 4) || !aligned(lap, 4) ||
      !aligned(bilap, 4))
    return FHB_ERR_MISALIGNED;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  return record(fhb::launch_forward_biharmonic(coords, params, u, lap, bilap, n, *dev, stream));
}

size_t fhb_backward_workspace_bytes(int64_t n) {
  const fhb::DeviceInfo* dev = nullptr;
  if (current_device(&dev) != FHB_OK) return 0;
  return backward_workspace_bytes(n, 0, *dev);
}

// Launches the gradient kernel of `tensor_core`'s family into workspace `ws`; *partials and
// *rows locate the partial-gradient rows it leaves for a row reduction.
static cudaError_t launch_gradient_kernel(const fhb::PointSets& ps, const float* params,
                                          const float* grad_u, const float* grad_lap,
                                          float* grad_coords, float* lap_out, bool poisson,
                                          bool tensor_core, int activation, float* ws,
                                          const fhb::DeviceInfo& dev, cudaStream_t stream,
                                          const float** partials, int* rows) {
  // The tensor-core kernel keeps the activations, not the pre-activations, for its adjoint
  // (tanh's derivatives are functions of tanh); other activations run the FP32 kernel.
  if (tensor_core && activation == FHB_ACTIVATION_TANH) {
    *partials = fhb::backward_tc_partials(ws);
    *rows = fhb::backward_tc_rows(ps.n, ps.nb, dev);
    return fhb::launch_backward_tc(ps, params, grad_u, grad_lap, grad_coords, lap_out, ws,
                                   poisson, dev, stream);
  }
  *partials = ws;
  *rows = fhb::backward_grid(ps.n, ps.nb, dev);
  return fhb::launch_backward_fp32(ps, params, grad_u, grad_lap, grad_coords, lap_out, ws,
                                   poisson, activation, dev, stream);
}

// Checks the point sets, parameters and workspace of a gradient launch.
static int check_gradient_inputs(const fhb::PointSets& ps, const float* params, bool poisson,
                                 const float* grad_lap, const void* workspace,
                                 size_t workspace_bytes, const fhb::DeviceInfo& dev) {
  if ((ps.n > 0 && !ps.interior) || (ps.nb > 0 && !ps.boundary) || (!poisson && !grad_lap))
    return FHB_ERR_INVALID_ARGUMENT;
  if (!aligned(ps.interior, 4) || !aligned(ps.boundary, 4) || !aligned(params, 4))
    return FHB_ERR_MISALIGNED;
  const size_t need = backward_workspace_bytes(ps.n, ps.nb, dev);
  if (workspace == nullptr || workspace_bytes < need) return FHB_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return FHB_ERR_MISALIGNED;
  return FHB_OK;
}

static int backward_common(const fhb::PointSets& ps, const float* params, const float* grad_u,
                           const float* grad_lap, float* grad_params, float* grad_coords,
                           float* lap_out, float* loss, bool poisson, bool tensor_core,
                           int activation, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  if (ps.n < 0 || ps.nb < 0 || !params || !grad_params) return FHB_ERR_INVALID_ARGUMENT;
  if (poisson && !loss) return FHB_ERR_INVALID_ARGUMENT;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  if (ps.n + ps.nb == 0) {
    cudaError_t e = cudaMemsetAsync(grad_params, 0, fhb::kParamCount * sizeof(float), stream);
    if (e == cudaSuccess && poisson) e = cudaMemsetAsync(loss, 0, sizeof(float), stream);
    return record(e);
  }
  code = check_gradient_inputs(ps, params, poisson, grad_lap, workspace, workspace_bytes, *dev);
  if (code != FHB_OK) return code;
  const float* partials = nullptr;
  int rows = 0;
  cudaError_t e = launch_gradient_kernel(ps, params, grad_u, grad_lap, grad_coords, lap_out,
                                         poisson, tensor_core, activation,
                                         static_cast<float*>(workspace), *dev, stream,
                                         &partials, &rows);
  if (e == cudaSuccess)
    e = fhb::launch_reduce_rows(partials, rows, grad_params, poisson ? loss : nullptr, stream);
  return record(e);
}

static fhb::PointSets interior_only(const float* coords, int64_t n, int64_t n_total) {
  fhb::PointSets ps;
  ps.interior = coords;
  ps.n = n;
  ps.inv_total = n_total > 0 ? static_cast<float>(1.0 / static_cast<double>(n_total)) : 0.0f;
  return ps;
}

int fhb_backward_ex(const float* coords, const float* params, const float* grad_u,
                    const float* grad_lap, float* grad_params, float* grad_coords, int64_t n,
                    int version, int activation, void* workspace, size_t workspace_bytes,
                    fhb_stream_t stream) {
  if (version < FHB_BACKWARD_VERSION_MIN || version > FHB_BACKWARD_VERSION_MAX ||
      !valid_activation(activation))
    return FHB_ERR_INVALID_ARGUMENT;
  return backward_common(interior_only(coords, n, n), params, grad_u, grad_lap, grad_params,
                         grad_coords, nullptr, nullptr, false,
                         version == FHB_BACKWARD_VERSION_TENSOR_CORE, activation, workspace,
                         workspace_bytes, stream);
}

int fhb_backward(const float* coords, const float* params, const float* grad_u,
                 const float* grad_lap, float* grad_params, float* grad_coords, int64_t n,
                 int version, void* workspace, size_t workspace_bytes, fhb_stream_t stream) {
  return fhb_backward_ex(coords, params, grad_u, grad_lap, grad_params, grad_coords, n, version,
                         FHB_ACTIVATION_TANH, workspace, workspace_bytes, stream);
}

int fhb_poisson_step_gradients(const float* coords, const float* params, int64_t n,
                               int64_t n_total, float* grad_params, float* grad_coords,
                               float* lap_out, float* loss, int version, void* workspace,
                               size_t workspace_bytes, fhb_stream_t stream) {
  if (version < FHB_BACKWARD_VERSION_MIN || version > FHB_BACKWARD_VERSION_MAX ||
      n_total < n)
    return FHB_ERR_INVALID_ARGUMENT;
  return backward_common(interior_only(coords, n, n_total), params, nullptr, nullptr,
                         grad_params, grad_coords, lap_out, loss, true,
                         version == FHB_BACKWARD_VERSION_TENSOR_CORE, FHB_ACTIVATION_TANH,
                         workspace, workspace_bytes, stream);
}

size_t fhb_pinn_step_workspace_bytes(int64_t n, int64_t n_boundary) {
  const fhb::DeviceInfo* dev = nullptr;
  if (n < 0 || n_boundary < 0 || current_device(&dev) != FHB_OK) return 0;
  return backward_workspace_bytes(n, n_boundary, *dev);
}

int fhb_pinn_step_gradients(const float* coords, int64_t n, int64_t n_total,
                            const float* boundary, int64_t n_boundary,
                            int64_t n_boundary_total, float boundary_weight,
                            const float* params, float* grad_params, float* loss, int version,
                            int activation, void* workspace, size_t workspace_bytes,
                            fhb_stream_t stream) {
  if (version < FHB_BACKWARD_VERSION_MIN || version > FHB_BACKWARD_VERSION_MAX || n < 0 ||
      !valid_activation(activation) ||
      n_boundary < 0 || n_total < n || n_boundary_total < n_boundary ||
      !(boundary_weight >= 0.0f))
    return FHB_ERR_INVALID_ARGUMENT;
  fhb::PointSets ps = interior_only(coords, n, n_total);
  ps.boundary = boundary;
  ps.nb = n_boundary;
  ps.inv_btotal = n_boundary_total > 0
                      ? static_cast<float>(1.0 / static_cast<double>(n_boundary_total))
                      : 0.0f;
  ps.bweight = boundary_weight;
  return backward_common(ps, params, nullptr, nullptr, grad_params, nullptr, nullptr, loss,
                         true, version == FHB_BACKWARD_VERSION_TENSOR_CORE, activation,
                         workspace, workspace_bytes, stream);
}

int fhb_adam_step(float* params, const float* grad, float* exp_avg, float* exp_avg_sq,
                  int64_t count, int64_t* step, float lr, float beta1, float beta2, float eps,
                  fhb_stream_t stream) {
  if (!params || !grad || !exp_avg || !exp_avg_sq || !step || count < 0)
    return FHB_ERR_INVALID_ARGUMENT;
  if (!valid_adam(lr, beta1, beta2, eps)) return FHB_ERR_INVALID_ARGUMENT;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  if (count == 0) return FHB_OK;
  return record(fhb::launch_adam(params, grad, exp_avg, exp_avg_sq, count, step, lr, beta1,
                                 beta2, eps, stream));
}

size_t fhb_exchange_buffer_bytes(void) { return fhb::kExchangeBytes; }

int fhb_exchange_create(int world, int rank, uint64_t wait_limit_ns, fhb_exchange** out) {
  if (!out || world < 1 || world > fhb::kMaxRanks || rank < 0 || rank >= world ||
      wait_limit_ns == 0)
    return FHB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  fhb_exchange* ex = new fhb_exchange;
  cudaError_t e = cudaGetDevice(&ex->device);
  ex->world = world;
  ex->rank = rank;
  ex->wait_limit_ns = wait_limit_ns;
  if (e == cudaSuccess) e = cudaMalloc(&ex->state, sizeof(fhb::ExchangeState));
  if (e == cudaSuccess && world > 1) {
    e = cudaMalloc(&ex->buffer, fhb::kExchangeBytes);
    if (e == cudaSuccess) e = cudaMemset(ex->buffer, 0, fhb::kExchangeBytes);
  }
  ex->peers[rank] = ex->buffer;
  code = e == cudaSuccess ? FHB_OK : record(e);
  if (code == FHB_OK) {
    code = publish_peers(ex);  // zero epoch and done count; the peer table is final at world 1
    ex->connected = world == 1;
  }
  if (code != FHB_OK) {
    cudaFree(ex->buffer);
    cudaFree(ex->state);
    delete ex;
    return code;
  }
  *out = ex;
  return FHB_OK;
}

int fhb_exchange_handle(const fhb_exchange* ex, void* handle_out) {
  if (!ex || !handle_out || ex->world < 2) return FHB_ERR_INVALID_ARGUMENT;
  return on_device(ex->device, [&] {
    cudaIpcMemHandle_t handle;
    const cudaError_t e = cudaIpcGetMemHandle(&handle, ex->buffer);
    if (e != cudaSuccess) return record(e);
    memcpy(handle_out, &handle, sizeof(handle));
    return FHB_OK;
  });
}

int fhb_exchange_connect(fhb_exchange* ex, const void* handles) {
  if (!ex || !handles || ex->connected) return FHB_ERR_INVALID_ARGUMENT;
  return on_device(ex->device, [&] {
    const unsigned char* bytes = static_cast<const unsigned char*>(handles);
    for (int q = 0; q < ex->world; ++q) {
      if (q == ex->rank) continue;
      cudaIpcMemHandle_t handle;
      memcpy(&handle, bytes + static_cast<size_t>(q) * sizeof(handle), sizeof(handle));
      void* peer = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&peer, handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        unmap_peers(ex);
        return record(e);
      }
      ex->peers[q] = static_cast<uint64_t*>(peer);
      ex->mapped[q] = true;
    }
    const int code = publish_peers(ex);
    if (code != FHB_OK) unmap_peers(ex);
    return code;
  });
}

int fhb_debug_exchange_connect_local(fhb_exchange* ex, void* const* peer_buffers) {
  if (!ex || !peer_buffers || ex->connected) return FHB_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < ex->world; ++q)
    if (q != ex->rank && (!peer_buffers[q] || !aligned(peer_buffers[q], 16)))
      return FHB_ERR_INVALID_ARGUMENT;
  return on_device(ex->device, [&] {
    for (int q = 0; q < ex->world; ++q)
      if (q != ex->rank) ex->peers[q] = static_cast<uint64_t*>(peer_buffers[q]);
    return publish_peers(ex);
  });
}

int fhb_exchange_buffer(const fhb_exchange* ex, void** buffer_out) {
  if (!ex || !buffer_out) return FHB_ERR_INVALID_ARGUMENT;
  *buffer_out = ex->buffer;
  return FHB_OK;
}

int fhb_exchange_destroy(fhb_exchange* ex) {
  if (!ex) return FHB_OK;
  const int code = on_device(ex->device, [&] {
    cudaError_t e = cudaDeviceSynchronize();
    unmap_peers(ex);
    const cudaError_t e1 = cudaFree(ex->buffer);
    const cudaError_t e2 = cudaFree(ex->state);
    if (e == cudaSuccess) e = e1 != cudaSuccess ? e1 : e2;
    return record(e);
  });
  delete ex;
  return code;
}

int fhb_train_step(const float* coords, int64_t n, int64_t n_total, const float* boundary,
                   int64_t n_boundary, int64_t n_boundary_total, float boundary_weight,
                   float* params, float* exp_avg, float* exp_avg_sq, int64_t* step, float lr,
                   float beta1, float beta2, float eps, fhb_exchange* exchange,
                   float* grad_out, float* loss_out, int version, int activation,
                   void* workspace, size_t workspace_bytes, fhb_stream_t stream) {
  if (version < FHB_BACKWARD_VERSION_MIN || version > FHB_BACKWARD_VERSION_MAX || n < 0 ||
      !valid_activation(activation) ||
      n_boundary < 0 || n_total < n || n_boundary_total < n_boundary ||
      !(boundary_weight >= 0.0f) || !params || !exp_avg || !exp_avg_sq || !step ||
      !valid_adam(lr, beta1, beta2, eps) || !exchange || !exchange->connected)
    return FHB_ERR_INVALID_ARGUMENT;
  if (!aligned(exp_avg, 4) || !aligned(exp_avg_sq, 4) || !aligned(step, 8) ||
      !aligned(grad_out, 4) || !aligned(loss_out, 4))
    return FHB_ERR_MISALIGNED;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return record(e);
  if (device != exchange->device) return FHB_ERR_INVALID_ARGUMENT;
  fhb::PointSets ps = interior_only(coords, n, n_total);
  ps.boundary = boundary;
  ps.nb = n_boundary;
  ps.inv_btotal = n_boundary_total > 0
                      ? static_cast<float>(1.0 / static_cast<double>(n_boundary_total))
                      : 0.0f;
  ps.bweight = boundary_weight;
  const float* partials = nullptr;
  int rows = 0;  // a rank with no points still takes part in the exchange, with zeros
  if (n + n_boundary > 0) {
    code = check_gradient_inputs(ps, params, true, nullptr, workspace, workspace_bytes, *dev);
    if (code != FHB_OK) return code;
    e = launch_gradient_kernel(ps, params, nullptr, nullptr, nullptr, nullptr, true,
                               version == FHB_BACKWARD_VERSION_TENSOR_CORE, activation,
                               static_cast<float*>(workspace), *dev, stream, &partials, &rows);
    if (e != cudaSuccess) return record(e);
  } else if (!aligned(params, 4)) {
    return FHB_ERR_MISALIGNED;
  }
  const fhb::AdamArgs adam{params, exp_avg, exp_avg_sq, step, lr, beta1, beta2, eps};
  return record(fhb::launch_step_update(partials, rows, exchange->state, exchange->world,
                                        exchange->rank, exchange->wait_limit_ns, adam,
                                        grad_out, loss_out, dev->status, stream));
}

int fhb_read_device_status(int device, unsigned int* status_out) {
  if (!status_out) return FHB_ERR_INVALID_ARGUMENT;
  int code = prepare(device);
  if (code != FHB_OK) return code;
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return record(e);
  if (previous != device && (e = cudaSetDevice(device)) != cudaSuccess) return record(e);
  const unsigned int zero = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status_out, g_status_word, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_status_word, &zero, sizeof(unsigned int));
  if (previous != device) cudaSetDevice(previous);
  return record(e);
}

int fhb_debug_bounded_wait_selftest(uint64_t limit_ns, fhb_stream_t stream) {
  if (limit_ns == 0 || limit_ns > 10ull * 1000000000ull) return FHB_ERR_INVALID_ARGUMENT;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  return record(fhb::launch_bounded_wait_selftest(limit_ns, dev->status, stream));
}

int fhb_debug_tanh(const float* x, float* out, int64_t n, int fast, fhb_stream_t stream) {
  if (n < 0 || (n > 0 && (!x || !out))) return FHB_ERR_INVALID_ARGUMENT;
  const fhb::DeviceInfo* dev = nullptr;
  int code = current_device(&dev);
  if (code != FHB_OK) return code;
  if (n == 0) return FHB_OK;
  return record(fhb::launch_debug_tanh(x, out, n, fast, stream));
}

}  // extern "C"
