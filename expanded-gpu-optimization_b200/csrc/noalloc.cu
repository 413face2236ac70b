// fhb_backward_noalloc: the backward (vector-Jacobian product) with its scratch memory in a
// file-scope device array instead of a caller-supplied workspace.
//
// Who needs this: callers that cannot allocate device memory where they call the backward.
// Hosts that reach this library through a thin FFI (ctypes, cgo, JNI) often have no handle
// on a device allocator at all; deployments that fix their device-memory budget at start-up
// (per-process limits under MPS, real-time services) forbid allocations later; and
// cudaMalloc synchronises the whole device, which a latency-bound caller cannot afford in
// its step. fhb_backward needs a workspace of fhb_backward_workspace_bytes(n) bytes; this
// variant needs none.
//
// The scratch: one partial-gradient row per CTA of the persistent grid, at most
// kNoAllocMaxRows rows (148 = one per SM of a B200; 148 x 12,740 floats = 7.5 MB). Every GPU
// that loads this library holds that array until the process exits. Each CTA overwrites its
// whole row before the row reduction reads it, so nothing needs clearing between calls, but
// every call shares the one array: calls that overlap on the GPU (two streams, two threads)
// race on it and give wrong gradients. Order them on one stream.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr int kNoAllocMaxRows = 148;
constexpr int kMaxDevices = 64;

// Device-side scratch. In host code this name is only a stand-in for the symbol, not a
// device address: its address on each device comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_rows[kNoAllocMaxRows * fhb::kRowStride];

struct NoAllocDevice {
  int code = FHB_OK;
  fhb::DeviceInfo info;
  float* rows = nullptr;  // device address of g_noalloc_rows on this device
};
NoAllocDevice g_state[kMaxDevices];
std::once_flag g_once[kMaxDevices];

// Once per device, with that device current: the kernels' attributes (fhb_prepare_device),
// the SM count, and the device address of the scratch array.
void set_up(int device) {
  NoAllocDevice& st = g_state[device];
  st.code = fhb_prepare_device(device);
  if (st.code != FHB_OK) return;
  cudaError_t e = cudaDeviceGetAttribute(&st.info.sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.rows), g_noalloc_rows);
  if (e != cudaSuccess || st.rows == nullptr) {
    st.code = FHB_ERR_CUDA;
    return;
  }
  st.info.status = nullptr;  // bounded-wait timeouts of this variant are not recorded
}

}  // namespace

extern "C" int fhb_backward_noalloc(const float* coords, const float* params,
                                    const float* grad_u, const float* grad_lap,
                                    float* grad_params, float* grad_coords, int64_t n,
                                    fhb_stream_t stream) {
  if (n < 0 || !params || !grad_params) return FHB_ERR_INVALID_ARGUMENT;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return FHB_ERR_CUDA;
  if (device < 0 || device >= kMaxDevices) return FHB_ERR_INVALID_ARGUMENT;
  std::call_once(g_once[device], [device] { set_up(device); });
  const NoAllocDevice& st = g_state[device];
  if (st.code != FHB_OK) return st.code;
  if (n == 0) {
    e = cudaMemsetAsync(grad_params, 0, fhb::kParamCount * sizeof(float), stream);
    return e == cudaSuccess ? FHB_OK : FHB_ERR_CUDA;
  }
  if (!coords || !grad_lap) return FHB_ERR_INVALID_ARGUMENT;
  const int rows = fhb::backward_grid(n, 0, st.info);
  if (rows > kNoAllocMaxRows) return FHB_ERR_TOO_LARGE;  // GPU with more SMs than rows
  fhb::PointSets ps;
  ps.interior = coords;
  ps.n = n;
  e = fhb::launch_backward_fp32(ps, params, grad_u, grad_lap, grad_coords, nullptr, st.rows,
                                false, FHB_ACTIVATION_TANH, st.info, stream);
  if (e == cudaSuccess) e = fhb::launch_reduce_rows(st.rows, rows, grad_params, nullptr, stream);
  return e == cudaSuccess ? FHB_OK : FHB_ERR_CUDA;
}
