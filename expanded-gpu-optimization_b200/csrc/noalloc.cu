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
  float* rows = nullptr;  // device address of g_noalloc_rows on this device
};
NoAllocDevice g_state[kMaxDevices];
std::once_flag g_once[kMaxDevices];

// Once per device, with that device current: the library's shared per-device set-up (kernel
// attributes, SM count, the status word every entry point reports bounded-wait timeouts
// into) and the device address of the scratch array.
void set_up(int device) {
  NoAllocDevice& st = g_state[device];
  const fhb::DeviceInfo* info = nullptr;
  st.code = fhb::current_device_info(&info);
  if (st.code != FHB_OK) return;
  st.code = fhb::record_cuda_error(
      cudaGetSymbolAddress(reinterpret_cast<void**>(&st.rows), g_noalloc_rows));
  if (st.code == FHB_OK && st.rows == nullptr) st.code = FHB_ERR_CUDA;
}

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

extern "C" int fhb_backward_noalloc(const float* coords, const float* params,
                                    const float* grad_u, const float* grad_lap,
                                    float* grad_params, float* grad_coords, int64_t n,
                                    fhb_stream_t stream) {
  // Argument checks come before any CUDA call, so a bad argument never reaches the device.
  if (n < 0 || !params || !grad_params) return FHB_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!coords || !grad_lap)) return FHB_ERR_INVALID_ARGUMENT;
  if (!aligned4(coords) || !aligned4(params) || !aligned4(grad_u) || !aligned4(grad_lap) ||
      !aligned4(grad_params) || !aligned4(grad_coords))
    return FHB_ERR_MISALIGNED;
  int device = 0;
  int code = fhb::record_cuda_error(cudaGetDevice(&device));
  if (code != FHB_OK) return code;
  if (device < 0 || device >= kMaxDevices) return FHB_ERR_INVALID_ARGUMENT;
  std::call_once(g_once[device], [device] { set_up(device); });
  const NoAllocDevice& st = g_state[device];
  if (st.code != FHB_OK) return st.code;
  const fhb::DeviceInfo* info = nullptr;
  code = fhb::current_device_info(&info);  // set up already: returns the shared record
  if (code != FHB_OK) return code;
  if (n == 0)
    return fhb::record_cuda_error(
        cudaMemsetAsync(grad_params, 0, fhb::kParamCount * sizeof(float), stream));
  const int rows = fhb::backward_grid(n, 0, *info);
  if (rows > kNoAllocMaxRows) return FHB_ERR_TOO_LARGE;  // GPU with more SMs than rows
  fhb::PointSets ps;
  ps.interior = coords;
  ps.n = n;
  // The device's status word goes to the kernel: a CTA whose bounded parameter-staging wait
  // gives up sets FHB_STATUS_STAGE_TIMEOUT there (read by fhb_read_device_status) before it
  // returns without writing its row, exactly as in fhb_backward.
  cudaError_t e = fhb::launch_backward_fp32(ps, params, grad_u, grad_lap, grad_coords, nullptr,
                                            st.rows, false, FHB_ACTIVATION_TANH, *info, stream);
  if (e == cudaSuccess) e = fhb::launch_reduce_rows(st.rows, rows, grad_params, nullptr, stream);
  return fhb::record_cuda_error(e);
}
