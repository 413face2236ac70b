// torch.utils.cpp_extension binding: the module fused_hoad._C with the reference's op
// contract (csrc/bindings.cpp:9-66 in the reference): same function names, argument names
// and defaults, same validation order and messages. Every op calls the C ABI of
// libfused_hoad_b200.so (include/fused_hoad_b200.h); outputs and workspaces come from the
// ATen caching allocator on the current stream, so the ops stay asynchronous and
// CUDA-graph capturable.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "../../include/fused_hoad_b200.h"

namespace {

constexpr int64_t kParameterCount = FHB_PARAMETER_COUNT;

void check_inputs(const torch::Tensor& coordinates, const torch::Tensor& parameters) {
  TORCH_CHECK(coordinates.is_cuda(), "coordinates must be a CUDA tensor");
  TORCH_CHECK(parameters.is_cuda(), "parameters must be a CUDA tensor");
  TORCH_CHECK(coordinates.is_contiguous(), "coordinates must be contiguous");
  TORCH_CHECK(parameters.is_contiguous(), "parameters must be contiguous");
  TORCH_CHECK(coordinates.scalar_type() == torch::kFloat32, "coordinates must use float32");
  TORCH_CHECK(parameters.scalar_type() == torch::kFloat32, "parameters must use float32");
  TORCH_CHECK(coordinates.dim() == 2 && coordinates.size(1) == 2,
              "coordinates must have shape [batch, 2]");
  TORCH_CHECK(parameters.dim() == 1 && parameters.numel() == kParameterCount,
              "parameters must have shape [12737]");
  TORCH_CHECK(coordinates.device() == parameters.device(),
              "coordinates and parameters must be on the same device");
}

void check_vector(const torch::Tensor& t, const torch::Tensor& like, int64_t numel,
                  const char* what) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == torch::kFloat32,
              what, " must be a contiguous float32 CUDA tensor");
  TORCH_CHECK(t.numel() == numel, what, " must have ", numel, " values");
  TORCH_CHECK(t.device() == like.device(), what, " must be on the parameters' device");
}

void check_status(int code, const char* op) {
  if (code == FHB_OK) return;
  if (code == FHB_ERR_CUDA) {
    const auto err = static_cast<cudaError_t>(fhb_last_cuda_error());
    TORCH_CHECK(false, op, " failed: ", fhb_status_string(code), ": ", cudaGetErrorString(err));
  }
  TORCH_CHECK(false, op, " failed: ", fhb_status_string(code));
}

// Hidden activation by name: "tanh" (the reference kernels' activation, the default) or
// "silu" (the other jet of the reference's PyTorch forward-Laplacian backend).
int activation_code(const std::string& activation) {
  if (activation == "tanh") return FHB_ACTIVATION_TANH;
  if (activation == "silu") return FHB_ACTIVATION_SILU;
  TORCH_CHECK(false, "activation must be \"tanh\" or \"silu\"");
  return -1;
}

torch::Tensor workspace_for(int64_t batch, const torch::Tensor& like) {
  const size_t bytes = fhb_backward_workspace_bytes(batch);
  return torch::empty({static_cast<int64_t>((bytes + 15) / 16) * 4}, like.options());
}

}  // namespace

std::vector<torch::Tensor> fused_forward_laplacian(torch::Tensor coordinates,
                                                   torch::Tensor parameters, int64_t version,
                                                   const std::string& activation) {
  TORCH_CHECK(version >= 0 && version <= 5, "version must be 0 to 5");
  check_inputs(coordinates, parameters);
  const int act = activation_code(activation);
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0);
  auto output = torch::empty({batch, 1}, coordinates.options());
  auto laplacian = torch::empty({batch, 1}, coordinates.options());
  if (batch == 0) return {output, laplacian};
  check_status(fhb_forward_ex(coordinates.data_ptr<float>(), parameters.data_ptr<float>(),
                              output.data_ptr<float>(), laplacian.data_ptr<float>(), batch,
                              static_cast<int>(version), act,
                              at::cuda::getCurrentCUDAStream()),
               "fused_forward_laplacian");
  return {output, laplacian};
}

// (u, lap, bilap) [N,1] each: the biharmonic of the tanh MLP (fhb_forward_biharmonic).
std::vector<torch::Tensor> fused_forward_biharmonic(torch::Tensor coordinates,
                                                    torch::Tensor parameters) {
  check_inputs(coordinates, parameters);
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0);
  auto output = torch::empty({batch, 1}, coordinates.options());
  auto laplacian = torch::empty({batch, 1}, coordinates.options());
  auto biharmonic = torch::empty({batch, 1}, coordinates.options());
  if (batch == 0) return {output, laplacian, biharmonic};
  check_status(fhb_forward_biharmonic(coordinates.data_ptr<float>(),
                                      parameters.data_ptr<float>(), output.data_ptr<float>(),
                                      laplacian.data_ptr<float>(), biharmonic.data_ptr<float>(),
                                      batch, at::cuda::getCurrentCUDAStream()),
               "fused_forward_biharmonic");
  return {output, laplacian, biharmonic};
}

std::vector<torch::Tensor> fused_forward_laplacian_backward(torch::Tensor coordinates,
                                                            torch::Tensor parameters,
                                                            torch::Tensor grad_output,
                                                            torch::Tensor grad_laplacian,
                                                            int64_t version,
                                                            const std::string& activation) {
  TORCH_CHECK(version >= 1 && version <= 6, "backward version must be 1 to 6");
  check_inputs(coordinates, parameters);
  const int act = activation_code(activation);
  for (const auto& grad : {grad_output, grad_laplacian}) {
    TORCH_CHECK(grad.is_cuda() && grad.is_contiguous() && grad.scalar_type() == torch::kFloat32,
                "upstream gradients must be contiguous float32 CUDA tensors");
    TORCH_CHECK(grad.numel() == coordinates.size(0), "upstream gradients must have [batch] values");
  }
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0);
  auto grad_coordinates = torch::empty_like(coordinates);
  if (batch == 0) return {torch::zeros_like(parameters), grad_coordinates};
  auto grad_parameters = torch::empty_like(parameters);
  auto workspace = workspace_for(batch, parameters);
  check_status(
      fhb_backward_ex(coordinates.data_ptr<float>(), parameters.data_ptr<float>(),
                      grad_output.data_ptr<float>(), grad_laplacian.data_ptr<float>(),
                      grad_parameters.data_ptr<float>(), grad_coordinates.data_ptr<float>(),
                      batch, static_cast<int>(version), act, workspace.data_ptr<float>(),
                      static_cast<size_t>(workspace.numel()) * sizeof(float),
                      at::cuda::getCurrentCUDAStream()),
      "fused_forward_laplacian_backward");
  return {grad_parameters, grad_coordinates};
}

// ---- B200-native additions (no counterpart in the reference's _C) ----

// Zero-copy evaluation of points that live in pinned host memory: pinned allocations are
// device-addressable, so the kernel reads the points and writes (u, lap) straight over the
// host link while it computes -- no staging copies, the transfer overlaps the work. Outputs
// are pinned host tensors ([N,1] each), valid once the current stream of the parameters'
// device has completed; pass `output`/`laplacian` to reuse buffers.
std::vector<torch::Tensor> fused_forward_laplacian_host(torch::Tensor coordinates,
                                                        torch::Tensor parameters,
                                                        int64_t version,
                                                        c10::optional<torch::Tensor> output,
                                                        c10::optional<torch::Tensor> laplacian,
                                                        const std::string& activation) {
  TORCH_CHECK(version >= 0 && version <= 5, "version must be 0 to 5");
  const int act = activation_code(activation);
  TORCH_CHECK(!coordinates.is_cuda() && coordinates.is_pinned(),
              "coordinates must be a pinned host tensor");
  TORCH_CHECK(parameters.is_cuda(), "parameters must be a CUDA tensor");
  TORCH_CHECK(coordinates.is_contiguous() && parameters.is_contiguous(),
              "coordinates and parameters must be contiguous");
  TORCH_CHECK(coordinates.scalar_type() == torch::kFloat32 &&
                  parameters.scalar_type() == torch::kFloat32,
              "coordinates and parameters must use float32");
  TORCH_CHECK(coordinates.dim() == 2 && coordinates.size(1) == 2,
              "coordinates must have shape [batch, 2]");
  TORCH_CHECK(parameters.dim() == 1 && parameters.numel() == kParameterCount,
              "parameters must have shape [12737]");
  const int64_t batch = coordinates.size(0);
  auto pinned = torch::TensorOptions().dtype(torch::kFloat32).pinned_memory(true);
  auto u = output.has_value() ? *output : torch::empty({batch, 1}, pinned);
  auto lap = laplacian.has_value() ? *laplacian : torch::empty({batch, 1}, pinned);
  for (const auto& t : {u, lap}) {
    TORCH_CHECK(!t.is_cuda() && t.is_pinned() && t.is_contiguous() &&
                    t.scalar_type() == torch::kFloat32 && t.numel() == batch,
                "outputs must be pinned contiguous float32 host tensors with [batch] values");
  }
  if (batch == 0) return {u, lap};
  const c10::cuda::CUDAGuard device_guard(parameters.device());
  check_status(fhb_forward_ex(coordinates.data_ptr<float>(), parameters.data_ptr<float>(),
                              u.data_ptr<float>(), lap.data_ptr<float>(), batch,
                              static_cast<int>(version), act, at::cuda::getCurrentCUDAStream()),
               "fused_forward_laplacian_host");
  return {u, lap};
}

// ---- B200-native training-step ops ----

// Fused Poisson step gradients; see fhb_poisson_step_gradients. Returns
// [grad_and_loss [12738] (gradient, then this shard's loss in the last slot),
//  laplacian [N,1] or empty, grad_coordinates [N,2] or empty]. `total_points` is the
// global batch (data-parallel shards pass the sum). One flat buffer lets a data-parallel
// step all-reduce gradient and loss with a single collective.
std::vector<torch::Tensor> poisson_step_gradients(torch::Tensor coordinates,
                                                  torch::Tensor parameters,
                                                  int64_t total_points, bool want_laplacian,
                                                  bool want_grad_coordinates, int64_t version) {
  check_inputs(coordinates, parameters);
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0);
  TORCH_CHECK(total_points >= batch, "total_points must be >= the local batch");
  TORCH_CHECK(version >= 1 && version <= 6, "backward version must be 1 to 6");
  auto grad_and_loss = torch::empty({kParameterCount + 1}, parameters.options());
  auto laplacian = want_laplacian ? torch::empty({batch, 1}, coordinates.options())
                                  : torch::empty({0}, coordinates.options());
  auto grad_coordinates = want_grad_coordinates ? torch::empty_like(coordinates)
                                                : torch::empty({0}, coordinates.options());
  auto workspace = workspace_for(batch, parameters);
  float* out = grad_and_loss.data_ptr<float>();
  check_status(fhb_poisson_step_gradients(
                   coordinates.data_ptr<float>(), parameters.data_ptr<float>(), batch,
                   total_points, out,
                   want_grad_coordinates ? grad_coordinates.data_ptr<float>() : nullptr,
                   want_laplacian ? laplacian.data_ptr<float>() : nullptr,
                   out + kParameterCount, static_cast<int>(version),
                   batch ? workspace.data_ptr<float>() : nullptr,
                   static_cast<size_t>(workspace.numel()) * sizeof(float),
                   at::cuda::getCurrentCUDAStream()),
               "poisson_step_gradients");
  return {grad_and_loss, laplacian, grad_coordinates};
}

// Fused gradients of the full PINN loss (residual on `coordinates` + boundary_weight *
// mean(u^2) on `boundary`); see fhb_pinn_step_gradients. Returns grad_and_loss [12738]
// (gradient, then this shard's loss). The totals are the global counts of each set.
torch::Tensor pinn_step_gradients(torch::Tensor coordinates, torch::Tensor boundary,
                                  torch::Tensor parameters, int64_t total_points,
                                  int64_t boundary_total, double boundary_weight,
                                  int64_t version, const std::string& activation) {
  const int act = activation_code(activation);
  check_inputs(coordinates, parameters);
  check_inputs(boundary, parameters);
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0), nb = boundary.size(0);
  TORCH_CHECK(total_points >= batch, "total_points must be >= the local batch");
  TORCH_CHECK(boundary_total >= nb, "boundary_total must be >= the local boundary batch");
  TORCH_CHECK(version >= 1 && version <= 6, "backward version must be 1 to 6");
  auto grad_and_loss = torch::empty({kParameterCount + 1}, parameters.options());
  const size_t bytes = fhb_pinn_step_workspace_bytes(batch, nb);
  auto workspace =
      torch::empty({static_cast<int64_t>((bytes + sizeof(float) - 1) / sizeof(float))},
                   parameters.options());
  float* out = grad_and_loss.data_ptr<float>();
  check_status(fhb_pinn_step_gradients(
                   coordinates.data_ptr<float>(), batch, total_points,
                   boundary.data_ptr<float>(), nb, boundary_total,
                   static_cast<float>(boundary_weight), parameters.data_ptr<float>(), out,
                   out + kParameterCount, static_cast<int>(version), act,
                   bytes ? workspace.data_ptr<float>() : nullptr,
                   static_cast<size_t>(workspace.numel()) * sizeof(float),
                   at::cuda::getCurrentCUDAStream()),
               "pinn_step_gradients");
  return grad_and_loss;
}

// In-place Adam on flat buffers; `step` is a CUDA int64 tensor of one element.
void adam_step(torch::Tensor parameters, torch::Tensor grad, torch::Tensor exp_avg,
               torch::Tensor exp_avg_sq, torch::Tensor step, double lr, double beta1,
               double beta2, double eps) {
  const int64_t count = parameters.numel();
  check_vector(parameters, parameters, count, "parameters");
  check_vector(grad, parameters, count, "grad");
  check_vector(exp_avg, parameters, count, "exp_avg");
  check_vector(exp_avg_sq, parameters, count, "exp_avg_sq");
  TORCH_CHECK(step.is_cuda() && step.scalar_type() == torch::kInt64 && step.numel() == 1,
              "step must be a CUDA int64 tensor with one element");
  const c10::cuda::CUDAGuard device_guard(parameters.device());
  check_status(fhb_adam_step(parameters.data_ptr<float>(), grad.data_ptr<float>(),
                             exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), count,
                             step.data_ptr<int64_t>(), static_cast<float>(lr),
                             static_cast<float>(beta1), static_cast<float>(beta2),
                             static_cast<float>(eps), at::cuda::getCurrentCUDAStream()),
               "adam_step");
}

// ---- data-parallel exchange and the fused training step ----
// An exchange object crosses into Python as its address (an int).

fhb_exchange* as_exchange(int64_t handle) {
  TORCH_CHECK(handle != 0, "exchange is closed");
  return reinterpret_cast<fhb_exchange*>(static_cast<intptr_t>(handle));
}

int64_t exchange_create(int64_t world, int64_t rank, double wait_limit_s, int64_t device) {
  TORCH_CHECK(wait_limit_s > 0.0 && wait_limit_s <= 3600.0, "wait_limit_s must be in (0, 3600]");
  const c10::cuda::CUDAGuard device_guard(static_cast<c10::DeviceIndex>(device));
  fhb_exchange* ex = nullptr;
  check_status(fhb_exchange_create(static_cast<int>(world), static_cast<int>(rank),
                                   static_cast<uint64_t>(wait_limit_s * 1e9), &ex),
               "exchange_create");
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(ex));
}

torch::Tensor exchange_handle(int64_t handle) {
  auto out = torch::empty({FHB_EXCHANGE_HANDLE_BYTES}, torch::kUInt8);
  check_status(fhb_exchange_handle(as_exchange(handle), out.data_ptr<uint8_t>()),
               "exchange_handle");
  return out;
}

void exchange_connect(int64_t handle, torch::Tensor handles) {
  TORCH_CHECK(!handles.is_cuda() && handles.scalar_type() == torch::kUInt8 &&
                  handles.is_contiguous() && handles.numel() % FHB_EXCHANGE_HANDLE_BYTES == 0,
              "handles must be a contiguous CPU uint8 tensor of whole IPC handles");
  check_status(fhb_exchange_connect(as_exchange(handle), handles.data_ptr<uint8_t>()),
               "exchange_connect");
}

void exchange_connect_local(int64_t handle, std::vector<int64_t> peer_buffers) {
  std::vector<void*> ptrs;
  for (int64_t p : peer_buffers) ptrs.push_back(reinterpret_cast<void*>(static_cast<intptr_t>(p)));
  check_status(fhb_debug_exchange_connect_local(as_exchange(handle), ptrs.data()),
               "exchange_connect_local");
}

int64_t exchange_buffer(int64_t handle) {
  void* buffer = nullptr;
  check_status(fhb_exchange_buffer(as_exchange(handle), &buffer), "exchange_buffer");
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(buffer));
}

void exchange_destroy(int64_t handle) {
  check_status(fhb_exchange_destroy(as_exchange(handle)), "exchange_destroy");
}

// One fused training step (fhb_train_step): gradient kernel, then sum over the exchange's
// ranks + Adam in one update kernel. Returns the global loss [1]; grad_out, when given, gets
// the global gradient and the loss (12,738 floats).
torch::Tensor train_step(torch::Tensor coordinates, torch::Tensor boundary,
                         torch::Tensor parameters, torch::Tensor exp_avg,
                         torch::Tensor exp_avg_sq, torch::Tensor step, double lr, double beta1,
                         double beta2, double eps, int64_t total_points, int64_t boundary_total,
                         double boundary_weight, int64_t exchange, int64_t version,
                         c10::optional<torch::Tensor> grad_out, const std::string& activation) {
  const int act = activation_code(activation);
  check_inputs(coordinates, parameters);
  check_inputs(boundary, parameters);
  check_vector(exp_avg, parameters, kParameterCount, "exp_avg");
  check_vector(exp_avg_sq, parameters, kParameterCount, "exp_avg_sq");
  TORCH_CHECK(step.is_cuda() && step.scalar_type() == torch::kInt64 && step.numel() == 1 &&
                  step.device() == parameters.device(),
              "step must be a CUDA int64 tensor with one element on the parameters' device");
  if (grad_out) check_vector(*grad_out, parameters, kParameterCount + 1, "grad_out");
  const c10::cuda::CUDAGuard device_guard(coordinates.device());
  const int64_t batch = coordinates.size(0), nb = boundary.size(0);
  TORCH_CHECK(total_points >= batch, "total_points must be >= the local batch");
  TORCH_CHECK(boundary_total >= nb, "boundary_total must be >= the local boundary batch");
  TORCH_CHECK(version >= 1 && version <= 6, "backward version must be 1 to 6");
  auto loss = torch::empty({1}, parameters.options());
  const size_t bytes = fhb_pinn_step_workspace_bytes(batch, nb);
  auto workspace =
      torch::empty({static_cast<int64_t>((bytes + 15) / 16) * 4}, parameters.options());
  check_status(
      fhb_train_step(coordinates.data_ptr<float>(), batch, total_points,
                     boundary.data_ptr<float>(), nb, boundary_total,
                     static_cast<float>(boundary_weight), parameters.data_ptr<float>(),
                     exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(),
                     step.data_ptr<int64_t>(), static_cast<float>(lr),
                     static_cast<float>(beta1), static_cast<float>(beta2),
                     static_cast<float>(eps), as_exchange(exchange),
                     grad_out ? grad_out->data_ptr<float>() : nullptr, loss.data_ptr<float>(),
                     static_cast<int>(version), act,
                     bytes ? workspace.data_ptr<float>() : nullptr,
                     static_cast<size_t>(workspace.numel()) * sizeof(float),
                     at::cuda::getCurrentCUDAStream()),
      "train_step");
  return loss;
}

void prepare_device(int64_t device) {
  check_status(fhb_prepare_device(static_cast<int>(device)), "prepare_device");
}

int64_t read_device_status(int64_t device) {
  unsigned int status = 0;
  check_status(fhb_read_device_status(static_cast<int>(device), &status), "read_device_status");
  return static_cast<int64_t>(status);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("fused_forward_laplacian", &fused_forward_laplacian,
             "Fixed MLP forward pass and input Laplacian (CUDA, sm_100a)",
             pybind11::arg("coordinates"), pybind11::arg("parameters"),
             pybind11::arg("version") = 2, pybind11::arg("activation") = "tanh");
  module.def("fused_forward_biharmonic", &fused_forward_biharmonic,
             "Fixed tanh MLP forward pass, its input Laplacian and biharmonic (CUDA, sm_100a)",
             pybind11::arg("coordinates"), pybind11::arg("parameters"));
  module.def("fused_forward_laplacian_backward", &fused_forward_laplacian_backward,
             "Gradients of the fused forward Laplacian w.r.t. parameters and coordinates "
             "(CUDA, sm_100a)",
             pybind11::arg("coordinates"), pybind11::arg("parameters"),
             pybind11::arg("grad_output"), pybind11::arg("grad_laplacian"),
             pybind11::arg("version") = 6, pybind11::arg("activation") = "tanh");
  module.def("fused_forward_laplacian_host", &fused_forward_laplacian_host,
             "Forward Laplacian of points in pinned host memory, read and written by the "
             "kernel over the host link (zero-copy)",
             pybind11::arg("coordinates"), pybind11::arg("parameters"),
             pybind11::arg("version") = 3, pybind11::arg("output") = pybind11::none(),
             pybind11::arg("laplacian") = pybind11::none(), pybind11::arg("activation") = "tanh");
  module.def("pinn_step_gradients", &pinn_step_gradients,
             "Fused gradients of the Poisson PINN loss (interior residual + boundary term)",
             pybind11::arg("coordinates"), pybind11::arg("boundary"),
             pybind11::arg("parameters"), pybind11::arg("total_points"),
             pybind11::arg("boundary_total"), pybind11::arg("boundary_weight") = 100.0,
             pybind11::arg("version") = 6, pybind11::arg("activation") = "tanh");
  module.def("poisson_step_gradients", &poisson_step_gradients,
             "Fused forward + interior Poisson loss + backward in one persistent kernel",
             pybind11::arg("coordinates"), pybind11::arg("parameters"),
             pybind11::arg("total_points"), pybind11::arg("want_laplacian") = false,
             pybind11::arg("want_grad_coordinates") = false, pybind11::arg("version") = 6);
  module.def("adam_step", &adam_step, "Fused Adam over a flat parameter buffer",
             pybind11::arg("parameters"), pybind11::arg("grad"), pybind11::arg("exp_avg"),
             pybind11::arg("exp_avg_sq"), pybind11::arg("step"), pybind11::arg("lr"),
             pybind11::arg("beta1"), pybind11::arg("beta2"), pybind11::arg("eps"));
  module.def("exchange_create", &exchange_create,
             "New data-parallel exchange for rank `rank` of `world` on `device`",
             pybind11::arg("world"), pybind11::arg("rank"), pybind11::arg("wait_limit_s"),
             pybind11::arg("device"));
  module.def("exchange_handle", &exchange_handle,
             "CUDA IPC handle of this rank's exchange buffer (CPU uint8 [64])",
             pybind11::arg("exchange"));
  module.def("exchange_connect", &exchange_connect,
             "Map the peers' exchange buffers from their IPC handles (rank order)",
             pybind11::arg("exchange"), pybind11::arg("handles"));
  module.def("exchange_connect_local", &exchange_connect_local,
             "Test hook: connect to peer buffers given as device addresses",
             pybind11::arg("exchange"), pybind11::arg("peer_buffers"));
  module.def("exchange_buffer", &exchange_buffer, "Device address of this rank's buffer",
             pybind11::arg("exchange"));
  module.def("exchange_destroy", &exchange_destroy, "Unmap the peers and free the buffers",
             pybind11::arg("exchange"));
  module.def("train_step", &train_step,
             "Fused training step: gradient kernel, then the sum over ranks and Adam in one "
             "update kernel",
             pybind11::arg("coordinates"), pybind11::arg("boundary"),
             pybind11::arg("parameters"), pybind11::arg("exp_avg"),
             pybind11::arg("exp_avg_sq"), pybind11::arg("step"), pybind11::arg("lr"),
             pybind11::arg("beta1"), pybind11::arg("beta2"), pybind11::arg("eps"),
             pybind11::arg("total_points"), pybind11::arg("boundary_total"),
             pybind11::arg("boundary_weight"), pybind11::arg("exchange"),
             pybind11::arg("version") = 6, pybind11::arg("grad_out") = pybind11::none(),
             pybind11::arg("activation") = "tanh");
  module.def("prepare_device", &prepare_device, "One-time per-device kernel set-up",
             pybind11::arg("device"));
  module.def("read_device_status", &read_device_status,
             "Read and clear the device's bounded-wait status word (synchronises)",
             pybind11::arg("device"));
}
