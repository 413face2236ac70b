// 3xTF32 tcgen05/TMEM forward kernel (forward versions 3..5): not built yet. The launcher
// reports cudaErrorNotSupported so a caller gets an error, never a different kernel.
#include "common.cuh"
#include "kernels.cuh"

namespace fhb {

cudaError_t prepare_forward_tc() { return cudaSuccess; }

cudaError_t launch_forward_tc(const float*, const float*, float*, float*, int64_t,
                              const DeviceInfo&, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace fhb
