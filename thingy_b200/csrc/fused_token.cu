// Instantiations of the fused kernels for one quantization mode (token).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_token(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQToken, 1>(a, sh, res, norm, stream);
}

cudaError_t device_error_token(int* out, bool clear) { return read_device_error(out, clear); }

}  // namespace cutie
