// Instantiations of the fused kernels for one quantization mode (g64).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_g64(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQGroup, 2>(a, sh, res, norm, stream);
}

cudaError_t device_error_g64(int* out, bool clear) { return read_device_error(out, clear); }

}  // namespace cutie
