// Instantiations of the fused kernel for one quantization mode (token).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_token(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQToken, 0>(a, sh, res, norm, stream);
}

}  // namespace cutie
