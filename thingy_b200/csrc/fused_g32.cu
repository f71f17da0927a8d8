// Instantiations of the fused kernel for one quantization mode (g32).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_g32(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQGroup, 4>(a, sh, res, norm, stream);
}

}  // namespace cutie
