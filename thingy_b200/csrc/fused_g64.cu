// Instantiations of the fused kernel for one quantization mode (g64).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_g64(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQGroup, 8>(a, sh, res, norm, stream);
}

}  // namespace cutie
