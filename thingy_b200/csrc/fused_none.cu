// Instantiations of the fused kernel for one quantization mode (none).
#include "launch.cuh"

namespace cutie {

cudaError_t launch_fused_none(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  return launch_fused_mode<kQNone, 0>(a, sh, res, norm, stream);
}

}  // namespace cutie
