// Launch plumbing shared by the per-mode translation units. Each mode's
// kernels are instantiated in their own .cu file so nvcc builds them in
// parallel; capi.cu only sees the launch_fused_* entry points below.
#pragma once

#include "fused_kernel.cuh"

namespace cutie {

// Defined in capi.cu. Both are cached per device / per (kernel, block size).
int device_sm_count();
int cached_blocks_per_sm(const void* kernel, int threads);

// Persistent grid: as many CTAs as can be resident at once, never more than
// the number of rows to walk.
template <int NV, int QM, int GL, bool RES, bool NORM>
cudaError_t launch_fused_one(const FusedArgs& a, int threads, cudaStream_t stream) {
  auto kernel = fused_rmsnorm_fp8_kernel<NV, QM, GL, RES, NORM>;
  const int per_sm = cached_blocks_per_sm(reinterpret_cast<const void*>(kernel), threads);
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  int64_t grid = (int64_t)per_sm * device_sm_count();
  if (grid > a.M_pad) grid = a.M_pad;
  if (grid <= 0) return cudaSuccess;
  kernel<<<(unsigned)grid, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

template <int QM, int GL, bool RES, bool NORM>
cudaError_t launch_fused_nv(const FusedArgs& a, LaunchShape sh, cudaStream_t stream) {
  switch (sh.nv) {
    case 1: return launch_fused_one<1, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 2: return launch_fused_one<2, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 3: return launch_fused_one<3, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 4: return launch_fused_one<4, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 5: return launch_fused_one<5, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 6: return launch_fused_one<6, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 7: return launch_fused_one<7, QM, GL, RES, NORM>(a, sh.threads, stream);
    case 8: return launch_fused_one<8, QM, GL, RES, NORM>(a, sh.threads, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int QM, int GL>
cudaError_t launch_fused_mode(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  if (!norm) {
    if constexpr (QM != kQNone) return launch_fused_nv<QM, GL, false, false>(a, sh, stream);
    return cudaErrorInvalidValue;
  }
  return res ? launch_fused_nv<QM, GL, true, true>(a, sh, stream)
             : launch_fused_nv<QM, GL, false, true>(a, sh, stream);
}

cudaError_t launch_fused_none(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream);
cudaError_t launch_fused_token(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                               cudaStream_t stream);
cudaError_t launch_fused_g32(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                             cudaStream_t stream);
cudaError_t launch_fused_g64(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                             cudaStream_t stream);
cudaError_t launch_fused_g128(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream);

struct F32Args {
  const float* x;
  int64_t ldx;
  const float* w;
  float* out;
  int64_t ldo;
  int64_t M;
  int H;
  int V;  // 16-byte vectors per row = H / 4
  float eps;
};

cudaError_t launch_rmsnorm_f32(const F32Args& a, LaunchShape sh, cudaStream_t stream);

}  // namespace cutie
