// Standalone fp32 RMSNorm, the reference's older baseline
// (src/cutie/rms_norm/rms_norm.py:11-20):
//   variance = mean(x^2) + eps;  out = x / sqrt(variance) * weight
// evaluated with the rounding of eager fp32 torch: every square, the sum, the
// mean, the eps add, the sqrt, the division and the weight product are each
// rounded to fp32 once. Same row-per-CTA, grid-stride structure as the fused
// kernel; 16-byte vectors hold 4 floats.
#include "launch.cuh"

namespace cutie {

template <int NV>
__global__ void __launch_bounds__(NV > 4 ? 512 : 1024) rmsnorm_f32_kernel(const F32Args a) {
  __shared__ float red[2][32];
  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  int flip = 0;

  griddep_wait();  // inputs of the previous kernel are complete from here on
  griddep_launch_dependents();
  float4 w[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = k * T + t;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (vi < a.V) u = ld_keep(a.w + (int64_t)vi * 4);
    w[k] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                       __uint_as_float(u.w));
  }

  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    float4 v[NV];
    const float* xr = a.x + row * a.ldx;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = k * T + t;
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (vi < a.V) u = ld_stream(xr + (int64_t)vi * 4);
      v[k] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                         __uint_as_float(u.w));
    }
    // x.pow(2) is rounded before the sum: multiply and add separately. The
    // adds are the scalar __fadd_rn, which is never merged into a multiply-add
    // (the packed fp32x2 forms are: a product feeding a packed add came out
    // rounded once).
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const float2 lo = make_float2(v[k].x, v[k].y), hi = make_float2(v[k].z, v[k].w);
      float2 sq = __fmul2_rn(lo, lo);
      acc = make_float2(__fadd_rn(acc.x, sq.x), __fadd_rn(acc.y, sq.y));
      sq = __fmul2_rn(hi, hi);
      acc = make_float2(__fadd_rn(acc.x, sq.x), __fadd_rn(acc.y, sq.y));
    }
    const float ss = block_reduce<false>(__fadd_rn(acc.x, acc.y), red[flip], lane, warp, nw);
    flip ^= 1;
    const float sd = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.H), a.eps));
    const float2 nb = make_float2(-sd, -sd);
    const float rcs = __frcp_rn(sd);
    const float2 rc = make_float2(rcs, rcs);
    float* orow = a.out + row * a.ldo;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = k * T + t;
      if (vi >= a.V) continue;
      float2 lo = div2_rn(make_float2(v[k].x, v[k].y), nb, rc);
      float2 hi = div2_rn(make_float2(v[k].z, v[k].w), nb, rc);
      // The one-step correction needs a normal quotient; redo tiny ones with
      // the IEEE division (a rare, data-dependent branch).
      if (fabsf(lo.x) < 0x1p-100f) lo.x = __fdiv_rn(v[k].x, sd);
      if (fabsf(lo.y) < 0x1p-100f) lo.y = __fdiv_rn(v[k].y, sd);
      if (fabsf(hi.x) < 0x1p-100f) hi.x = __fdiv_rn(v[k].z, sd);
      if (fabsf(hi.y) < 0x1p-100f) hi.y = __fdiv_rn(v[k].w, sd);
      lo = __fmul2_rn(lo, make_float2(w[k].x, w[k].y));
      hi = __fmul2_rn(hi, make_float2(w[k].z, w[k].w));
      const uint32_t out4[4] = {__float_as_uint(lo.x), __float_as_uint(lo.y),
                                __float_as_uint(hi.x), __float_as_uint(hi.y)};
      st_stream(orow + (int64_t)vi * 4, out4);
    }
  }
}

template <int NV>
static cudaError_t launch_f32_one(const F32Args& a, int threads, cudaStream_t stream) {
  auto kernel = rmsnorm_f32_kernel<NV>;
  const int per_sm = cached_blocks_per_sm(reinterpret_cast<const void*>(kernel), threads, 0);
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  int64_t grid = (int64_t)per_sm * device_sm_count();
  if (grid > a.M) grid = a.M;
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kernel, (unsigned)grid, (unsigned)threads, (size_t)0, stream, a);
}

cudaError_t launch_rmsnorm_f32(const F32Args& a, F32Shape sh, cudaStream_t stream) {
  switch (sh.nv) {
    case 1: return launch_f32_one<1>(a, sh.threads, stream);
    case 2: return launch_f32_one<2>(a, sh.threads, stream);
    case 3: return launch_f32_one<3>(a, sh.threads, stream);
    case 4: return launch_f32_one<4>(a, sh.threads, stream);
    case 5: return launch_f32_one<5>(a, sh.threads, stream);
    case 6: return launch_f32_one<6>(a, sh.threads, stream);
    case 7: return launch_f32_one<7>(a, sh.threads, stream);
    case 8: return launch_f32_one<8>(a, sh.threads, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cutie
