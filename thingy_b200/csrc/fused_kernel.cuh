// Fused [residual add] -> RMSNorm -> [FP8 e4m3 quantization] for sm_100a.
//
// Semantics follow the reference's PyTorch path, step by step:
//   residual add in bf16                 src/cutie/rms_norm/bench.py:97
//   fp32 statistics, rsqrt, bf16 cast
//   before the weight multiply           src/cutie/rms_norm/bench.py:58-65
//   per-group amax, max(amax/448, 1e-4),
//   optional 2^ceil(log2 s), n / s, e4m3 src/cutie/vendor/prime_rl/fp8_utils.py:50-57
// and the single-pass structure of the reference's fused kernel
// (src/cutie/rms_norm/rms_norm.py:115-311): one row team per row, the whole
// row held in registers, one fp32 block reduction for sum(x^2), a lane-group
// shuffle reduction for each group amax (a block reduction in per-token mode).
//
// Layout of work: a CTA of T threads (multiple of 32) owns one row at a time
// and walks rows with a grid stride (persistent grid sized to the resident
// CTA count). Thread t owns the 16-byte vectors v = k*T + t, k < NV, of its
// row, so every load/store instruction of a warp covers 512 contiguous bytes.
// A quantization group of G elements is G/8 consecutive vectors, i.e. G/8
// consecutive lanes for the same k; its amax is a butterfly over those lanes.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace cutie {

enum : int { kQNone = 0, kQToken = 1, kQGroup = 2 };
enum : int { kFmtF32 = 0, kFmtPow2 = 1, kFmtE8M0 = 2 };
enum : int { kLayStrided = 0, kLaySwizzled = 1 };

// Every pointer is device memory; bf16 tensors are passed as raw 16-bit words.
struct FusedArgs {
  const uint16_t* x;
  int64_t ldx;
  const uint16_t* res;  // residual (only read when the kernel has RES)
  int64_t ldr;
  const uint16_t* w;    // RMSNorm weight [H]
  uint16_t* res_out;    // may be null
  int64_t ldro;
  uint16_t* norm_out;   // may be null
  int64_t ldn;
  uint8_t* q;           // e4m3 codes
  int64_t ldq;
  void* scale;          // fp32 or e8m0 bytes
  int64_t s_row;        // strided layout: element offset = row*s_row + g*s_grp
  int64_t s_grp;
  int64_t M;            // rows with data
  int64_t M_pad;        // rows incl. swizzle padding (== M unless swizzled)
  int H;                // columns
  int V;                // 16-byte vectors per row = H / 8
  int n_groups;         // ceil(H / G)
  int n_groups_pad;     // n_groups rounded up to 4 (swizzled) else n_groups
  float eps;
  int scale_fmt;
  int scale_layout;
};

// ---------------------------------------------------------------- bit helpers

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// Round two fp32 values to bf16 (round to nearest even), low half = f.x.
__device__ __forceinline__ uint32_t f2_to_bf2(float2 f) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f.y), "f"(f.x));
  return r;
}

// bf16 x bf16 -> bf16 (exact product, one rounding): the same value torch
// produces for bf16 * bf16 on the CPU (fp32 product, which is exact for two
// 8-bit significands, rounded once to bf16).
__device__ __forceinline__ uint32_t mul_bf2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Running max of magnitudes on bf16 pairs; the sign bits of the result are
// meaningless and are cleared by the caller.
__device__ __forceinline__ uint32_t absmax_bf2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Two fp32 -> two e4m3 codes (round to nearest even, saturate to +-448);
// byte 0 = f.x. |value| never exceeds 448*(1+2^-23) on this path, where
// saturation and the CPU cast (NaN above 464) agree.
__device__ __forceinline__ uint32_t f2_to_e4m3x2(float2 f) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(f.y), "f"(f.x));
  return r;
}

// ------------------------------------------------------------ memory helpers

// Streaming 16-byte load: each activation byte is read exactly once, so keep
// it out of L1 and ask L2 to fetch the whole 256-byte line.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Read-only cached load (weights are shared by every row).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_stream(void* p, uint32_t a, uint32_t b, uint32_t c,
                                          uint32_t d) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_stream2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

// ------------------------------------------------------------ arithmetic

// RN(a / b) from rc = RN(1/b): q0 = RN(a*rc) is within one ulp of a/b, the
// FMA remainder a - b*q0 is then exact, and one correction step
// RN(q0 + rem*rc) yields the correctly rounded quotient (Markstein's theorem,
// P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990). Valid while the
// quotient is a normal fp32 number; below that the fp8 code is 0 anyway.
// nb = -b.
__device__ __forceinline__ float2 div2_rn(float2 a, float2 nb, float2 rc) {
  const float2 q0 = __fmul2_rn(a, rc);
  const float2 rem = __ffma2_rn(q0, nb, a);
  return __ffma2_rn(rem, rc, q0);
}

constexpr float kE4m3Max = 448.0f;
constexpr float kRcpE4m3Max = 1.0f / 448.0f;  // RN(1/448), folded by the compiler
constexpr float kMinScale = 1e-4f;            // fp8_utils.py:51 clamp

// s = max(RN(amax / 448), 1e-4) [rounded up to a power of two for POW2/E8M0].
__device__ __forceinline__ float make_scale(float amax, int fmt) {
  const float q0 = __fmul_rn(amax, kRcpE4m3Max);
  const float rem = __fmaf_rn(q0, -kE4m3Max, amax);
  float s = fmaxf(__fmaf_rn(rem, kRcpE4m3Max, q0), kMinScale);
  if (fmt != kFmtF32) {
    // 2^ceil(log2 s), exactly: keep the exponent, bump it if any mantissa bit
    // is set (s >= 1e-4 is a normal number).
    uint32_t u = __float_as_uint(s);
    if (u & 0x007fffffu) u = (u & 0x7f800000u) + 0x00800000u;
    s = __uint_as_float(u);
  }
  return s;
}

// Byte offset of scale (row, g) in the Blackwell block-scaled GEMM layout:
// 128x4 tiles of 512 bytes, row-block major; inside a tile row r sits at
// (r%32)*16 + (r/32)*4 and group column c at +c.
__device__ __forceinline__ int64_t swizzled_offset(int64_t row, int g, int tiles_per_row) {
  const int64_t tile = (row >> 7) * tiles_per_row + (g >> 2);
  const int r = (int)(row & 127);
  return (tile << 9) + ((r & 31) << 4) + ((r >> 5) << 2) + (g & 3);
}

__device__ __forceinline__ void store_scale(const FusedArgs& a, int64_t row, int g, float s) {
  const uint8_t e8 = (uint8_t)(__float_as_uint(s) >> 23);
  if (a.scale_layout == kLaySwizzled) {
    static_cast<uint8_t*>(a.scale)[swizzled_offset(row, g, a.n_groups_pad >> 2)] = e8;
  } else {
    const int64_t off = row * a.s_row + (int64_t)g * a.s_grp;
    if (a.scale_fmt == kFmtE8M0)
      static_cast<uint8_t*>(a.scale)[off] = e8;
    else
      static_cast<float*>(a.scale)[off] = s;
  }
}

// ------------------------------------------------------------ reductions

template <bool kMax>
__device__ __forceinline__ float warp_reduce(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, u) : __fadd_rn(v, u);
  }
  return v;
}

// Block-wide reduction; every thread returns the same bits (each warp runs
// the identical butterfly over the identical partials). `buf` alternates
// between two 32-float slots so one barrier per reduction suffices.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* buf, int lane, int warp, int nw) {
  v = warp_reduce<kMax>(v);
  if (nw > 1) {
    if (lane == 0) buf[warp] = v;
    __syncthreads();
    v = lane < nw ? buf[lane] : 0.0f;  // 0 is neutral for sums and for max of magnitudes
    v = warp_reduce<kMax>(v);
  }
  return v;
}

// ------------------------------------------------------------ the kernel

template <int NV>
__device__ __forceinline__ void load_row(uint32_t (&v)[NV][4], const uint16_t* row, int t, int T,
                                         int V) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = k * T + t;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (vi < V) u = ld_stream(row + (int64_t)vi * 8);
    v[k][0] = u.x;
    v[k][1] = u.y;
    v[k][2] = u.z;
    v[k][3] = u.w;
  }
}

template <int NV>
__device__ __forceinline__ void store_row(const uint32_t (&v)[NV][4], uint16_t* row, int t, int T,
                                          int V) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int vi = k * T + t;
    if (vi < V) st_stream(row + (int64_t)vi * 8, v[k][0], v[k][1], v[k][2], v[k][3]);
  }
}

// Quantize one 8-element vector with scale s (nb = -s, rc = RN(1/s)) and
// store the 8 codes.
__device__ __forceinline__ void quant_store8(const uint32_t (&n)[4], float s, float rc,
                                             uint8_t* dst) {
  const float2 nb = make_float2(-s, -s), rc2 = make_float2(rc, rc);
  uint32_t c[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) c[j] = f2_to_e4m3x2(div2_rn(bf2_to_f2(n[j]), nb, rc2));
  st_stream2(dst, c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}

__device__ __forceinline__ void zero_scale_padding(const FusedArgs& a, int64_t row, int g0,
                                                   int t, int T) {
  for (int g = g0 + t; g < a.n_groups_pad; g += T)
    static_cast<uint8_t*>(a.scale)[swizzled_offset(row, g, a.n_groups_pad >> 2)] = 0;
}

// NV: 16-byte vectors per thread. QM: quantization mode. GL: lanes per group
// (G/8) in group mode. RES: add the residual first. NORM: apply RMSNorm
// (false = quantize x as is, the per_token_cast_to_fp8 path).
template <int NV, int QM, int GL, bool RES, bool NORM>
__global__ void __launch_bounds__(NV > 4 ? 512 : 1024)
    fused_rmsnorm_fp8_kernel(const FusedArgs a) {
  static_assert(QM != kQGroup || (GL >= 2 && GL <= 16 && (GL & (GL - 1)) == 0), "group lanes");
  static_assert(NORM || !RES, "residual needs the norm");
  __shared__ float red[2][32];

  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  int flip = 0;

  // Weight vectors of this thread, loaded once for all its rows.
  uint32_t w[NV][4];
  if constexpr (NORM) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int vi = k * T + t;
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (vi < a.V) u = ld_keep(a.w + (int64_t)vi * 8);
      w[k][0] = u.x;
      w[k][1] = u.y;
      w[k][2] = u.z;
      w[k][3] = u.w;
    }
  }

  for (int64_t row = blockIdx.x; row < a.M_pad; row += gridDim.x) {
    if (row >= a.M) {  // swizzled-layout padding row: scales only
      zero_scale_padding(a, row, 0, t, T);
      continue;
    }
    uint32_t v[NV][4];
    load_row<NV>(v, a.x + row * a.ldx, t, T, a.V);

    if constexpr (RES) {
      uint32_t r[NV][4];
      load_row<NV>(r, a.res + row * a.ldr, t, T, a.V);
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[k][j] = f2_to_bf2(__fadd2_rn(bf2_to_f2(v[k][j]), bf2_to_f2(r[k][j])));
      if (a.res_out != nullptr) store_row<NV>(v, a.res_out + row * a.ldro, t, T, a.V);
    }

    if constexpr (NORM) {
      // Squares of bf16 values are exact in fp32, so fma == mul-then-add.
      float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = bf2_to_f2(v[k][j]);
          acc = __ffma2_rn(f, f, acc);
        }
      const float ss = block_reduce<false>(__fadd_rn(acc.x, acc.y), red[flip], lane, warp, nw);
      flip ^= 1;
      // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))), not a correctly
      // rounded reciprocal square root; reproduce the double rounding.
      const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.H), a.eps)));
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[k][j] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[k][j]), inv2)), w[k][j]);
      if (a.norm_out != nullptr) store_row<NV>(v, a.norm_out + row * a.ldn, t, T, a.V);
    }

    if constexpr (QM == kQGroup) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = k * T + t;
        const uint32_t m2 = absmax_bf2(absmax_bf2(v[k][0], v[k][1]), absmax_bf2(v[k][2], v[k][3])) &
                            0x7fff7fffu;
        float m = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
#pragma unroll
        for (int o = GL / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (vi < a.V) {
          const float s = make_scale(m, a.scale_fmt);
          if ((t & (GL - 1)) == 0) store_scale(a, row, vi / GL, s);
          quant_store8(v[k], s, __frcp_rn(s), a.q + row * a.ldq + (int64_t)vi * 8);
        }
      }
      if (a.scale_layout == kLaySwizzled && a.n_groups_pad > a.n_groups)
        zero_scale_padding(a, row, a.n_groups, t, T);
    } else if constexpr (QM == kQToken) {
      uint32_t m2 = 0u;
#pragma unroll
      for (int k = 0; k < NV; ++k)
        m2 = absmax_bf2(m2, absmax_bf2(absmax_bf2(v[k][0], v[k][1]), absmax_bf2(v[k][2], v[k][3])));
      m2 &= 0x7fff7fffu;
      float m = fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xffff0000u));
      m = block_reduce<true>(m, red[flip], lane, warp, nw);
      flip ^= 1;
      const float s = make_scale(m, a.scale_fmt);
      const float rc = __frcp_rn(s);
      if (t == 0) store_scale(a, row, 0, s);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int vi = k * T + t;
        if (vi < a.V) quant_store8(v[k], s, rc, a.q + row * a.ldq + (int64_t)vi * 8);
      }
    }
  }
}

// Host-side launcher for one quantization mode (one translation unit each).
// Returns the launch error, if any.
struct LaunchShape {
  int nv;       // vectors per thread, 1..8
  int threads;  // threads per row (= per CTA)
};

}  // namespace cutie
