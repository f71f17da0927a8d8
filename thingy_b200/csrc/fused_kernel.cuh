// Fused [residual add] -> RMSNorm -> [FP8 e4m3 quantization] for sm_100a.
//
// Semantics follow the reference's PyTorch path, step by step:
//   residual add in bf16                 src/cutie/rms_norm/bench.py:97
//   fp32 statistics, rsqrt, bf16 cast
//   before the weight multiply           src/cutie/rms_norm/bench.py:58-65
//   per-group amax, max(amax/448, 1e-4),
//   optional 2^ceil(log2 s), n / s, e4m3 src/cutie/vendor/prime_rl/fp8_utils.py:50-57
// and the single-pass structure of the reference's fused kernel
// (src/cutie/rms_norm/rms_norm.py:115-311): the row held on chip, one fp32
// block reduction for sum(x^2), per-group amax by lane shuffles (a block
// reduction in per-token mode).
//
// Data movement: the copy engine streams whole rows (x and residual) into a
// ring of shared-memory stages with cp.async.bulk, each stage tracked by an
// mbarrier. A persistent CTA walks rows with a grid stride; thread 0 refills
// a stage with the row `stages` iterations ahead as soon as every thread has
// read it (the first block barrier of the row), so HBM reads run ahead of the
// arithmetic without holding registers. Outputs leave through streaming
// stores from registers.
//
// Work layout: a row is cut into 64-byte chunks of 4 vectors (32 elements);
// thread t of a T-thread CTA owns chunks c*T + t, c < NCH. A 1x32 group is
// one chunk (one thread, no shuffles), 1x64 two lanes, 1x128 four lanes, so
// scale and reciprocal are computed once per 32 elements. Thread t visits the
// 4 vectors of its chunk starting at vector (t>>1)&3: with 64-byte chunks the
// 16-byte shared-memory reads of a warp would otherwise fall into two bank
// groups; rotated, each quarter-warp covers all 32 banks.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace cutie {

enum : int { kQNone = 0, kQToken = 1, kQGroup = 2 };
enum : int { kFmtF32 = 0, kFmtPow2 = 1, kFmtE8M0 = 2 };
enum : int { kLayStrided = 0, kLaySwizzled = 1 };

// Device-side error word (bounded waits that ran out). Written only on
// failure; read and cleared through cutie_device_error(). Each translation
// unit that launches kernels has its own copy (internal linkage, no
// relocatable device code needed); the host side reads all of them.
enum : int { kDevErrNone = 0, kDevErrBulkWaitTimeout = 1, kDevErrBadLaunch = 2 };
static __device__ int g_cutie_device_error = 0;

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
  int64_t s_row;        // strided layouts: element offset of (row, g) =
  int64_t s_grp;        //   row*s_row + (g/4)*s_grp4 + (g%4)*s_grp
  int64_t s_grp4;       // (4*s_grp, except for e8m0 bytes packed 4 to a word)
  int64_t M;            // rows with data
  int64_t M_pad;        // rows incl. swizzle padding (== M unless swizzled)
  int H;                // columns
  int V;                // 16-byte vectors per row = H / 8
  int n_groups;         // ceil(H / G)
  int n_groups_pad;     // n_groups rounded up to 4 (swizzled) else n_groups
  float eps;
  float rcp_H;          // RN(1 / H)
  int scale_fmt;
  int scale_layout;
  int stages;           // shared-memory ring depth (>= 2)
  long long wait_limit; // SM cycles a wait may block before it gives up (< 0: never blocks)
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

// Lane-wise max of two non-negative bf16 pairs.
__device__ __forceinline__ uint32_t max_bf2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Four fp32 -> four e4m3 codes in one word (round to nearest even, saturate
// to +-448); byte 0 = a.x. |value| never exceeds 448*(1+2^-23) on this path,
// where saturation and the CPU cast (NaN above 464) agree.
__device__ __forceinline__ uint32_t f4_to_e4m3x4(float2 a, float2 b) {
  uint32_t r;
  asm("{\n .reg .b16 lo, hi;\n"
      " cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
      " cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
      " mov.b32 %0, {lo, hi};\n}"
      : "=r"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// ------------------------------------------------- programmatic dependent launch
//
// Kernels here are launched with programmatic stream serialization: the next
// kernel of the stream may be scheduled as soon as every CTA of the current
// one has called griddep_launch_dependents(), and runs its prologue (shared
// memory and barrier set-up) while the current one drains. Every kernel calls
// griddep_wait() before its first global-memory access; it returns once the
// preceding grid has completed and its writes are visible, so inputs written
// by the previous kernel are never read early. Without the launch attribute
// both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ memory helpers

// Read-only cached load (weights are shared by every row).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Streaming 16-byte load: read once, keep out of L1, fetch whole L2 lines.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_smem(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(addr));
  return r;
}

__device__ __forceinline__ void st_stream(void* p, const uint32_t (&v)[4]) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

__device__ __forceinline__ void st_stream2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

// Streaming stores guarded by `ok` inside the instruction (no branch).
__device__ __forceinline__ void st_stream_if(bool ok, void* p, const uint32_t (&v)[4]) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.u32 q, %5, 0;\n"
      " @q st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};\n}" ::"l"(p),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"((uint32_t)ok)
      : "memory");
}

__device__ __forceinline__ void st_stream2_if(bool ok, void* p, uint32_t a, uint32_t b) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.u32 q, %3, 0;\n"
      " @q st.global.cs.v2.u32 [%0], {%1,%2};\n}" ::"l"(p),
      "r"(a), "r"(b), "r"((uint32_t)ok)
      : "memory");
}

// 32-byte streaming store (one full sector), address 32-byte aligned.
__device__ __forceinline__ void st_stream8(void* p, const uint32_t* v) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// ------------------------------------------------- natural-order chunk stores
//
// A thread visits the 4 vectors of its 64-byte chunk in a rotated order (slot
// k holds vector (k + rot) & 3; see the kernels). Stored in that order, every
// store instruction of a warp covers each 32-byte sector of the output only
// partly. These helpers put a chunk back in vector order and store it as
// whole sectors: 32 e4m3 codes are one 32-byte sector, 32 bf16 values two.

// slots c[b .. b+3] -> vector order: d[j] = c[b + ((j - rot) & 3)], two selects
// per word (b: the chunk's first slot, a constant after unrolling)
template <int W, int N>
__device__ __forceinline__ void unrotate_chunk(const uint32_t (&c)[N][W], int b, int rot,
                                               uint32_t (&d)[4 * W]) {
  const bool r1 = (rot & 1) != 0, r2 = (rot & 2) != 0;
  uint32_t e[4][W];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int i = 0; i < W; ++i) e[k][i] = r2 ? c[b + ((k + 2) & 3)][i] : c[b + k][i];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < W; ++i) d[W * j + i] = r1 ? e[(j + 3) & 3][i] : e[j][i];
}

// 32 codes of one chunk at p (chunk's first vector index vfirst, row of V
// vectors). a32 / a16: p is 32- / 16-byte aligned.
template <bool FULL>
__device__ __forceinline__ void store_chunk_codes(uint8_t* p, const uint32_t (&d)[8], bool a32,
                                                  bool a16, int vfirst, int V) {
  if (FULL && a32) {
    st_stream8(p, d);
  } else if (FULL && a16) {
    const uint32_t lo[4] = {d[0], d[1], d[2], d[3]}, hi[4] = {d[4], d[5], d[6], d[7]};
    st_stream(p, lo);
    st_stream(p + 16, hi);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) st_stream2_if(FULL || vfirst + j < V, p + 8 * j, d[2 * j], d[2 * j + 1]);
  }
}

// 32 bf16 values of one chunk at p (16-byte aligned; a32: 32-byte aligned)
template <bool FULL>
__device__ __forceinline__ void store_chunk_bf16(uint8_t* p, const uint32_t (&d)[16], bool a32,
                                                 int vfirst, int V) {
  if (FULL && a32) {
    st_stream8(p, d);
    st_stream8(p + 32, d + 8);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t q[4] = {d[4 * j], d[4 * j + 1], d[4 * j + 2], d[4 * j + 3]};
      st_stream_if(FULL || vfirst + j < V, p + 16 * j, q);
    }
  }
}

__device__ __forceinline__ bool aligned_rows(const void* p, int64_t ld_bytes, unsigned n) {
  return ((reinterpret_cast<uint64_t>(p) | (uint64_t)ld_bytes) & (n - 1u)) == 0;
}

// ------------------------------------------------- mbarrier + bulk copies

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// One try_wait: the thread is suspended in hardware until the phase
// completes or about kSuspendHintNs pass, so waiting costs no issue slots.
constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Non-blocking: has phase `parity` of the mbarrier completed?
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for phase `parity` of an mbarrier: one non-blocking test (the phase
// has usually completed), then suspending try_waits while fewer than `limit`
// SM cycles have passed. limit < 0 never blocks: the wait gives up as soon as
// the test finds the phase incomplete (the failure path can be exercised with
// copies that are valid and still land).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long limit) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  while (clock64() - t0 <= limit)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Global -> shared bulk copy (no multicast), completion counted on `bar`.
// Source, destination and size are multiples of 16 bytes.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

constexpr long long kWaitLimitCycles = 4000000000LL;  // default limit: ~2 s at the B200's clocks
constexpr long long kDrainLimitCycles = 400000000LL;  // per stage, after an error

// ------------------------------------------------------------ arithmetic

// RN(a / b) from rc = RN(1/b): q0 = RN(a*rc) is within one ulp of a/b, the
// FMA remainder a - b*q0 is then exact, and one correction step
// RN(q0 + rem*rc) yields the correctly rounded quotient (Markstein's theorem,
// P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990). Valid while the
// quotient is a normal fp32 number; below that the fp8 code is 0 anyway.
// nb = -b, b > 0. The remainder is exact, so its rounding mode only decides
// the sign of an exact zero: rounding down makes it -0, which keeps the sign
// of a zero dividend (-0 / b = -0, as IEEE division gives) and leaves every
// other quotient unchanged.
__device__ __forceinline__ float2 div2_rn(float2 a, float2 nb, float2 rc) {
  const float2 q0 = __fmul2_rn(a, rc);
  const float2 rem = __ffma2_rd(q0, nb, a);
  return __ffma2_rn(rem, rc, q0);
}

// Scalar form of the same division.
__device__ __forceinline__ float div_rn(float a, float b, float rc) {
  const float q0 = __fmul_rn(a, rc);
  const float rem = __fmaf_rd(q0, -b, a);
  return __fmaf_rn(rem, rc, q0);
}

constexpr float kE4m3Max = 448.0f;
constexpr float kRcpE4m3Max = 1.0f / 448.0f;  // RN(1/448), folded by the compiler
constexpr float kMinScale = 1e-4f;            // fp8_utils.py:51 clamp

// s = max(RN(amax / 448), 1e-4) [rounded up to a power of two for POW2/E8M0].
__device__ __forceinline__ float make_scale(float amax, bool pow2) {
  float s = fmaxf(div_rn(amax, kE4m3Max, kRcpE4m3Max), kMinScale);
  if (pow2) {
    // 2^ceil(log2 s), exactly: keep the exponent, bump it if any mantissa bit
    // is set (s >= 1e-4 is a normal number).
    uint32_t u = __float_as_uint(s);
    u = (u & 0x007fffffu) ? (u & 0x7f800000u) + 0x00800000u : u;
    s = __uint_as_float(u);
  }
  return s;
}

// RN(1 / s) for a scale that make_scale produced without the power-of-two
// rounding, by Markstein's reciprocal iteration (P. Markstein, IBM J. Res.
// Dev. 34(1), 1990): y0 = rcp.approx(s), at most 1 ulp from 1/s (PTX ISA);
// e = RN(1 - s*y0); y1 = RN(y0 + e*y0). One step is not correctly rounded for
// every fp32 s, but it is for every scale this path can produce, s =
// max(RN(a / 448), 1e-4) with a a bf16 magnitude (16969 values), from any
// start within 2 ulps of 1/s: tests/test_scale_reciprocal.py checks all of
// them in exact rational arithmetic. Three instructions instead of the
// general correctly rounded reciprocal.
__device__ __forceinline__ float rcp_scale(float s) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
  const float e = __fmaf_rn(-s, y, 1.0f);
  return __fmaf_rn(e, y, y);
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
    const int64_t off = row * a.s_row + (int64_t)(g >> 2) * a.s_grp4 + (int64_t)(g & 3) * a.s_grp;
    if (a.scale_fmt == kFmtE8M0)
      static_cast<uint8_t*>(a.scale)[off] = e8;
    else
      static_cast<float*>(a.scale)[off] = s;
  }
}

__device__ __forceinline__ void zero_scale_padding(const FusedArgs& a, int64_t row, int g0,
                                                   int t, int T) {
  for (int g = g0 + t; g < a.n_groups_pad; g += T)
    static_cast<uint8_t*>(a.scale)[swizzled_offset(row, g, a.n_groups_pad >> 2)] = 0;
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

// Second half of a block reduction: every warp combines the per-warp
// partials in `buf` with the same butterfly, so every thread gets the same bits.
template <bool kMax>
__device__ __forceinline__ float combine_partials(const float* buf, int lane, int nw) {
  return warp_reduce<kMax>(lane < nw ? buf[lane] : 0.0f);  // 0: neutral for sums and |max|
}

// Block-wide reduction; `buf` alternates between two 32-float slots so one
// barrier per reduction suffices.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* buf, int lane, int warp, int nw) {
  v = warp_reduce<kMax>(v);
  if (nw > 1) {
    if (lane == 0) buf[warp] = v;
    __syncthreads();
    v = combine_partials<kMax>(buf, lane, nw);
  }
  return v;
}

// ------------------------------------------------------------ the kernel

// Max magnitude of 8 elements as a bf16 pair (two partial maxima).
__device__ __forceinline__ uint32_t vec_absmax(const uint32_t (&v)[4]) {
  return absmax_bf2(absmax_bf2(v[0], v[1]), absmax_bf2(v[2], v[3]));
}

// Scale store of one group. The destination kind is fixed for a launch:
// fp32 strided, e8m0 strided or e8m0 swizzled.
__device__ __forceinline__ void put_scale(const FusedArgs& a, int64_t row, char* srow, int g,
                                          float s) {
  if (a.scale_layout == kLaySwizzled) {
    static_cast<uint8_t*>(a.scale)[swizzled_offset(row, g, a.n_groups_pad >> 2)] =
        (uint8_t)(__float_as_uint(s) >> 23);
  } else {
    const int64_t off = (int64_t)(g >> 2) * a.s_grp4 + (int64_t)(g & 3) * a.s_grp;
    if (a.scale_fmt == kFmtE8M0)
      srow[off] = (char)(__float_as_uint(s) >> 23);
    else
      reinterpret_cast<float*>(srow)[off] = s;
  }
}

// NCH: 64-byte chunks per thread. QM: quantization mode. LPG: lanes per
// group in group mode (G/32). RES: add the residual first. NORM: apply
// RMSNorm (false = quantize x as is, the per_token_cast_to_fp8 path).
// FULL: every thread's chunks lie wholly inside the row (T * NCH * 4 == V),
// so no store needs a bounds predicate.
//
// Dynamic shared memory: `a.stages` stages of [x row | residual row], each
// row buffer = the row rounded up to whole 64-byte chunks plus one more
// 64-byte chunk; everything past the copied bytes is zeroed once and never
// written by the copies. Vectors past the row end read that zero pad (the
// partial last chunk reads it in place, chunks wholly past the end read the
// extra chunk), so every shared-memory read is in bounds and unpredicated.
// One mbarrier per stage follows the ring.
//
// Per row: wait for the stage; read it; [residual add]; sum of squares;
// barrier 1 (also releases the stage for its refill and votes on failed
// waits); warp 0 turns the per-warp partial sums into inv_rms; barrier 2
// publishes it; normalise; group maxima; scales; FP8 codes. The weights are
// re-read from L1 each row instead of being held in registers, which keeps
// the kernel small enough for 40+ resident warps per SM.
template <int NCH, int QM, int LPG, bool RES, bool NORM, bool FULL>
__global__ void __launch_bounds__(NCH == 1 ? 1024 : 512) fused_rmsnorm_fp8_kernel(const FusedArgs a) {
  static_assert(QM != kQGroup || LPG == 1 || LPG == 2 || LPG == 4, "lanes per group");
  static_assert(NORM || !RES, "residual needs the norm");
  constexpr int NV = 4 * NCH;  // vectors per thread
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[2][32];
  __shared__ float inv_slot[2];

  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int S = a.stages;
  const uint32_t row_bytes = (uint32_t)a.V * 16u;           // bytes copied per row
  const uint32_t row_chunks = (row_bytes + 63u) & ~63u;      // whole chunks
  const uint32_t row_pad = row_chunks + 64u;                 // + one zero chunk
  const uint32_t stage_bytes = RES ? 2u * row_pad : row_pad;
  const uint32_t ring = smem_addr(smem);
  const uint32_t bars = ring + (uint32_t)S * stage_bytes;
  const int64_t G = gridDim.x;

  // Byte offset (within a row) of this thread's k-th 16-byte vector, and
  // whether it lies inside the row. Vector j of a chunk is visited at
  // position (j + rot) & 3 (bank spreading, see above).
  const int rot = (t >> 1) & 3;
  uint32_t voff[NV];
  bool vok[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int ci = (k >> 2) * T + t;  // chunk index in the row
    const int j = ((k & 3) + rot) & 3;
    const int vi = ci * 4 + j;
    vok[k] = FULL || vi < a.V;
    voff[k] = FULL || (uint32_t)ci * 64u < row_chunks ? (uint32_t)vi * 16u
                                                       : row_chunks + 16u * (uint32_t)j;
  }

  auto issue = [&](int s, int64_t row) {
    const uint32_t bar = bars + 8u * (uint32_t)s;
    const uint32_t dst = ring + (uint32_t)s * stage_bytes;
    mbar_arrive_expect_tx(bar, RES ? 2u * row_bytes : row_bytes);
    bulk_g2s(dst, a.x + row * a.ldx, row_bytes, bar);
    if constexpr (RES) bulk_g2s(dst + row_pad, a.res + row * a.ldr, row_bytes, bar);
  };

  // zero the pad of every row buffer once
  for (int s = 0; s < S * (RES ? 2 : 1); ++s)
    for (uint32_t b = row_bytes + 4u * (uint32_t)t; b < row_pad; b += 4u * (uint32_t)T)
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(ring + (uint32_t)s * row_pad + b), "r"(0u)
                   : "memory");
  if (t == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bars + 8u * (uint32_t)s, 1);
    mbar_init_fence();
  }
  __syncthreads();
  griddep_wait();  // inputs of the previous kernel are complete from here on
  griddep_launch_dependents();
  if (t == 0)
    for (int s = 0; s < S; ++s) {
      const int64_t row = blockIdx.x + (int64_t)s * G;
      if (row < a.M) issue(s, row);
    }

  const bool pow2 = a.scale_fmt != kFmtF32;
  const bool store_ro = RES && a.res_out != nullptr;
  const bool store_no = NORM && a.norm_out != nullptr;
  // output rows on 32- / 16-byte boundaries take whole-sector stores
  const bool q32 = aligned_rows(a.q, a.ldq, 32), q16 = aligned_rows(a.q, a.ldq, 16);
  const bool ro32 = aligned_rows(a.res_out, a.ldro * 2, 32);
  const bool no32 = aligned_rows(a.norm_out, a.ldn * 2, 32);
  // Row pointers advance by G rows per iteration.
  const int esz = a.scale_fmt == kFmtE8M0 ? 1 : 4;
  uint8_t* qrow = a.q + (int64_t)blockIdx.x * a.ldq;
  char* srow = static_cast<char*>(a.scale) + (int64_t)blockIdx.x * a.s_row * esz;
  uint8_t* norow = reinterpret_cast<uint8_t*>(a.norm_out) + (int64_t)blockIdx.x * a.ldn * 2;
  uint8_t* rorow = reinterpret_cast<uint8_t*>(a.res_out) + (int64_t)blockIdx.x * a.ldro * 2;
  const int64_t q_step = G * a.ldq, s_step = G * a.s_row * esz, n_step = G * a.ldn * 2,
                r_step = G * a.ldro * 2;
  // Chunks past the row end hold zeros and still take part in the shuffles;
  // only the leader lane of a group inside the row writes its scale.
  const bool chunk_ok0 = FULL || (int64_t)t * 4 < a.V;
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(a.w);

  int flip = 0;
  int s = 0;
  uint32_t parity = 0;
  for (int64_t row = blockIdx.x; row < a.M_pad;
       row += G, qrow += q_step, srow += s_step, norow += n_step, rorow += r_step) {
    if (row >= a.M) {  // swizzled-layout padding row: scales only
      zero_scale_padding(a, row, 0, t, T);
      continue;
    }
    const uint32_t bar = bars + 8u * (uint32_t)s;
    const uint32_t base = ring + (uint32_t)s * stage_bytes;
    int bad = mbar_wait_bounded(bar, parity, a.wait_limit) ? 0 : 1;

    uint32_t v[NV][4];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const uint4 u = ld_smem(base + voff[k]);
      v[k][0] = u.x;
      v[k][1] = u.y;
      v[k][2] = u.z;
      v[k][3] = u.w;
    }
    if constexpr (RES) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const uint4 u = ld_smem(base + row_pad + voff[k]);
        const uint32_t r[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[k][j] = f2_to_bf2(__fadd2_rn(bf2_to_f2(v[k][j]), bf2_to_f2(r[j])));
      }
      if (store_ro) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t d[16];
          unrotate_chunk(v, 4 * c, rot, d);
          const int ch = c * T + t;
          store_chunk_bf16<FULL>(rorow + 64 * ch, d, ro32, 4 * ch, a.V);
        }
      }
    }

    float inv = 0.0f, ss = 0.0f;
    if constexpr (NORM) {
      // Squares of bf16 values are exact in fp32, so fma == mul-then-add.
      // One accumulator pair per vector keeps the dependency chains short.
      float2 acc[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const float2 f0 = bf2_to_f2(v[k][0]);
        acc[k] = __fmul2_rn(f0, f0);
#pragma unroll
        for (int j = 1; j < 4; ++j) {
          const float2 f = bf2_to_f2(v[k][j]);
          acc[k] = __ffma2_rn(f, f, acc[k]);
        }
      }
#pragma unroll
      for (int k = 1; k < NV; ++k) acc[0] = __fadd2_rn(acc[0], acc[k]);
      ss = warp_reduce<false>(__fadd_rn(acc[0].x, acc[0].y));  // every lane: the warp's sum
      if (lane == 0) red[flip][warp] = ss;
    }
    // Barrier 1: every thread has read the stage, so thread 0 may refill
    // it; the barrier also votes on failed waits.
    if (nw > 1)
      bad = __syncthreads_or(bad);
    else
      bad = __any_sync(0xffffffffu, bad);
    if (bad) {
      // A copy never completed: report it, let every stage that still has a
      // copy in flight finish (bounded), and leave.
      if (t == 0) {
        atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
        for (int k = 0; k < S; ++k) {
          const int64_t pending = row + (int64_t)k * G;
          if (pending >= a.M) break;
          const int ps = (s + k) % S;
          const uint32_t pp = parity ^ (uint32_t)((s + k) / S);
          mbar_wait_bounded(bars + 8u * (uint32_t)ps, pp & 1u, kDrainLimitCycles);
        }
      }
      return;
    }
    if (t == 0) {
      const int64_t next = row + (int64_t)S * G;
      if (next < a.M) issue(s, next);
    }
    if (++s == S) {
      s = 0;
      parity ^= 1u;
    }

    if constexpr (NORM) {
      // Weights for this row from L1 (issued before the finalisation so the
      // loads overlap it).
      uint32_t w[NV][4];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (FULL || vok[k]) u = ld_keep(wbase + voff[k]);
        w[k][0] = u.x;
        w[k][1] = u.y;
        w[k][2] = u.z;
        w[k][3] = u.w;
      }
      if (nw > 1) {
        // Warp 0 combines the partials and computes inv_rms; barrier 2
        // publishes it. torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))), not a
        // correctly rounded reciprocal square root; the double rounding is
        // reproduced. The mean is RN(ss / H) through the one-correction
        // division (a quotient below the normal range takes the IEEE one).
        if (warp == 0) {
          const float total = combine_partials<false>(red[flip], lane, nw);
          float mean = div_rn(total, (float)a.H, a.rcp_H);
          if (mean < 0x1p-100f) mean = __fdiv_rn(total, (float)a.H);
          if (lane == 0) inv_slot[flip] = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
        }
        __syncthreads();
        inv = inv_slot[flip];
      } else {  // one warp: the butterfly already left the row sum in every lane
        float mean = div_rn(ss, (float)a.H, a.rcp_H);
        if (mean < 0x1p-100f) mean = __fdiv_rn(ss, (float)a.H);
        inv = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
      }
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int k = 0; k < NV; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[k][j] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[k][j]), inv2)), w[k][j]);
      if (store_no) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t d[16];
          unrotate_chunk(v, 4 * c, rot, d);
          const int ch = c * T + t;
          store_chunk_bf16<FULL>(norow + 64 * ch, d, no32, 4 * ch, a.V);
        }
      }
    }
    flip ^= 1;

    if constexpr (QM != kQNone) {
      float sc[NCH], rc[NCH];
      if constexpr (QM == kQGroup) {
        // Chunk maxima; with LPG > 1 the lanes of a group combine by shuffles
        // (two chunks share one bf16 pair per shuffle).
        uint32_t m2[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const uint32_t p = absmax_bf2(absmax_bf2(vec_absmax(v[4 * c]), vec_absmax(v[4 * c + 1])),
                                        absmax_bf2(vec_absmax(v[4 * c + 2]), vec_absmax(v[4 * c + 3])));
          m2[c] = p & 0x7fff7fffu;
        }
        float m[NCH];
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          uint32_t p;
          if (c + 1 < NCH)
            p = max_bf2(__byte_perm(m2[c], m2[c + 1], 0x5410), __byte_perm(m2[c], m2[c + 1], 0x7632));
          else
            p = max_bf2(m2[c], m2[c] >> 16);
#pragma unroll
          for (int o = LPG / 2; o > 0; o >>= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
          m[c] = __uint_as_float(p << 16);
          if (c + 1 < NCH) m[c + 1] = __uint_as_float(p & 0xffff0000u);
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          sc[c] = make_scale(m[c], pow2);
          // a power-of-two scale has an exact reciprocal: negate the exponent
          rc[c] = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sc[c])) : rcp_scale(sc[c]);
          const int ch = c * T + t;  // chunk index in the row
          if ((t & (LPG - 1)) == 0 && (c == 0 ? chunk_ok0 : (FULL || ch * 4 < a.V)))
            put_scale(a, row, srow, ch / LPG, sc[c]);
        }
        if (a.scale_layout == kLaySwizzled && a.n_groups_pad > a.n_groups)
          zero_scale_padding(a, row, a.n_groups, t, T);
      } else {  // one scale per row
        uint32_t p = 0u;
#pragma unroll
        for (int k = 0; k < NV; ++k) p = absmax_bf2(p, vec_absmax(v[k]));
        p &= 0x7fff7fffu;
        float m = warp_reduce<true>(fmaxf(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u)));
        if (nw > 1) {
          if (lane == 0) red[flip][warp] = m;
          __syncthreads();
          m = combine_partials<true>(red[flip], lane, nw);
          flip ^= 1;
        }
        const float s1 = make_scale(m, pow2);
        const float r1 = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(s1)) : rcp_scale(s1);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          sc[c] = s1;
          rc[c] = r1;
        }
        if (t == 0) store_scale(a, row, 0, s1);
      }
      uint32_t cw[NV][2];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const float2 rc2 = make_float2(rc[k >> 2], rc[k >> 2]);
        float2 y[4];
        if (pow2) {  // power-of-two scale: n * (1/s) is exact
#pragma unroll
          for (int j = 0; j < 4; ++j) y[j] = __fmul2_rn(bf2_to_f2(v[k][j]), rc2);
        } else {
          const float2 nb = make_float2(-sc[k >> 2], -sc[k >> 2]);
#pragma unroll
          for (int j = 0; j < 4; ++j) y[j] = div2_rn(bf2_to_f2(v[k][j]), nb, rc2);
        }
        cw[k][0] = f4_to_e4m3x4(y[0], y[1]);
        cw[k][1] = f4_to_e4m3x4(y[2], y[3]);
      }
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint32_t d[8];
        unrotate_chunk(cw, 4 * c, rot, d);
        const int ch = c * T + t;
        store_chunk_codes<FULL>(qrow + 32 * ch, d, q32, q16, 4 * ch, a.V);
      }
    }
  }
}

// ------------------------------------------------ one warp per row, two passes

// residual add of one chunk, rounding exactly as the single-pass kernel does
__device__ __forceinline__ void add_chunk(uint32_t (&v)[4][4], const uint32_t (&r)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) v[j][i] = f2_to_bf2(__fadd2_rn(bf2_to_f2(v[j][i]), bf2_to_f2(r[j][i])));
}

__device__ __forceinline__ void norm_chunk(uint32_t (&v)[4][4], const uint32_t (&w)[4][4],
                                           float2 inv2) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) v[j][i] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[j][i]), inv2)), w[j][i]);
}

__device__ __forceinline__ uint32_t chunk_absmax(const uint32_t (&v)[4][4]) {
  return absmax_bf2(absmax_bf2(vec_absmax(v[0]), vec_absmax(v[1])),
                    absmax_bf2(vec_absmax(v[2]), vec_absmax(v[3]))) &
         0x7fff7fffu;
}

// Large batches: each warp owns whole rows (grid-stride over rows). A row is
// read in pieces of 2 KB (32 chunks of 64 bytes, one per lane); the warp's
// lane 0 streams pieces into a private ring of `a.stages` shared-memory
// slots with cp.async.bulk (x and, with RES, the residual piece beside it),
// running `stages` pieces ahead of the lanes across piece, pass and row
// boundaries. Pass 1 reads the row for the sum of squares (adding the
// residual and writing residual_out on the way); pass 2 streams it again
// (from L2) to normalise, take group maxima (1x128 = 4 lanes) and write the
// codes; per-token scaling streams a third pass once the row maximum is
// known. Rows need no block barrier: the row reduction is one warp
// butterfly, and the per-row scalar work is spread over 224 elements a lane
// at H = 7168. Inputs must not alias outputs (the host routes in-place calls
// to the single-pass kernel). FULL: V % 128 == 0 (whole pieces), so no read
// or store needs a bounds predicate.
//
// Dynamic shared memory: per warp `stages` slots of (RES ? 4096 : 2048)
// bytes, then per warp `stages` mbarriers.
constexpr int kRowwarpWarps = 4;            // warps per CTA
constexpr uint32_t kPieceBytes = 2048;      // 32 lanes x 64 bytes

template <int QM, int LPG, bool RES, bool NORM, bool FULL>
__global__ void __launch_bounds__(kRowwarpWarps * 32, RES ? 6 : 8)
    rowwarp_rmsnorm_fp8_kernel(const FusedArgs a) {
  static_assert(QM != kQGroup || LPG == 1 || LPG == 2 || LPG == 4, "lanes per group");
  static_assert(NORM || !RES, "residual needs the norm");
  constexpr int NPASS = (QM == kQToken ? 2 : 1) + (NORM ? 1 : 0);  // stream passes per row
  constexpr uint32_t kSlot = RES ? 2 * kPieceBytes : kPieceBytes;
  extern __shared__ __align__(128) uint8_t smem[];

  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;  // warp in block
  const int64_t nwarp = (int64_t)gridDim.x * kRowwarpWarps;
  const int64_t wid = (int64_t)blockIdx.x * kRowwarpWarps + wib;
  const int P = a.stages;
  const uint32_t ring = smem_addr(smem) + (uint32_t)wib * (uint32_t)P * kSlot;
  const uint32_t bars = smem_addr(smem) + (uint32_t)(kRowwarpWarps * P) * kSlot +
                        8u * (uint32_t)(wib * P);
  const int V = a.V;
  const uint32_t row_bytes = (uint32_t)V * 16u;
  const int np = (int)((row_bytes + kPieceBytes - 1) / kPieceBytes);  // pieces per row
  const int64_t my_rows = wid < a.M ? (a.M - 1 - wid) / nwarp + 1 : 0;
  const int64_t total = my_rows * NPASS * np;  // stream positions of this warp
  const bool pow2 = a.scale_fmt != kFmtF32;
  const int esz = a.scale_fmt == kFmtE8M0 ? 1 : 4;
  const bool store_ro = RES && a.res_out != nullptr;
  const bool store_no = NORM && a.norm_out != nullptr;
  const uint8_t* wrow = reinterpret_cast<const uint8_t*>(a.w);
  // lane's chunk within a piece, vector j visited at (j + rot) & 3
  const int rot = (lane >> 1) & 3;
  uint32_t loff[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) loff[k] = 64u * (uint32_t)lane + 16u * (uint32_t)((k + rot) & 3);

  // Producer state (lane 0): next stream position to issue, as (row, pass,
  // piece) and ring slot, advanced one step per issue.
  int64_t iss = 0, iss_row = wid;
  int iss_pass = 0, iss_piece = 0, iss_slot = 0;
  auto issue_next = [&]() {
    const uint32_t slot = (uint32_t)iss_slot;
    const uint32_t bar = bars + 8u * slot;
    const uint32_t dst = ring + slot * kSlot;
    const uint32_t off = (uint32_t)iss_piece * kPieceBytes;
    const uint32_t n = row_bytes - off < kPieceBytes ? row_bytes - off : kPieceBytes;
    mbar_arrive_expect_tx(bar, RES ? 2u * n : n);
    bulk_g2s(dst, reinterpret_cast<const uint8_t*>(a.x) + iss_row * a.ldx * 2 + off, n, bar);
    if constexpr (RES)
      bulk_g2s(dst + kPieceBytes, reinterpret_cast<const uint8_t*>(a.res) + iss_row * a.ldr * 2 + off,
               n, bar);
    ++iss;
    if (++iss_slot == P) iss_slot = 0;
    if (++iss_piece == np) {
      iss_piece = 0;
      if (++iss_pass == NPASS) {
        iss_pass = 0;
        iss_row += nwarp;
      }
    }
  };

  if (lane == 0) {
    for (int k = 0; k < P; ++k) mbar_init(bars + 8u * (uint32_t)k, 1);
    mbar_init_fence();
  }
  __syncwarp();
  griddep_wait();  // inputs of the previous kernel are complete from here on
  griddep_launch_dependents();
  if (lane == 0)
    while (iss < total && iss < P) issue_next();

  // Consumer: wait for stream position `pos`, read this lane's chunk (x and
  // residual) into registers, release the slot and refill it. Returns false
  // (for the whole warp) if the copy never arrived.
  int64_t pos = 0;
  int pos_slot = 0;
  uint32_t pos_par = 0;
  auto take = [&](uint32_t (&x)[4][4], uint32_t (&r)[4][4], int piece) -> bool {
    const uint32_t slot = (uint32_t)pos_slot;
    const bool ok = mbar_wait_bounded(bars + 8u * slot, pos_par, a.wait_limit);
    const uint32_t base = ring + slot * kSlot;
    const int c = piece * 32 + lane;  // chunk index in the row
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const bool in = FULL || c * 4 + ((k + rot) & 3) < V;
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (in) u = ld_smem(base + loff[k]);
      x[k][0] = u.x; x[k][1] = u.y; x[k][2] = u.z; x[k][3] = u.w;
      if constexpr (RES) {
        uint4 q = make_uint4(0u, 0u, 0u, 0u);
        if (in) q = ld_smem(base + kPieceBytes + loff[k]);
        r[k][0] = q.x; r[k][1] = q.y; r[k][2] = q.z; r[k][3] = q.w;
      }
    }
    const bool all_ok = __all_sync(0xffffffffu, ok);
    __syncwarp();  // every lane's reads of the slot are ordered before its refill
    ++pos;
    if (++pos_slot == P) {
      pos_slot = 0;
      pos_par ^= 1u;
    }
    if (all_ok && lane == 0 && iss < total) issue_next();
    return all_ok;
  };

  auto fail = [&]() {
    // A copy never completed: report it, let the copies in flight finish
    // (bounded), and stop this warp.
    if (lane == 0) {
      atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
      for (int64_t q = pos > 0 ? pos - 1 : 0; q < iss; ++q)
        mbar_wait_bounded(bars + 8u * (uint32_t)(q % P), (uint32_t)((q / P) & 1), kDrainLimitCycles);
    }
  };

  // byte offset of vector k of this lane's chunk within the row / piece
  auto voff = [&](int piece, int k) -> uint32_t {
    return (uint32_t)piece * kPieceBytes + loff[k];
  };
  auto vin = [&](int piece, int k) -> bool {
    return FULL || (piece * 32 + lane) * 4 + ((k + rot) & 3) < V;
  };

  int64_t row = wid;
  for (int64_t kr = 0; kr < my_rows; ++kr, row += nwarp) {
    uint8_t* ror = RES ? reinterpret_cast<uint8_t*>(a.res_out) + row * a.ldro * 2 : nullptr;
    uint8_t* nor = reinterpret_cast<uint8_t*>(a.norm_out) + row * a.ldn * 2;
    uint8_t* qr = a.q + row * a.ldq;
    char* srow = static_cast<char*>(a.scale) + row * a.s_row * esz;
    uint32_t v[4][4], r[4][4];

    // ---- pass 1: sum of squares (residual add and residual_out on the way)
    float2 inv2 = make_float2(0.0f, 0.0f);
    if constexpr (NORM) {
      float2 acc = make_float2(0.0f, 0.0f);
      for (int pc = 0; pc < np; ++pc) {
        if (!take(v, r, pc)) return fail();
        if constexpr (RES) {
          add_chunk(v, r);
          if (store_ro) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (FULL) st_stream(ror + voff(pc, k), v[k]);
              else st_stream_if(vin(pc, k), ror + voff(pc, k), v[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = bf2_to_f2(v[k][j]);
            acc = __ffma2_rn(f, f, acc);
          }
      }
      const float ss = warp_reduce<false>(__fadd_rn(acc.x, acc.y));
      // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))); the mean is RN(ss / H)
      float mean = div_rn(ss, (float)a.H, a.rcp_H);
      if (mean < 0x1p-100f) mean = __fdiv_rn(ss, (float)a.H);
      const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
      inv2 = make_float2(inv, inv);
    }

    // normalised values of the lane's chunk in piece pc, from a fresh take
    auto normalized = [&](int pc) -> bool {
      if (!take(v, r, pc)) return false;
      if constexpr (RES) add_chunk(v, r);
      if constexpr (NORM) {
        uint32_t w[4][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 u = make_uint4(0u, 0u, 0u, 0u);
          if (vin(pc, k)) u = ld_keep(wrow + voff(pc, k));
          w[k][0] = u.x; w[k][1] = u.y; w[k][2] = u.z; w[k][3] = u.w;
        }
        norm_chunk(v, w, inv2);
      }
      return true;
    };
    auto store_norm = [&](int pc) {
      if (!store_no) return;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (FULL) st_stream(nor + voff(pc, k), v[k]);
        else st_stream_if(vin(pc, k), nor + voff(pc, k), v[k]);
    };
    auto store_codes = [&](int pc, float sc, float rc) {
      const float2 rc2 = make_float2(rc, rc), nb = make_float2(-sc, -sc);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 y[4];
        if (pow2) {
#pragma unroll
          for (int j = 0; j < 4; ++j) y[j] = __fmul2_rn(bf2_to_f2(v[k][j]), rc2);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) y[j] = div2_rn(bf2_to_f2(v[k][j]), nb, rc2);
        }
        const uint32_t c0 = f4_to_e4m3x4(y[0], y[1]), c1 = f4_to_e4m3x4(y[2], y[3]);
        uint8_t* p = qr + (voff(pc, k) >> 1);
        if (FULL) st_stream2(p, c0, c1);
        else st_stream2_if(vin(pc, k), p, c0, c1);
      }
    };

    if constexpr (QM == kQGroup) {
      // ---- pass 2: normalise, group maxima, scales, codes
      for (int pc = 0; pc < np; ++pc) {
        if (!normalized(pc)) return fail();
        store_norm(pc);
        uint32_t p = chunk_absmax(v);
        p = max_bf2(p, p >> 16);
#pragma unroll
        for (int o = LPG / 2; o > 0; o >>= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
        const float sc = make_scale(__uint_as_float(p << 16), pow2);
        const float rc = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sc)) : rcp_scale(sc);
        const int c = pc * 32 + lane;
        if ((lane & (LPG - 1)) == 0 && (FULL || c * 4 < V)) put_scale(a, row, srow, c / LPG, sc);
        store_codes(pc, sc, rc);
      }
      if (a.scale_layout == kLaySwizzled && a.n_groups_pad > a.n_groups)
        zero_scale_padding(a, row, a.n_groups, lane, 32);
    } else if constexpr (QM == kQToken) {
      // ---- pass 2: normalise (+ normalized_out) and the row maximum
      uint32_t pm = 0u;
      for (int pc = 0; pc < np; ++pc) {
        if (!normalized(pc)) return fail();
        store_norm(pc);
        pm = max_bf2(pm, chunk_absmax(v));
      }
      const float m = warp_reduce<true>(fmaxf(__uint_as_float(pm << 16), __uint_as_float(pm & 0xffff0000u)));
      const float sc = make_scale(m, pow2);
      const float rc = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sc)) : rcp_scale(sc);
      if (lane == 0) store_scale(a, row, 0, sc);
      // ---- pass 3: codes (normalised values recomputed: same bits)
      for (int pc = 0; pc < np; ++pc) {
        if (!normalized(pc)) return fail();
        store_codes(pc, sc, rc);
      }
    } else {
      // ---- pass 2: plain RMSNorm output
      for (int pc = 0; pc < np; ++pc) {
        if (!normalized(pc)) return fail();
        store_norm(pc);
      }
    }
  }
  // swizzled-layout padding rows: scales only
  for (; row < a.M_pad; row += nwarp)
    if (row >= a.M) zero_scale_padding(a, row, 0, lane, 32);
}

// Host-side launch shape.
struct LaunchShape {
  int nch;        // single-pass kernel: 64-byte chunks per thread, 1 or 2
  int threads;    // single-pass kernel: threads per CTA (one row at a time)
  bool rowwarp;   // use the warp-per-row two-pass kernel instead
  bool pipe;      // nch == 1: prefer the pipelined kernel (pipe_kernel.cuh) where it applies
  bool rowstage;  // automatic shape: prefer the row-staged kernel (rowstage_kernel.cuh)
};

}  // namespace cutie
