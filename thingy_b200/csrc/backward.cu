// Backward of the fused [residual add] -> RMSNorm path, with optional FP8
// quantization of the input gradient, for sm_100a.
//
// The reference has no backward pass. What is computed is what torch
// autograd computes for the reference's forward (src/cutie/rms_norm/bench.py:
// 58-65 and the residual add of :97), op for op in fp32. Per row, with r the
// RMSNorm input (x + residual), dn the gradient of the bf16 normalized output
// and dro the gradient of residual_out:
//
//   inv  = RN(1 / RN(sqrt(RN(sum r^2) / H + eps)))     (the forward's value)
//   dt   = bf16(dn * w)                                  (bf16 mul backward)
//   b    = sum dt * r                                    (fp32)
//   dvar = (-0.5 * b) * ((inv * inv) * inv)              (rsqrt backward)
//   dsq  = dvar / H                                      (mean backward)
//   dx   = bf16(dt * inv + dsq * (2 * r))                (mul + square backward)
//   dr   = bf16(dx + dro)                                (gradient accumulation)
//   dw  += bf16(dn * bf16(r * inv))  over rows           (fp32 sums)
//
// dr is the gradient of x and of residual. Both row sums (sum r^2 and
// sum dt * r) take one block reduction of a float pair. The weight gradient
// is summed per CTA in shared memory, written as one fp32 row of partial
// sums per CTA to a caller-provided workspace, and reduced over CTAs in a
// fixed order by a second kernel, so it is deterministic.
//
// Thread layout: the interleaved layout of the pipelined forward kernel (lane
// i of octet o of warp w holds vectors w*128 + o*32 + i + 8k), read directly
// from global memory: an octet reads 128 contiguous bytes per slot, and an
// octet covers two whole 1x128 groups, so the optional quantization of dr is
// the forward's two-groups-an-octet scheme.
#include "launch.cuh"


namespace cutie {

// Scratch of cutie_rms_norm_backward_noalloc, the entry point for callers
// that cannot allocate device memory (include/cutie.h says which): the
// per-CTA partial sums of d_weight go to this file-scope array instead of a
// caller-provided workspace. kNoAllocScratchFloats floats (4 MiB) on every GPU
// that loads the library, held until the process exits. Host code cannot use
// the array's name as a device address (it names a host-side stand-in);
// noalloc_scratch() resolves the device address.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch in the calling thread's current
// context, resolved on every call. Once the library's module is loaded in a
// context the lookup is a host-side table read (the first call in a context
// loads the module there). An address kept from an earlier call could be
// stale: after cudaDeviceReset the module is loaded again in a new primary
// context, and a caller that makes another driver context current on the
// same device sees that context's copy of the array; a kernel given the old
// address would write through it.
cudaError_t noalloc_scratch(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<float*>(p);
  return cudaSuccess;
}

// This translation unit's device error word (set by a ring wait that gave up).
cudaError_t device_error_bwd(int* out, bool clear) { return read_device_error(out, clear); }

__device__ __forceinline__ void st_bf16x8(void* p, const uint32_t (&v)[4], bool ok) {
  st_stream_if(ok, p, v);
}

// The direct kernel serves rows wider than 16384 (more than 512 threads;
// the ring kernel below takes the rest). MAXT: the largest block of the
// instantiation; 1024 caps the registers at 64 a thread.
template <bool RES, bool QUANT, bool DW, bool FULL, int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 256 ? 2 : 1)
    rmsnorm_backward_kernel(const BwdArgs a, float eps, float rcp_H) {
  constexpr int NV = 4;
  extern __shared__ __align__(16) float wacc[];  // [V * 8] partial dw of this CTA
  __shared__ float2 red[2][32];

  const FusedArgs& qa = a.qa;
  const int T = blockDim.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int V = qa.V;
  const int tvec = warp * 128 + (lane >> 3) * 32 + (lane & 7);
  bool vok[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) vok[k] = FULL || tvec + 8 * k < V;

  if (DW)
    for (int i = t; i < V * 8; i += T) wacc[i] = 0.0f;
  // weights: the same columns for every row
  griddep_wait();  // inputs of the previous kernel are complete from here on
  uint32_t w[NV][4];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (vok[k]) u = ld_keep(a.w + (int64_t)(tvec + 8 * k) * 8);
    w[k][0] = u.x;
    w[k][1] = u.y;
    w[k][2] = u.z;
    w[k][3] = u.w;
  }
  griddep_launch_dependents();
  __syncthreads();

  // this thread's quantization group and whether it writes its scale (lanes
  // 0 and 1 of an octet, for the octet's two groups)
  const int gidx = warp * 8 + (lane >> 3) * 2 + (lane & 1);
  const bool gput = (lane & 6) == 0 && (FULL || gidx * 16 < V);
  const int64_t goff = ((int64_t)(gidx >> 2) * qa.s_grp4 + (int64_t)(gidx & 3) * qa.s_grp) *
                       ((qa.scale_fmt == kFmtE8M0) ? 1 : 4);
  int flip = 0;

  for (int64_t row = blockIdx.x; row < qa.M; row += gridDim.x) {
    const uint16_t* rrow = a.r + row * a.ldr;
    const uint16_t* drow = a.dn + row * a.lddn;
    uint32_t rv[NV][4], dv[NV][4];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      uint4 u = make_uint4(0u, 0u, 0u, 0u), e = make_uint4(0u, 0u, 0u, 0u);
      if (vok[k]) {
        u = ld_stream(rrow + (int64_t)(tvec + 8 * k) * 8);
        e = ld_stream(drow + (int64_t)(tvec + 8 * k) * 8);
      }
      rv[k][0] = u.x; rv[k][1] = u.y; rv[k][2] = u.z; rv[k][3] = u.w;
      dv[k][0] = e.x; dv[k][1] = e.y; dv[k][2] = e.z; dv[k][3] = e.w;
    }
    // (sum r^2, sum dt * r): squares per pair in the forward's order, then
    // the products; one butterfly on the pair of sums
    float2 sq = make_float2(0.0f, 0.0f), pr = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = bf2_to_f2(rv[k][j]);
        const float2 dt = bf2_to_f2(mul_bf2(dv[k][j], w[k][j]));
        sq = __ffma2_rn(rf, rf, sq);
        pr = __ffma2_rn(dt, rf, pr);
      }
    float2 s2 = make_float2(__fadd_rn(sq.x, sq.y), __fadd_rn(pr.x, pr.y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s2.x = __fadd_rn(s2.x, __shfl_xor_sync(0xffffffffu, s2.x, o));
      s2.y = __fadd_rn(s2.y, __shfl_xor_sync(0xffffffffu, s2.y, o));
    }
    if (lane == 0) red[flip][warp] = s2;
    __syncthreads();
    float2 tot = lane < nw ? red[flip][lane] : make_float2(0.0f, 0.0f);
    flip ^= 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot.x = __fadd_rn(tot.x, __shfl_xor_sync(0xffffffffu, tot.x, o));
      tot.y = __fadd_rn(tot.y, __shfl_xor_sync(0xffffffffu, tot.y, o));
    }
    float mean = div_rn(tot.x, (float)qa.H, rcp_H);
    if (mean < 0x1p-100f) mean = __fdiv_rn(tot.x, (float)qa.H);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
    const float dvar = __fmul_rn(__fmul_rn(-0.5f, tot.y), __fmul_rn(__fmul_rn(inv, inv), inv));
    const float dsq = __fdiv_rn(dvar, (float)qa.H);
    const float2 inv2 = make_float2(inv, inv), dsq2 = make_float2(dsq, dsq);

    uint16_t* xrow = a.dx + row * a.lddx;
    const uint16_t* grow = RES ? a.dro + row * a.lddro : nullptr;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      uint4 g = make_uint4(0u, 0u, 0u, 0u);
      if (RES && vok[k]) g = ld_stream(grow + (int64_t)(tvec + 8 * k) * 8);
      const uint32_t gg[4] = {g.x, g.y, g.z, g.w};
      float* acc = wacc + (tvec + 8 * k) * 8;
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
      if (DW && vok[k]) {
        a0 = *reinterpret_cast<float4*>(acc);
        a1 = *reinterpret_cast<float4*>(acc + 4);
      }
      float2 accp[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w),
                        make_float2(a1.x, a1.y), make_float2(a1.z, a1.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = bf2_to_f2(rv[k][j]);
        const float2 dt = bf2_to_f2(mul_bf2(dv[k][j], w[k][j]));
        // dt * inv + dsq * (2 r), each product rounded, then the sum
        // dt * inv + dsq * (2 r): both products rounded, then the sum. The
        // sum is taken with the scalar __fadd_rn, which is never merged into
        // a multiply-add (packed fp32x2 multiplies and adds were, even as
        // explicit .rn instructions: the result came out rounded once).
        const float2 g1 = __fmul2_rn(dt, inv2);
        const float2 g2 = __fmul2_rn(dsq2, __fadd2_rn(rf, rf));
        uint32_t d = f2_to_bf2(make_float2(__fadd_rn(g1.x, g2.x), __fadd_rn(g1.y, g2.y)));
        if (RES) d = add_bf2(d, gg[j]);
        if (DW) {
          const uint32_t tb = f2_to_bf2(__fmul2_rn(rf, inv2));  // the forward's bf16(r * inv)
          accp[j] = __fadd2_rn(accp[j], bf2_to_f2(mul_bf2(dv[k][j], tb)));
        }
        rv[k][j] = d;  // rv now holds dr
      }
      if (DW && vok[k]) {
        *reinterpret_cast<float4*>(acc) = make_float4(accp[0].x, accp[0].y, accp[1].x, accp[1].y);
        *reinterpret_cast<float4*>(acc + 4) =
            make_float4(accp[2].x, accp[2].y, accp[3].x, accp[3].y);
      }
      st_bf16x8(xrow + (int64_t)(tvec + 8 * k) * 8, rv[k], vok[k]);
    }

    if constexpr (QUANT) {
      // two 1x128 groups an octet (slots 0-1, 2-3), as in the forward kernel
      const uint32_t pa = absmax_bf2(vec_absmax(rv[0]), vec_absmax(rv[1]));
      const uint32_t pb = absmax_bf2(vec_absmax(rv[2]), vec_absmax(rv[3]));
      uint32_t p =
          absmax_bf2(__byte_perm(pa, pb, 0x5410), __byte_perm(pa, pb, 0x7632)) & 0x7fff7fffu;
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
      const float2 am = bf2_to_f2(p);
      const bool pow2 = qa.scale_fmt != kFmtF32;
      const float sa = make_scale(am.x, pow2), sb = make_scale(am.y, pow2);
      const float ra = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sa)) : rcp_scale(sa);
      const float rb = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sb)) : rcp_scale(sb);
      char* srow = static_cast<char*>(qa.scale) +
                   row * qa.s_row * ((qa.scale_fmt == kFmtE8M0) ? 1 : 4);
      if (gput) {
        if (qa.scale_layout == kLaySwizzled)
          put_scale(qa, row, srow, gidx, (lane & 1) ? sb : sa);
        else if (qa.scale_fmt == kFmtE8M0)
          srow[goff] = (char)(__float_as_uint((lane & 1) ? sb : sa) >> 23);
        else
          *reinterpret_cast<float*>(srow + goff) = (lane & 1) ? sb : sa;
      }
      if (qa.scale_layout == kLaySwizzled && qa.n_groups_pad > qa.n_groups)
        zero_scale_padding(qa, row, qa.n_groups, t, T);
      uint32_t* qthr = reinterpret_cast<uint32_t*>(qa.q + row * qa.ldq + (int64_t)tvec * 8);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const float rcs = k < 2 ? ra : rb, ns = k < 2 ? -sa : -sb;
        const float2 rc2 = make_float2(rcs, rcs), nb = make_float2(ns, ns);
        float2 y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          y[j] = pow2 ? __fmul2_rn(bf2_to_f2(rv[k][j]), rc2) : div2_rn(bf2_to_f2(rv[k][j]), nb, rc2);
        st_stream2_if(vok[k], qthr + 16 * k, f4_to_e4m3x4(y[0], y[1]), f4_to_e4m3x4(y[2], y[3]));
      }
    }
  }
  if constexpr (QUANT)  // swizzled-layout padding rows: scales only
    if (qa.scale_layout == kLaySwizzled) {
      const int64_t nrows = (int64_t)blockIdx.x < qa.M ? (qa.M - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      for (int64_t r = blockIdx.x + nrows * gridDim.x; r < qa.M_pad; r += gridDim.x)
        zero_scale_padding(qa, r, 0, t, T);
    }
  if (DW) {
    __syncthreads();
    float* out = a.partial + (int64_t)blockIdx.x * V * 8;
    for (int i = t; i < V * 8; i += T) out[i] = wacc[i];
  }
}

// Bulk-copy ring variant of the kernel above (rows of up to 16384, 512
// threads): the same arithmetic in the same order, with the loads moved off
// the threads. Dynamic shared memory holds S stages of [r row | dn row |
// dro row], each row buffer bwd_row_pad() bytes (the bytes past the copied
// row are zeroed once and never written by a copy, so vector slots past the
// row end read zeros). Row k of the CTA (row = blockIdx.x + k * gridDim.x)
// sits in stage k % S; its copies were issued when row k - S left the stage.
//
// Per row: wait for the stage; pass 1 reads r and dn and forms both row sums;
// one block barrier (the sums, and a vote on failed waits); pass 2 reads r,
// dn and dro again, writes dx and accumulates dw in registers; the warp then
// counts itself out of the stage and the last warp out refills it with row
// k + S (a shared-memory counter, no block barrier); dx is then quantized
// from registers. A wait that gives up (about 2 s) fails the vote: the CTA
// sets the device error word, lets every copy it issued land (bounded) and
// exits.
constexpr int kBwdMaxStages = 4;

__host__ __device__ inline uint32_t bwd_row_pad(int V, int T) {
  const uint32_t row_bytes = (uint32_t)V * 16u, span = (uint32_t)T * 64u;
  return span > row_bytes ? span : row_bytes;
}

// MAXT: the largest block of the instantiation: 256 (two CTAs an SM) or 512
// (one), up to 128 registers a thread either way.
template <bool RES, bool QUANT, bool DW, bool FULL, int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 256 ? 2 : 1)
    rmsnorm_backward_ring_kernel(const BwdArgs a, float eps, float rcp_H, int S) {
  constexpr int NV = 4;
  constexpr uint32_t NB = RES ? 3u : 2u;  // row buffers a stage
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float2 red[2][32];
  __shared__ __align__(8) uint64_t full_bar[kBwdMaxStages];
  __shared__ uint32_t done_cnt[kBwdMaxStages];    // warps that left each stage, cumulative
  __shared__ uint32_t issued_cnt[kBwdMaxStages];  // copies issued into each stage

  const FusedArgs& qa = a.qa;
  const int T = blockDim.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int V = qa.V;
  const uint32_t row_bytes = (uint32_t)V * 16u;
  const uint32_t row_pad = bwd_row_pad(V, T);
  const uint32_t stage_bytes = NB * row_pad;
  const uint32_t ring = smem_addr(smem);
  const int64_t G = gridDim.x;
  const int64_t nrows = (int64_t)blockIdx.x < qa.M ? (qa.M - 1 - blockIdx.x) / G + 1 : 0;
  const int tvec = warp * 128 + (lane >> 3) * 32 + (lane & 7);
  const uint32_t toff = (uint32_t)tvec * 16u;
  bool vok[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) vok[k] = FULL || tvec + 8 * k < V;

  // the barrier and counter arrays hold kBwdMaxStages stages; the host plans
  // 2-4 (anything else is refused before any set-up)
  if (S < 2 || S > kBwdMaxStages) {
    if (t == 0) atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBadLaunch);
    return;
  }

  auto issue = [&](int s, int64_t row) {
    const uint32_t bar = smem_addr(&full_bar[s]);
    const uint32_t dst = ring + (uint32_t)s * stage_bytes;
    mbar_arrive_expect_tx(bar, NB * row_bytes);
    bulk_g2s(dst, a.r + row * a.ldr, row_bytes, bar);
    bulk_g2s(dst + row_pad, a.dn + row * a.lddn, row_bytes, bar);
    if constexpr (RES) bulk_g2s(dst + 2u * row_pad, a.dro + row * a.lddro, row_bytes, bar);
  };

  // zero the pad of every row buffer once (the copies never write it)
  for (uint32_t b = 0; b < (uint32_t)S * NB; ++b)
    for (uint32_t o = row_bytes + 4u * (uint32_t)t; o < row_pad; o += 4u * (uint32_t)T)
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(ring + b * row_pad + o), "r"(0u) : "memory");
  if (t == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      done_cnt[s] = 0;
      issued_cnt[s] = 0;
    }
    mbar_init_fence();
  }
  __syncthreads();
  griddep_wait();  // inputs of the previous kernel are complete from here on
  if (t == 0)
    for (int s = 0; s < S && s < nrows; ++s) {
      issued_cnt[s] = 1;
      issue(s, blockIdx.x + (int64_t)s * G);
    }
  // weights: the same columns for every row
  uint32_t w[NV][4];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (vok[k]) u = ld_keep(a.w + (int64_t)(tvec + 8 * k) * 8);
    w[k][0] = u.x;
    w[k][1] = u.y;
    w[k][2] = u.z;
    w[k][3] = u.w;
  }
  griddep_launch_dependents();

  // this thread's quantization group and whether it writes its scale (lanes
  // 0 and 1 of an octet, for the octet's two groups)
  const int gidx = warp * 8 + (lane >> 3) * 2 + (lane & 1);
  const bool gput = (lane & 6) == 0 && (FULL || gidx * 16 < V);
  const int64_t goff = ((int64_t)(gidx >> 2) * qa.s_grp4 + (int64_t)(gidx & 3) * qa.s_grp) *
                       ((qa.scale_fmt == kFmtE8M0) ? 1 : 4);
  float2 dwa[NV][4];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 4; ++j) dwa[k][j] = make_float2(0.0f, 0.0f);

  int flip = 0, s = 0;
  uint32_t use = 0;  // how many times the ring wrapped at this row
  int64_t row = blockIdx.x;
  for (int64_t k = 0; k < nrows; ++k, row += G) {
    const uint32_t base = ring + (uint32_t)s * stage_bytes;
    int bad = mbar_wait_bounded(smem_addr(&full_bar[s]), use & 1u, qa.wait_limit) ? 0 : 1;
    // (sum r^2, sum dt * r) in the order of the kernel above
    float2 sq = make_float2(0.0f, 0.0f), pr = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      const uint4 u = ld_smem(base + toff + 128u * k2);
      const uint4 e = ld_smem(base + row_pad + toff + 128u * k2);
      const uint32_t rv[4] = {u.x, u.y, u.z, u.w}, dv[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = bf2_to_f2(rv[j]);
        const float2 dt = bf2_to_f2(mul_bf2(dv[j], w[k2][j]));
        sq = __ffma2_rn(rf, rf, sq);
        pr = __ffma2_rn(dt, rf, pr);
      }
    }
    float2 s2 = make_float2(__fadd_rn(sq.x, sq.y), __fadd_rn(pr.x, pr.y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s2.x = __fadd_rn(s2.x, __shfl_xor_sync(0xffffffffu, s2.x, o));
      s2.y = __fadd_rn(s2.y, __shfl_xor_sync(0xffffffffu, s2.y, o));
    }
    if (lane == 0) red[flip][warp] = s2;
    bad = __syncthreads_or(bad);
    if (bad) {
      // A copy never completed: report it, let every copy this CTA issued
      // land (bounded), and leave. Every refill so far was issued before its
      // warp reached this barrier, so issued_cnt is complete here.
      if (t == 0) {
        atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
        for (int si = 0; si < S; ++si)
          if (issued_cnt[si] > 0)
            mbar_wait_bounded(smem_addr(&full_bar[si]), (issued_cnt[si] - 1u) & 1u,
                              kDrainLimitCycles);
      }
      return;
    }
    float2 tot = lane < nw ? red[flip][lane] : make_float2(0.0f, 0.0f);
    flip ^= 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot.x = __fadd_rn(tot.x, __shfl_xor_sync(0xffffffffu, tot.x, o));
      tot.y = __fadd_rn(tot.y, __shfl_xor_sync(0xffffffffu, tot.y, o));
    }
    float mean = div_rn(tot.x, (float)qa.H, rcp_H);
    if (mean < 0x1p-100f) mean = __fdiv_rn(tot.x, (float)qa.H);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
    const float dvar = __fmul_rn(__fmul_rn(-0.5f, tot.y), __fmul_rn(__fmul_rn(inv, inv), inv));
    const float dsq = __fdiv_rn(dvar, (float)qa.H);
    const float2 inv2 = make_float2(inv, inv), dsq2 = make_float2(dsq, dsq);

    uint16_t* xrow = a.dx + row * a.lddx;
    uint32_t dr[NV][4];
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      const uint4 u = ld_smem(base + toff + 128u * k2);
      const uint4 e = ld_smem(base + row_pad + toff + 128u * k2);
      uint4 g = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (RES) g = ld_smem(base + 2u * row_pad + toff + 128u * k2);
      const uint32_t rv[4] = {u.x, u.y, u.z, u.w}, dv[4] = {e.x, e.y, e.z, e.w};
      const uint32_t gg[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = bf2_to_f2(rv[j]);
        const float2 dt = bf2_to_f2(mul_bf2(dv[j], w[k2][j]));
        // dt * inv + dsq * (2 r): both products rounded, then the sum, taken
        // with the scalar __fadd_rn (never merged into a multiply-add)
        const float2 g1 = __fmul2_rn(dt, inv2);
        const float2 g2 = __fmul2_rn(dsq2, __fadd2_rn(rf, rf));
        uint32_t d = f2_to_bf2(make_float2(__fadd_rn(g1.x, g2.x), __fadd_rn(g1.y, g2.y)));
        if (RES) d = add_bf2(d, gg[j]);
        if (DW) {
          const uint32_t tb = f2_to_bf2(__fmul2_rn(rf, inv2));  // the forward's bf16(r * inv)
          dwa[k2][j] = __fadd2_rn(dwa[k2][j], bf2_to_f2(mul_bf2(dv[j], tb)));
        }
        dr[k2][j] = d;
      }
      st_bf16x8(xrow + (int64_t)(tvec + 8 * k2) * 8, dr[k2], vok[k2]);
    }
    // Count this warp out of the stage; the last warp refills it. The
    // acq_rel add orders every lane's reads (joined by __syncwarp) before the
    // refill, and the proxy fence orders them before the copy engine's writes.
    __syncwarp();
    if (lane == 0) {
      const uint32_t old = atom_add_acq_rel(smem_addr(&done_cnt[s]), 1u);
      if (old + 1u == (use + 1u) * (uint32_t)nw && k + S < nrows) {
        fence_proxy_async_smem();
        issued_cnt[s] = use + 2u;
        issue(s, row + (int64_t)S * G);
      }
    }
    if (++s == S) {
      s = 0;
      ++use;
    }

    if constexpr (QUANT) {
      // two 1x128 groups an octet (slots 0-1, 2-3), as in the forward kernel
      const uint32_t pa = absmax_bf2(vec_absmax(dr[0]), vec_absmax(dr[1]));
      const uint32_t pb = absmax_bf2(vec_absmax(dr[2]), vec_absmax(dr[3]));
      uint32_t p =
          absmax_bf2(__byte_perm(pa, pb, 0x5410), __byte_perm(pa, pb, 0x7632)) & 0x7fff7fffu;
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
      const float2 am = bf2_to_f2(p);
      const bool pow2 = qa.scale_fmt != kFmtF32;
      const float sa = make_scale(am.x, pow2), sb = make_scale(am.y, pow2);
      const float ra = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sa)) : rcp_scale(sa);
      const float rb = pow2 ? __uint_as_float((254u << 23) - __float_as_uint(sb)) : rcp_scale(sb);
      char* srow = static_cast<char*>(qa.scale) +
                   row * qa.s_row * ((qa.scale_fmt == kFmtE8M0) ? 1 : 4);
      if (gput) {
        if (qa.scale_layout == kLaySwizzled)
          put_scale(qa, row, srow, gidx, (lane & 1) ? sb : sa);
        else if (qa.scale_fmt == kFmtE8M0)
          srow[goff] = (char)(__float_as_uint((lane & 1) ? sb : sa) >> 23);
        else
          *reinterpret_cast<float*>(srow + goff) = (lane & 1) ? sb : sa;
      }
      if (qa.scale_layout == kLaySwizzled && qa.n_groups_pad > qa.n_groups)
        zero_scale_padding(qa, row, qa.n_groups, t, T);
      uint32_t* qthr = reinterpret_cast<uint32_t*>(qa.q + row * qa.ldq + (int64_t)tvec * 8);
#pragma unroll
      for (int k2 = 0; k2 < NV; ++k2) {
        const float rcs = k2 < 2 ? ra : rb, ns = k2 < 2 ? -sa : -sb;
        const float2 rc2 = make_float2(rcs, rcs), nb = make_float2(ns, ns);
        float2 y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          y[j] = pow2 ? __fmul2_rn(bf2_to_f2(dr[k2][j]), rc2) : div2_rn(bf2_to_f2(dr[k2][j]), nb, rc2);
        st_stream2_if(vok[k2], qthr + 16 * k2, f4_to_e4m3x4(y[0], y[1]), f4_to_e4m3x4(y[2], y[3]));
      }
    }
  }
  if constexpr (QUANT)  // swizzled-layout padding rows: scales only
    if (qa.scale_layout == kLaySwizzled)
      for (int64_t r = blockIdx.x + nrows * G; r < qa.M_pad; r += G) zero_scale_padding(qa, r, 0, t, T);
  if (DW) {  // this CTA's row of partial sums: each thread its own columns
    float* out = a.partial + (int64_t)blockIdx.x * V * 8;
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2)
      if (vok[k2]) {
        float4* o4 = reinterpret_cast<float4*>(out + (int64_t)(tvec + 8 * k2) * 8);
        o4[0] = make_float4(dwa[k2][0].x, dwa[k2][0].y, dwa[k2][1].x, dwa[k2][1].y);
        o4[1] = make_float4(dwa[k2][2].x, dwa[k2][2].y, dwa[k2][3].x, dwa[k2][3].y);
      }
  }
}

// dw[j] = bf16(sum of the CTAs' partial rows). A block takes 32 columns; 8
// warps each sum every 8th partial row of them (rows s, s + 8, ...: one
// 128-byte load a warp a step, eight loads in flight), then the 8 slice sums
// are added in slice order. The order is fixed, so the result is
// deterministic.
__global__ void __launch_bounds__(256) rmsnorm_backward_dw_kernel(const float* partial, int rows,
                                                                 int H, uint16_t* dw) {
  __shared__ float slice[8][33];
  griddep_wait();
  griddep_launch_dependents();
  const int c = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + c;
  float s = 0.0f;
  if (j < H) {
#pragma unroll 8
    for (int b = sl; b < rows; b += 8) s = __fadd_rn(s, partial[(int64_t)b * H + j]);
  }
  slice[sl][c] = s;
  __syncthreads();
  if (sl == 0 && j < H) {
    float t = slice[0][c];
#pragma unroll
    for (int k = 1; k < 8; ++k) t = __fadd_rn(t, slice[k][c]);
    const __nv_bfloat16 v = __float2bfloat16_rn(t);
    dw[j] = *reinterpret_cast<const uint16_t*>(&v);
  }
}

namespace {

// Shared memory of one SM (228 KB) and what a CTA holds besides its ring
// (the 1 KB the hardware reserves a CTA, and the static arrays).
constexpr size_t kSmemPerSm = 228 * 1024;
constexpr size_t kCtaSmemOverhead = 2048;

// CTAs an SM runs at once: the ring kernel is compiled for up to 128
// registers a thread (512 threads' worth of the 64K registers: two CTAs of up
// to 256 threads, or one of up to 512), the direct kernel (MAXT = 1024) for
// 64 registers (1024 threads); at most 8 CTAs an SM either way.
int backward_ctas_per_sm(int T) {
  int per_sm = T <= 512 ? 512 / T : 1024 / T;
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 8) per_sm = 8;
  return per_sm;
}

// Stages of the ring kernel that fit next to per_sm - 1 other CTAs (0: the
// ring does not fit).
int backward_ring_stages(int V, int T, int per_sm, bool res) {
  if (T > 512) return 0;
  const size_t stage = (res ? 3u : 2u) * (size_t)bwd_row_pad(V, T);
  size_t budget = kSmemPerSm / (size_t)per_sm;
  budget = budget > kCtaSmemOverhead ? budget - kCtaSmemOverhead : 0;
  if (budget > 227 * 1024 - kCtaSmemOverhead) budget = 227 * 1024 - kCtaSmemOverhead;
  int S = (int)(budget / stage);
  if (S > kBwdMaxStages) S = kBwdMaxStages;
  return S >= 2 ? S : 0;
}

template <typename K, typename... Args>
cudaError_t launch_with_smem(K k, int grid, int threads, size_t smem, cudaStream_t st,
                             Args... args) {
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(k, (unsigned)grid, (unsigned)threads, smem, st, args...);
}

// Rows of up to 16384 (T <= 512): the ring kernel (MAXT 256 or 512); wider
// rows: the direct kernel (MAXT = 1024).
template <bool RES, bool QUANT, bool DW>
cudaError_t launch_bwd3(const BwdArgs& a, float eps, int threads, int grid, int stages,
                        size_t direct_smem, cudaStream_t st) {
  const bool full = (int64_t)threads * 4 == a.qa.V;
  const float rcp_H = 1.0f / (float)a.qa.H;
  if (stages > 0) {
    const size_t smem = (size_t)stages * (RES ? 3u : 2u) * bwd_row_pad(a.qa.V, threads);
    if (threads <= 256)
      return full ? launch_with_smem(rmsnorm_backward_ring_kernel<RES, QUANT, DW, true, 256>,
                                     grid, threads, smem, st, a, eps, rcp_H, stages)
                  : launch_with_smem(rmsnorm_backward_ring_kernel<RES, QUANT, DW, false, 256>,
                                     grid, threads, smem, st, a, eps, rcp_H, stages);
    return full ? launch_with_smem(rmsnorm_backward_ring_kernel<RES, QUANT, DW, true, 512>, grid,
                                   threads, smem, st, a, eps, rcp_H, stages)
                : launch_with_smem(rmsnorm_backward_ring_kernel<RES, QUANT, DW, false, 512>, grid,
                                   threads, smem, st, a, eps, rcp_H, stages);
  }
  return full ? launch_with_smem(rmsnorm_backward_kernel<RES, QUANT, DW, true, 1024>, grid,
                                 threads, direct_smem, st, a, eps, rcp_H)
              : launch_with_smem(rmsnorm_backward_kernel<RES, QUANT, DW, false, 1024>, grid,
                                 threads, direct_smem, st, a, eps, rcp_H);
}

}  // namespace

// Threads of one row and CTAs of the grid for a backward launch; the grid is
// also the number of partial dw rows the workspace must hold.
void backward_shape(int64_t M, int64_t H, int* threads, int* grid) {
  const int64_t V = H / 8;
  int T = (int)((V + 127) / 128 * 32);
  if (T < 32) T = 32;
  *threads = T;
  int64_t g = (int64_t)backward_ctas_per_sm(T) * device_sm_count();
  if (g > M) g = M;
  if (g < 1) g = 1;
  *grid = (int)g;
}

cudaError_t launch_backward(const BwdArgs& a, float eps, bool dw_wanted, uint16_t* dw,
                            int max_grid, cudaStream_t st) {
  int T = 0, grid = 0;
  backward_shape(a.qa.M, a.qa.H, &T, &grid);
  if (max_grid > 0 && grid > max_grid) grid = max_grid;
  if (a.qa.M_pad == 0)  // no rows: d_weight is zero (a sum over no partial rows)
    return dw_wanted ? launch_pdl(rmsnorm_backward_dw_kernel, (unsigned)((a.qa.H + 31) / 32),
                                  256u, 0, st, (const float*)a.partial, 0, a.qa.H, dw)
                     : cudaSuccess;
  const bool res = a.dro != nullptr, quant = a.qa.q != nullptr;
  const int stages = backward_ring_stages(a.qa.V, T, backward_ctas_per_sm(T), res);
  const size_t smem = dw_wanted ? (size_t)a.qa.V * 8 * sizeof(float) : 0;  // direct kernel
  cudaError_t e;
  if (dw_wanted) {
    e = res ? (quant ? launch_bwd3<true, true, true>(a, eps, T, grid, stages, smem, st)
                     : launch_bwd3<true, false, true>(a, eps, T, grid, stages, smem, st))
            : (quant ? launch_bwd3<false, true, true>(a, eps, T, grid, stages, smem, st)
                     : launch_bwd3<false, false, true>(a, eps, T, grid, stages, smem, st));
  } else {
    e = res ? (quant ? launch_bwd3<true, true, false>(a, eps, T, grid, stages, smem, st)
                     : launch_bwd3<true, false, false>(a, eps, T, grid, stages, smem, st))
            : (quant ? launch_bwd3<false, true, false>(a, eps, T, grid, stages, smem, st)
                     : launch_bwd3<false, false, false>(a, eps, T, grid, stages, smem, st));
  }
  if (e != cudaSuccess || !dw_wanted) return e;
  const int H = a.qa.H;
  return launch_pdl(rmsnorm_backward_dw_kernel, (unsigned)((H + 31) / 32), 256u, 0, st,
                    (const float*)a.partial, grid, H, dw);
}

}  // namespace cutie
