// Pipelined single-pass kernel for [residual add] -> RMSNorm -> [1xG group
// FP8 quantization | no quantization], the default path for rows that fit
// one CTA (H <= 32768).
//
// Same per-element arithmetic as fused_rmsnorm_fp8_kernel (fused_kernel.cuh);
// for 1x32 and 1x64 groups also the same chunk layout (64-byte chunks, one
// per thread, rotated reads) and so the same bits. 1x128 groups and plain
// RMSNorm output use an interleaved layout (below) whose sum of squares adds
// the same terms in another order. What changes most is how a CTA moves from
// row to row. The single-pass kernel
// stops every warp at two block barriers per row. Here nothing waits on a
// block barrier inside the row loop:
//
//  * rows of a CTA are numbered k = 0, 1, ... (row = blockIdx.x + k * G);
//    iteration k runs phase A of row k + 1, then phase B of row k;
//  * phase A: wait for the row's bulk copy, read it (adding the residual in
//    bf16 and writing residual_out), publish the warp's sum of squares in a
//    slot of a 4-deep ring and arrive on that slot's mbarrier;
//  * the "finisher" of row k, warp k % nw, waits for all partial sums of row
//    k (published one iteration earlier), turns them into inv_rms and
//    publishes it through a second 4-deep mbarrier ring;
//  * phase B: read the row from its stage again (and the weights), count
//    this warp out of the stage (a shared-memory counter; the last warp out
//    refills the stage with row k + S), wait for row k's inv_rms, then
//    normalise, take group maxima, write scales and FP8 codes.
//
// A warp can run up to about three rows ahead of the slowest one, which is
// why the rings are four deep (the argument is spelled out at the rings).
// Waits are bounded (FusedArgs::wait_limit, about 2 s by default): a wait
// that gives up sets the device error word and an abort flag that ends every
// other wait of the CTA, no stage is refilled after that, and the CTA lets
// the last copy it issued into each stage land (bounded) before it exits.
//
// Arithmetic shared with the single-pass kernel lives in fused_kernel.cuh;
// the two sm_90+ forms used only here are the mixed-precision square
// (fma.rn.f32.bf16: exact product, one rounding, the same value as the fp32
// FMA on the widened inputs) and the bf16x2 residual add (add.rn.bf16x2:
// for two bf16 values the exact sum rounded once to bf16 equals the fp32 sum
// rounded to bf16, the reference's `(x + residual)` on bf16 tensors).
#pragma once

#include "fused_kernel.cuh"

namespace cutie {

// Scale destination of a launch (fixed per launch, so compiled in).
enum : int {
  kSkF32 = 0,      // fp32 values, strided
  kSkF32Pow2 = 1,  // fp32 powers of two (UE8M0 values), strided
  kSkE8 = 2,       // e8m0 bytes, strided
  kSkE8Swz = 3,    // e8m0 bytes, Blackwell block-scaled swizzle
};
constexpr int kPipeMaxStages = 4;
constexpr int kPipeRing = 4;  // depth of the partial-sum and inv_rms rings

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Wait for phase `parity` as mbar_wait_bounded does (one non-blocking test,
// then suspending try_waits for at most `limit` cycles; limit < 0 never
// blocks), giving up at once when the CTA's abort flag is set. A wait that
// gives up sets the flag, so every later wait of the CTA returns at once.
__device__ __forceinline__ bool mbar_wait_abortable(uint32_t bar, uint32_t parity,
                                                    volatile uint32_t* abort_flag,
                                                    long long limit) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  while (!*abort_flag && clock64() - t0 <= limit)
    if (mbar_try_wait(bar, parity)) return true;
  *abort_flag = 1u;
  return false;
}

// Streaming fp32 store guarded by `ok` inside the instruction (no branch).
__device__ __forceinline__ void st_f32_if(bool ok, void* p, float v) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.u32 q, %2, 0;\n @q st.global.f32 [%0], %1;\n}" ::"l"(p),
      "f"(v), "r"((uint32_t)ok)
      : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(addr), "r"(v)
               : "memory");
  return old;
}

// Orders this thread's view of generic-proxy shared-memory accesses before
// its subsequent async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_smem(uint32_t addr, const uint32_t (&v)[4]) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

// bf16 pair + bf16 pair, each rounded once to bf16 (nearest even).
__device__ __forceinline__ uint32_t add_bf2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// (lo^2, hi^2) of a bf16 pair, and acc += (lo^2, hi^2); the products are
// exact, each sum is rounded once.
__device__ __forceinline__ float2 sq_first(uint32_t u) {
  float2 r;
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n"
      " fma.rn.f32.bf16 %0, lo, lo, 0f00000000;\n fma.rn.f32.bf16 %1, hi, hi, 0f00000000;\n}"
      : "=f"(r.x), "=f"(r.y)
      : "r"(u));
  return r;
}
__device__ __forceinline__ void sq_acc(float2& acc, uint32_t u) {
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n"
      " fma.rn.f32.bf16 %0, lo, lo, %0;\n fma.rn.f32.bf16 %1, hi, hi, %1;\n}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(u));
}

// Scale of one group, written by the group's leader lane (`put`).
template <int SK>
__device__ __forceinline__ void put_group_scale(bool put, const FusedArgs& a, int64_t row,
                                                char* srow, int64_t goff, int g, float s) {
  if constexpr (SK == kSkE8Swz) {
    if (put)
      static_cast<uint8_t*>(a.scale)[swizzled_offset(row, g, a.n_groups_pad >> 2)] =
          (uint8_t)(__float_as_uint(s) >> 23);
  } else if constexpr (SK == kSkE8) {
    if (put) srow[goff] = (char)(__float_as_uint(s) >> 23);
  } else {
    st_f32_if(put, srow + goff, s);
  }
}

// Thread layouts. Every thread holds 4 vectors (32 elements) of a row.
//  * chunked (1x32 and 1x64 groups): the 4 vectors are one contiguous 64-byte
//    chunk, so a 1x32 group is one thread and a 1x64 group two lanes; the
//    chunk is visited in a per-thread rotated order (see fused_kernel.cuh).
//  * interleaved (1x128 groups and no quantization): lane i of octet o of
//    warp w holds vectors w*128 + o*32 + i + 8k, k = 0..3. The 8 lanes of an
//    octet read 128 contiguous bytes per vector slot (conflict-free shared
//    loads, and whole 32-byte sectors per store), every address is the
//    thread's base plus a constant, and an octet covers two 1x128 groups:
//    slots 0-1 are the first, slots 2-3 the second.
template <int QM, int LPG>
struct PipeLayout {
  static constexpr bool kInterleaved = QM == kQNone || LPG == 4;
};

// Bytes of one row buffer in shared memory: the copied row plus a zero pad
// that every vector slot past the row end reads. Chunked: whole chunks plus
// one more zero chunk; interleaved: T * 64 bytes (4 vectors a thread).
__host__ __device__ inline uint32_t pipe_row_pad(int V, int T, bool interleaved) {
  const uint32_t row_bytes = (uint32_t)V * 16u;
  if (interleaved) {
    const uint32_t span = (uint32_t)T * 64u;
    return span > row_bytes ? span : row_bytes;
  }
  return ((row_bytes + 63u) & ~63u) + 64u;
}

// QM: kQGroup (LPG lanes a group) or kQNone. FULL: T * 4 == V (no store
// predicates). SK: scale destination. MAXT: the largest block this
// instantiation is launched with; 224 lets the compiler use 72 registers a
// thread (four 7-warp CTAs an SM), 1024 caps it at 64. (A 56-register cap
// for five CTAs an SM measured slower: the extra warps did not raise the
// issue rate, and the cap added instructions.)
//
// Dynamic shared memory: `a.stages` stages of [x row | residual row], each
// row buffer pipe_row_pad() bytes.
template <int QM, int LPG, bool RES, bool FULL, int SK, int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 224 ? 4 : 1)
    pipe_rmsnorm_fp8_kernel(const FusedArgs a) {
  static_assert(QM == kQGroup || QM == kQNone, "group or no quantization");
  static_assert(QM != kQGroup || LPG == 1 || LPG == 2 || LPG == 4, "lanes per group");
  constexpr bool ILV = PipeLayout<QM, LPG>::kInterleaved;
  constexpr int NV = 4;  // 4 vectors (32 elements) a thread
  constexpr bool kPow2 = SK != kSkF32;
  constexpr int kEsz = (SK == kSkE8 || SK == kSkE8Swz) ? 1 : 4;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float part[kPipeRing][32];
  __shared__ float inv_slot[kPipeRing];
  __shared__ __align__(8) uint64_t full_bar[kPipeMaxStages];
  __shared__ __align__(8) uint64_t red_bar[kPipeRing];
  __shared__ __align__(8) uint64_t inv_bar[kPipeRing];
  __shared__ uint32_t done_cnt[kPipeMaxStages];    // warps that left each stage, cumulative
  __shared__ uint32_t issued_cnt[kPipeMaxStages];  // copies issued into each stage
  __shared__ uint32_t abort_flag;

  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nw = T >> 5;
  const int S = a.stages;
  const uint32_t row_bytes = (uint32_t)a.V * 16u;
  const uint32_t row_chunks = (row_bytes + 63u) & ~63u;
  const uint32_t row_pad = pipe_row_pad(a.V, T, ILV);
  const uint32_t stage_bytes = RES ? 2u * row_pad : row_pad;
  const uint32_t ring = smem_addr(smem);
  const int64_t G = gridDim.x;
  const int64_t nrows = (int64_t)blockIdx.x < a.M ? (a.M - 1 - blockIdx.x) / G + 1 : 0;

  // Byte offset of this thread's k-th vector within a row (voff[k], or
  // tvec * 16 + 128 k interleaved) and whether it lies inside the row.
  // Chunked: vector j of the chunk is visited at (j + rot) & 3, as in the
  // single-pass kernel.
  const int rot = (t >> 1) & 3;
  const int tvec = warp * 128 + (lane >> 3) * 32 + (lane & 7);  // interleaved: slot 0
  const uint32_t toff = (uint32_t)tvec * 16u;
  uint32_t voff[NV];
  bool vok[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if constexpr (ILV) {
      vok[k] = FULL || tvec + 8 * k < a.V;
      voff[k] = toff + 128u * (uint32_t)k;
    } else {
      const int j = (k + rot) & 3;
      const int vi = t * 4 + j;
      vok[k] = FULL || vi < a.V;
      voff[k] = FULL || (uint32_t)t * 64u < row_chunks ? (uint32_t)vi * 16u
                                                        : row_chunks + 16u * (uint32_t)j;
    }
  }

  auto issue = [&](int s, int64_t row) {
    const uint32_t bar = smem_addr(&full_bar[s]);
    const uint32_t dst = ring + (uint32_t)s * stage_bytes;
    mbar_arrive_expect_tx(bar, RES ? 2u * row_bytes : row_bytes);
    bulk_g2s(dst, a.x + row * a.ldx, row_bytes, bar);
    if constexpr (RES) bulk_g2s(dst + row_pad, a.res + row * a.ldr, row_bytes, bar);
  };

  // the barrier and counter arrays hold kPipeMaxStages stages; the host plans
  // 2-3 (a plan outside [2, kPipeMaxStages] is refused before any set-up)
  if (S < 2 || S > kPipeMaxStages) {
    if (t == 0) atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBadLaunch);
    return;
  }

  // zero the pad of every row buffer once (the copies never write it)
  for (int s = 0; s < S * (RES ? 2 : 1); ++s)
    for (uint32_t b = row_bytes + 4u * (uint32_t)t; b < row_pad; b += 4u * (uint32_t)T)
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(ring + (uint32_t)s * row_pad + b), "r"(0u)
                   : "memory");
  if (t == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      done_cnt[s] = 0;
      issued_cnt[s] = 0;
    }
    for (int k = 0; k < kPipeRing; ++k) {
      mbar_init(smem_addr(&red_bar[k]), (uint32_t)T);  // every thread arrives
      mbar_init(smem_addr(&inv_bar[k]), 1);
    }
    abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  griddep_wait();  // inputs of the previous kernel are complete from here on
  griddep_launch_dependents();
  if (t == 0)
    for (int s = 0; s < S && s < nrows; ++s) {
      issued_cnt[s] = 1;
      issue(s, blockIdx.x + (int64_t)s * G);
    }

  const bool store_ro = RES && a.res_out != nullptr;
  const bool store_no = a.norm_out != nullptr;
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(a.w);
  // this thread's group: index, byte offset within a strided scale row, and
  // whether it writes the scale (leader lane of a group inside the row;
  // interleaved: lanes 0 and 1 of each octet, for its two groups)
  const int gidx = ILV ? warp * 8 + (lane >> 3) * 2 + (lane & 1) : t / LPG;
  const int64_t goff = ((int64_t)(gidx >> 2) * a.s_grp4 + (int64_t)(gidx & 3) * a.s_grp) * kEsz;
  const bool gput = ILV ? (lane & 6) == 0 : (t & (LPG - 1)) == 0 && (FULL || t * 4 < a.V);
  volatile uint32_t* abortp = &abort_flag;
  bool ok = true;  // every wait of this thread completed
  // code rows on 32- (16-) byte boundaries take one 32-byte store a thread
  const bool q32 = aligned_rows(a.q, a.ldq, 32), q16 = aligned_rows(a.q, a.ldq, 16);

  // Rings. Row k uses slot k & 3 of part/red_bar and of inv_slot/inv_bar.
  // Reuse is safe: a warp writes row k + 4's partial in phase A(k + 4),
  // which follows its phase B(k + 2); B(k + 2) needed inv_rms(k + 2), which
  // needed every warp's phase A(k + 2), and each of those follows that warp's
  // use of slot k (the finisher's read in iteration k, everyone's B(k)). The
  // same chain keeps any mbarrier from running two phases ahead of a waiter.

  // ---------------------------------------------------------------- phase A
  auto phase_a = [&](int k, int s, uint32_t par, uint8_t* rorow) {
    const uint32_t base = ring + (uint32_t)s * stage_bytes;
    ok &= mbar_wait_abortable(smem_addr(&full_bar[s]), par, abortp, a.wait_limit);
    uint32_t v[NV][4];
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      const uint4 u = ld_smem(base + voff[k2]);
      v[k2][0] = u.x;
      v[k2][1] = u.y;
      v[k2][2] = u.z;
      v[k2][3] = u.w;
    }
    if constexpr (RES) {
#pragma unroll
      for (int k2 = 0; k2 < NV; ++k2) {
        const uint4 u = ld_smem(base + row_pad + voff[k2]);
        v[k2][0] = add_bf2(v[k2][0], u.x);
        v[k2][1] = add_bf2(v[k2][1], u.y);
        v[k2][2] = add_bf2(v[k2][2], u.z);
        v[k2][3] = add_bf2(v[k2][3], u.w);
        st_smem(base + voff[k2], v[k2]);  // phase B reads the sum back (same thread)
      }
      if (store_ro) {
#pragma unroll
        for (int k2 = 0; k2 < NV; ++k2) {
          if constexpr (FULL)
            st_stream(rorow + voff[k2], v[k2]);
          else
            st_stream_if(vok[k2], rorow + voff[k2], v[k2]);
        }
      }
    }
    // Squares per vector pair, then the vectors, then the pair, then the
    // warp butterfly: the order of the single-pass kernel.
    float2 acc[NV];
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      acc[k2] = sq_first(v[k2][0]);
#pragma unroll
      for (int j = 1; j < 4; ++j) sq_acc(acc[k2], v[k2][j]);
    }
#pragma unroll
    for (int k2 = 1; k2 < NV; ++k2) acc[0] = __fadd2_rn(acc[0], acc[k2]);
    const float ss = warp_reduce<false>(__fadd_rn(acc[0].x, acc[0].y));
    // every lane holds the warp's sum: all store it (one value) and arrive
    // (release: orders the store before the arrival), no branch
    const int slot = k & (kPipeRing - 1);
    part[slot][warp] = ss;
    mbar_arrive(smem_addr(&red_bar[slot]));
  };

  // ---------------------------------------------------------------- finisher
  // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))), not a correctly rounded
  // reciprocal square root; the double rounding is reproduced. The mean is
  // RN(ss / H) through the one-correction division (a quotient below the
  // normal range takes the IEEE one).
  auto finalize = [&](int k) {
    const int slot = k & (kPipeRing - 1);
    const uint32_t par = (uint32_t)(k >> 2) & 1u;
    ok &= mbar_wait_abortable(smem_addr(&red_bar[slot]), par, abortp, a.wait_limit);
    const float total = combine_partials<false>(part[slot], lane, nw);
    float mean = div_rn(total, (float)a.H, a.rcp_H);
    if (mean < 0x1p-100f) mean = __fdiv_rn(total, (float)a.H);
    if (lane == 0) {
      inv_slot[slot] = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
      mbar_arrive(smem_addr(&inv_bar[slot]));
    }
  };

  // ---------------------------------------------------------------- phase B
  auto phase_b = [&](int k, int s, uint32_t use, int64_t row, uint8_t* qrow, char* srow,
                     uint8_t* norow) {
    const int slot = k & (kPipeRing - 1);
    const uint32_t par = (uint32_t)(k >> 2) & 1u;
    // The row has been in this stage since phase A and the weights never
    // change: both are read, and the stage released, before the wait for
    // inv_rms, so their latency overlaps it and the refill starts earlier.
    const uint32_t base = ring + (uint32_t)s * stage_bytes;
    uint32_t v[NV][4];
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      const uint4 u = ld_smem(base + voff[k2]);
      v[k2][0] = u.x;
      v[k2][1] = u.y;
      v[k2][2] = u.z;
      v[k2][3] = u.w;
    }
    // Count this warp out of the stage; the last warp refills it. The
    // acq_rel add orders every lane's reads (joined by __syncwarp) before the
    // refill, and the proxy fence orders them before the copy engine's writes.
    // No refill once the CTA is aborting: a warp whose wait for this stage's
    // copy gave up set the abort flag before it counted out, so the last warp
    // sees the flag, and the copy that may still be landing in the stage is
    // the only one there when the CTA drains.
    __syncwarp();
    if (lane == 0) {
      const uint32_t old = atom_add_acq_rel(smem_addr(&done_cnt[s]), 1u);
      if (old + 1u == (use + 1u) * (uint32_t)nw && k + S < nrows && !*abortp) {
        fence_proxy_async_smem();
        issued_cnt[s] = use + 2u;
        issue(s, row + (int64_t)S * G);
      }
    }
    uint32_t w[NV][4];
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) {
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (FULL || vok[k2]) u = ld_keep(wbase + voff[k2]);
      w[k2][0] = u.x;
      w[k2][1] = u.y;
      w[k2][2] = u.z;
      w[k2][3] = u.w;
    }
    ok &= mbar_wait_abortable(smem_addr(&inv_bar[slot]), par, abortp, a.wait_limit);
    const float inv = inv_slot[slot];
    const float2 inv2 = make_float2(inv, inv);
    {
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[k2][j] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[k2][j]), inv2)), w[k2][j]);
      if (store_no) {
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
          if constexpr (FULL)
            st_stream(norow + voff[k2], v[k2]);
          else
            st_stream_if(vok[k2], norow + voff[k2], v[k2]);
        }
      }
      if constexpr (QM == kQGroup && ILV) {
        // Two 1x128 groups an octet: slots 0-1 belong to group A, slots 2-3
        // to group B. Both maxima travel in one bf16 pair
        // (A low, B high) through the octet's three butterfly steps.
        const uint32_t pa = absmax_bf2(vec_absmax(v[0]), vec_absmax(v[1]));
        const uint32_t pb = absmax_bf2(vec_absmax(v[2]), vec_absmax(v[3]));
        // (the sign bits of absmax results are meaningless: combine magnitudes
        // once more, then clear them before any plain max)
        uint32_t p =
            absmax_bf2(__byte_perm(pa, pb, 0x5410), __byte_perm(pa, pb, 0x7632)) & 0x7fff7fffu;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
        const float2 am = bf2_to_f2(p);
        const float sa = make_scale(am.x, kPow2), sb = make_scale(am.y, kPow2);
        float ra, rb;
        if constexpr (kPow2) {  // exact reciprocals of powers of two: negate the exponent
          ra = __uint_as_float((254u << 23) - __float_as_uint(sa));
          rb = __uint_as_float((254u << 23) - __float_as_uint(sb));
        } else {
          ra = rcp_scale(sa);
          rb = rcp_scale(sb);
        }
        // lanes 0 and 1 of the octet write the scales of groups A and B
        put_group_scale<SK>(gput && (FULL || gidx * 16 < a.V), a, row, srow, goff, gidx,
                            (lane & 1) ? sb : sa);
        if constexpr (SK == kSkE8Swz)
          if (a.n_groups_pad > a.n_groups) zero_scale_padding(a, row, a.n_groups, t, T);
        uint32_t* qthr = reinterpret_cast<uint32_t*>(qrow + (int64_t)tvec * 8);
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
          const float rcs = k2 < 2 ? ra : rb, ns = k2 < 2 ? -sa : -sb;
          const float2 rc2 = make_float2(rcs, rcs), nb = make_float2(ns, ns);
          float2 y[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (kPow2)
              y[j] = __fmul2_rn(bf2_to_f2(v[k2][j]), rc2);  // n * 2^-e is exact
            else
              y[j] = div2_rn(bf2_to_f2(v[k2][j]), nb, rc2);
          }
          // 8 codes of vector tvec + 8 k2: an octet writes 64 contiguous bytes
          if constexpr (FULL)
            st_stream2(qthr + 16 * k2, f4_to_e4m3x4(y[0], y[1]), f4_to_e4m3x4(y[2], y[3]));
          else
            st_stream2_if(vok[k2], qthr + 16 * k2, f4_to_e4m3x4(y[0], y[1]),
                          f4_to_e4m3x4(y[2], y[3]));
        }
      } else if constexpr (QM == kQGroup) {
        // chunk maximum, combined over the LPG lanes of the group
        uint32_t p = absmax_bf2(absmax_bf2(vec_absmax(v[0]), vec_absmax(v[1])),
                                absmax_bf2(vec_absmax(v[2]), vec_absmax(v[3]))) &
                     0x7fff7fffu;
        p = max_bf2(p, p >> 16);
#pragma unroll
        for (int o = LPG / 2; o > 0; o >>= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
        const float sc = make_scale(__uint_as_float(p << 16), kPow2);
        // a power-of-two scale has an exact reciprocal: negate the exponent
        const float rc = kPow2 ? __uint_as_float((254u << 23) - __float_as_uint(sc)) : rcp_scale(sc);
        put_group_scale<SK>(gput, a, row, srow, goff, gidx, sc);
        if constexpr (SK == kSkE8Swz)
          if (a.n_groups_pad > a.n_groups) zero_scale_padding(a, row, a.n_groups, t, T);
        const float2 rc2 = make_float2(rc, rc), nb = make_float2(-sc, -sc);
        uint32_t cw[4][2];
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
          float2 y[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (kPow2)
              y[j] = __fmul2_rn(bf2_to_f2(v[k2][j]), rc2);  // n * 2^-e is exact
            else
              y[j] = div2_rn(bf2_to_f2(v[k2][j]), nb, rc2);
          }
          cw[k2][0] = f4_to_e4m3x4(y[0], y[1]);
          cw[k2][1] = f4_to_e4m3x4(y[2], y[3]);
        }
        // back to vector order, whole 32-byte sectors where the rows allow
        uint32_t d[8];
        unrotate_chunk(cw, 0, rot, d);
        store_chunk_codes<FULL>(qrow + 32 * t, d, q32, q16, 4 * t, a.V);
      }
    }
  };

  // ------------------------------------------------------------ main loop
  const int64_t q_step = G * a.ldq, s_step = G * a.s_row * kEsz, n_step = G * a.ldn * 2,
                r_step = G * a.ldro * 2;
  uint8_t* qrow = a.q + (int64_t)blockIdx.x * a.ldq;
  char* srow = static_cast<char*>(a.scale) + (int64_t)blockIdx.x * a.s_row * kEsz;
  uint8_t* norow = reinterpret_cast<uint8_t*>(a.norm_out) + (int64_t)blockIdx.x * a.ldn * 2;
  uint8_t* rorow = reinterpret_cast<uint8_t*>(a.res_out) + (int64_t)blockIdx.x * a.ldro * 2;
  int sB = 0, sA = 0;           // stages of rows k (phase B) and k + 1 (phase A)
  uint32_t useB = 0, useA = 0;  // how many times the ring wrapped at those rows
  int fin = 0;                  // k % nw
  const int nr = (int)nrows;    // the host keeps rows per CTA below 2^31
  if (nr > 0) {
    phase_a(0, 0, 0u, rorow);
    rorow += r_step;
  }
  int64_t row = blockIdx.x;
  // A failed wait does not branch out of a phase (the rows it touches are
  // garbage, never out of bounds); the warp leaves at the end of the row.
  for (int k = 0; k < nr; ++k, row += G) {
    if (warp == fin) finalize(k);
    if (++fin == nw) fin = 0;
    if (++sA == S) {
      sA = 0;
      ++useA;
    }
    if (k + 1 < nr) {
      phase_a(k + 1, sA, useA & 1u, rorow);
      rorow += r_step;
    }
    phase_b(k, sB, useB, row, qrow, srow, norow);
    if (++sB == S) {
      sB = 0;
      ++useB;
    }
    qrow += q_step;
    srow += s_step;
    norow += n_step;
    if (!__all_sync(0xffffffffu, ok)) break;
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0) {
    atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
    abort_flag = 1u;
  }
  __syncthreads();
  if (abort_flag) {
    // let every copy that was issued land (bounded) before the CTA exits
    if (t == 0)
      for (int s = 0; s < S; ++s)
        if (issued_cnt[s] > 0)
          mbar_wait_bounded(smem_addr(&full_bar[s]), (issued_cnt[s] - 1u) & 1u, kDrainLimitCycles);
    return;
  }
  if constexpr (SK == kSkE8Swz)  // swizzled-layout padding rows: scales only
    for (int64_t r = blockIdx.x + nrows * G; r < a.M_pad; r += G) zero_scale_padding(a, r, 0, t, T);
}

}  // namespace cutie
