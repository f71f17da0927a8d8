// Fused RMSNorm -> MXFP8 quantization -> block-scaled GEMM on the tensor
// cores (sm_100a): the GEMM's A operand is produced from the bf16 rows of x
// inside the GEMM, so its e4m3 codes and e8m0 scales never go to HBM.
//
//   n = bf16(bf16(x * inv_rms) * w)               (per row of x [M, K], as the forward)
//   s = 2^ceil(log2(max(amax32(n) / 448, 1e-4)))  (per 1x32 group; e8m0)
//   q = e4m3(n / s)
//   D[M, N] (bf16) = sum_k q[m, k] s[m, k/32] * B[n, k] sB[n, k/32]
//
// A and its scales are exactly what cutie_rms_norm_fp8 (group 32, e8m0,
// swizzled) writes for x; D is what cutie_gemm_mxfp8 computes from them.
//
// One CTA computes one 128 x 128 tile of D; the kernel is built for the
// decode-size batches this fusion pays for (a 128-row block of x is small
// next to the N x K weight the tile streams).
//
//  * inv_rms needs whole rows before the first K block. The CTAs that share
//    a 128-row block of x form a thread-block cluster of C CTAs along N and
//    split the columns: CTA c loads columns [c K/C, (c+1) K/C) of the block's
//    rows with one TMA box a round (up to the staging area's rows), sums
//    their squares, and writes its partial sums into every CTA of the cluster
//    (distributed shared memory). After a cluster barrier each CTA adds the C
//    partials in rank order, so all of them derive the same inv_rms bits.
//  * The K loop is then independent per CTA (no cluster traffic): warp 6
//    streams the block's x rows through a TMA ring (128-byte swizzled boxes
//    of 64 columns x 2 x 32 rows, one box per 32-row quarter with data), warps
//    0-3 normalise, take the 1x32 maxima, scale and convert them into the A
//    stage (K-major, 128-byte swizzle) and its scale atom, warp 4 streams the
//    weight tiles and their scale atoms through a deeper TMA ring, and one
//    thread of warp 5 issues tcgen05.mma.kind::mxf8f6f4.block_scale into
//    tensor memory (scales copied in with tcgen05.cp). Warps 0-3 finish with
//    the epilogue (tcgen05.ld, bf16, streaming stores).
//
// The x rows and the weight are read with plain TMA / bulk loads of this
// GPU's memory; nothing is multicast. Rows of a block past M are zero in A
// and are not stored. Every mbarrier wait is bounded: one that gives up sets
// the CTA's abort flag and the device error word (code 1); each CTA lets its
// own copies land before it leaves, and all threads still reach the cluster
// barriers, which are the only unbounded waits and have no dependencies.
#include "cutie.h"
#include "launch.cuh"
#include "tcgen05.cuh"

namespace cutie {

// This translation unit's device error word is g_cutie_device_error
// (fused_kernel.cuh: one copy per translation unit).
cudaError_t device_error_prologue(int* out, bool clear) { return read_device_error(out, clear); }

namespace {

constexpr int kTM = 128, kTN = 128, kTK = 128;  // tile; K in elements
constexpr uint32_t kTile = 16384;               // one 128 x 128 e4m3 tile
constexpr uint32_t kAtom = 512;                 // one 128 x 4 e8m0 scale atom
constexpr int kSA = 4;                          // A stages: one per quantizing warp
constexpr int kProducerWarps = 4;
constexpr int kProducers = kProducerWarps * 32;
constexpr int kWarpB = 4, kWarpMma = 5, kWarpX = 6;
constexpr int kThreads = 7 * 32;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kAccCol = 0, kSfCol = 128;  // K block kb: kSfCol + 8 (kb % 4) (A), + 4 (B)
constexpr int kBarProducers = 1;               // named barrier of the quantizing warps
constexpr int kBarPass1 = 2;                   // named barrier of pass 1 (warps 0-3 and 5)
constexpr int kPass1Threads = 5 * 32;

struct ProArgs {
  const uint16_t* w;  // [K]
  const uint8_t* sfb;
  uint16_t* d;
  int64_t ldd;        // elements
  uint8_t* q;         // optional: the A codes [M, K]
  int64_t ldq;
  uint8_t* qs;        // optional: the A scales, swizzled
  int M;
  int K;
  int pass1_rows;     // rows of one pass-1 box
  float eps;
  float rcp_K;
  long long wait_limit;
};

// QB: 32-row quarters of a block with data (1-4), fixed per launch from M.
template <int QB>
struct Plan {
  static constexpr uint32_t kXStage = (uint32_t)QB * 8192u;  // QB boxes of 32 rows x 128 bf16
  static constexpr int XS = QB <= 2 ? 4 : 2;                 // x ring stages
  static constexpr int SB = QB == 1 ? 7 : QB == 3 ? 6 : 5;    // B ring stages
  static constexpr uint32_t kOffA = 0;
  static constexpr uint32_t kOffSfA = kSA * kTile;
  static constexpr uint32_t kOffW = kOffSfA + kSA * kAtom;  // XS chunks of 128 weights
  static constexpr uint32_t kOffX = (kOffW + XS * 256u + 1023u) & ~1023u;
  static constexpr uint32_t kOffB = kOffX + XS * kXStage;
  static constexpr uint32_t kOffSfB = kOffB + SB * kTile;
  static constexpr uint32_t kBytes = kOffSfB + SB * kAtom;
  static constexpr size_t kSmem = kBytes + 1024;  // + alignment of the base to 1 KB
  // pass 1 stages its boxes over the A tiles only: the x and B rings fill meanwhile
  static constexpr uint32_t kStageArea = kOffSfA;

  static_assert(kOffX % 1024 == 0 && kOffB % 1024 == 0, "swizzled tiles on 1 KB boundaries");
  static_assert(kSmem + 1024 <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void st_smem_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_smem_u8(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

template <int C, int QB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_rmsnorm_mxfp8_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_xs,
                              const __grid_constant__ CUtensorMap map_b, const ProArgs a) {
  using P = Plan<QB>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_a[kSA], empty_a[kSA];
  __shared__ __align__(8) uint64_t full_b[P::SB], empty_b[P::SB];
  // x_full is indexed by K block mod 4 (the quantizing warp that waits on
  // it), x_empty by x stage: each waiter then trails its barrier by at most
  // one phase even when the x ring has fewer stages than there are warps
  __shared__ __align__(8) uint64_t x_full[kProducerWarps], x_empty[P::XS];
  __shared__ __align__(8) uint64_t stage_bar, acc_bar;
  __shared__ float part[C][kTM];  // partial sums of squares from every CTA of the cluster
  __shared__ float inv_s[kTM];    // inv_rms of the block's rows
  __shared__ uint32_t tmem_slot, abort_flag;
  __shared__ uint32_t issued_b[P::SB], issued_x[kProducerWarps];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const uint32_t crank = C > 1 ? tc::cluster_ctarank() : 0u;
  const int n0 = blockIdx.x * kTN;
  const int64_t m0 = (int64_t)blockIdx.y * kTM;
  const int Mr = (int)((int64_t)a.M - m0 < kTM ? (int64_t)a.M - m0 : kTM);  // rows with data
  const int nq = (Mr + 31) >> 5;  // quarters with data (<= QB)
  const int KB = a.K / kTK;
  volatile uint32_t* abortp = &abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSA; ++s) {
      mbar_init(smem_addr(&full_a[s]), 1);
      mbar_init(smem_addr(&empty_a[s]), 1);
    }
    for (int s = 0; s < P::SB; ++s) {
      mbar_init(smem_addr(&full_b[s]), 1);
      mbar_init(smem_addr(&empty_b[s]), 1);
      issued_b[s] = 0;
    }
    for (int s = 0; s < kProducerWarps; ++s) {
      mbar_init(smem_addr(&x_full[s]), 1);
      issued_x[s] = 0;
    }
    for (int s = 0; s < P::XS; ++s) mbar_init(smem_addr(&x_empty[s]), 1);
    mbar_init(smem_addr(&stage_bar), 1);
    mbar_init(smem_addr(&acc_bar), 1);
    abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == kWarpMma) tc::tmem_alloc(smem_addr(&tmem_slot), kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_slot;
  tc::cluster_sync();  // the part[] arrays of every CTA exist before peers write them
  griddep_wait();      // x, w and B written by the previous kernel are complete
  griddep_launch_dependents();

  // Neither stream depends on pass 1: the B and x producers start at once and
  // fill their rings while pass 1 runs (pass 1 stages in the A tiles only).
  // Their warps arrive on the end-of-pass-1 cluster barrier first (they have
  // no part in pass 1) and wait on it only after streaming.
  if (warp == kWarpX) {
    tc::cluster_arrive();
    if (lane == 0) {
      for (int kb = 0; kb < KB; ++kb) {
        const int xs = kb % P::XS;
        const uint32_t use = (uint32_t)(kb / P::XS);
        if (use > 0 &&
            !mbar_wait_abortable(smem_addr(&x_empty[xs]), (use - 1u) & 1u, abortp, a.wait_limit))
          break;
        const uint32_t bar = smem_addr(&x_full[kb % kProducerWarps]);
        issued_x[kb % kProducerWarps] = (uint32_t)(kb / kProducerWarps) + 1u;
        mbar_arrive_expect_tx(bar, (uint32_t)nq * 8192u + 256u);
        for (int q = 0; q < nq; ++q)
          tc::tma_load_3d(base + P::kOffX + (uint32_t)xs * P::kXStage + (uint32_t)q * 8192u,
                          &map_x, 0, 2 * kb, (int)(m0 + 32 * q), bar);
        bulk_g2s(base + P::kOffW + 256u * (uint32_t)xs, a.w + kb * kTK, 256u, bar);
      }
    }
    __syncwarp();
    tc::cluster_wait();
  } else if (warp == kWarpB) {
    tc::cluster_arrive();
    if (lane == 0) {
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % P::SB;
      const uint32_t use = (uint32_t)(kb / P::SB);
      if (use > 0 &&
          !mbar_wait_abortable(smem_addr(&empty_b[s]), (use - 1u) & 1u, abortp, a.wait_limit))
        break;
      const uint32_t bar = smem_addr(&full_b[s]);
      issued_b[s] = use + 1u;
      mbar_arrive_expect_tx(bar, kTile + kAtom);
      tc::tma_load_2d(base + P::kOffB + (uint32_t)s * kTile, &map_b, kb * kTK, n0, bar);
      bulk_g2s(base + P::kOffSfB + (uint32_t)s * kAtom,
               a.sfb + ((int64_t)blockIdx.x * KB + kb) * kAtom, kAtom, bar);
    }
    }
    __syncwarp();
    tc::cluster_wait();
  } else {
  // ------------------------------------------------ pass 1: sums of squares
  // (warps 0-3 and 5; the two streaming warps are busy)
  bool pass1_failed = false;
  {
    const int pw = warp < kProducerWarps ? warp : kProducerWarps;  // 0..4
    const int pt = pw * 32 + lane;                                  // 0..159
    const int KC = a.K / C;  // columns of this CTA's slice
    const uint32_t SBy = (uint32_t)KC * 2u;
    const int RR = a.pass1_rows;  // rows of one box (host: RR * SBy <= kStageArea)
    uint32_t par = 0;
    for (int r0 = 0; r0 < Mr; r0 += RR) {
      const int nr = Mr - r0 < RR ? Mr - r0 : RR;
      if (threadIdx.x == 0) {
        tc::fence_async_smem();  // the previous round's reads come before these writes
        mbar_arrive_expect_tx(smem_addr(&stage_bar), (uint32_t)RR * SBy);
        tc::tma_load_3d(base, &map_xs, 0, (int)crank * (KC / 64), (int)(m0 + r0),
                        smem_addr(&stage_bar));
      }
      {
        if (__all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&stage_bar), par, a.wait_limit))) {
          for (int j = pw; j < nr; j += kPass1Threads / 32) {
            const uint32_t row = base + (uint32_t)j * SBy;
            float2 acc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
            int v = lane;
            for (; v + 96 < KC / 8; v += 128) {  // four loads in flight a lane
              uint4 u[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) u[i] = ld_smem(row + 16u * (v + 32 * i));
#pragma unroll
              for (int i = 0; i < 4; ++i)
                sq_acc(acc[i], u[i].x), sq_acc(acc[i], u[i].y), sq_acc(acc[i], u[i].z),
                    sq_acc(acc[i], u[i].w);
            }
            for (; v < KC / 8; v += 32) {
              const uint4 u = ld_smem(row + 16u * v);
              sq_acc(acc[0], u.x), sq_acc(acc[0], u.y), sq_acc(acc[0], u.z), sq_acc(acc[0], u.w);
            }
            acc[0] = make_float2(__fadd_rn(acc[0].x, acc[1].x), __fadd_rn(acc[0].y, acc[1].y));
            acc[2] = make_float2(__fadd_rn(acc[2].x, acc[3].x), __fadd_rn(acc[2].y, acc[3].y));
            acc[0] = make_float2(__fadd_rn(acc[0].x, acc[2].x), __fadd_rn(acc[0].y, acc[2].y));
            const float ss = warp_reduce<false>(__fadd_rn(acc[0].x, acc[0].y));
            if constexpr (C > 1) {
              if (lane < C)
                tc::st_cluster_f32(tc::mapa(smem_addr(&part[crank][r0 + j]), (uint32_t)lane), ss);
            } else if (lane == 0) {
              part[0][r0 + j] = ss;
            }
          }
        } else {
          *abortp = 1u;
        }
      }
      par ^= 1u;
      asm volatile("bar.sync %0, %1;" ::"n"(kBarPass1), "n"(kPass1Threads) : "memory");
      if (*abortp) {  // written only before the barrier above: every thread agrees
        if (threadIdx.x == 0)  // let the round's box land before the memory is reused
          mbar_wait_bounded(smem_addr(&stage_bar), par ^ 1u, kDrainLimitCycles);
        pass1_failed = true;
        break;
      }
    }
    // A rows without data stay zero for the rest of the launch (codes and
    // scale bytes); pass 1 used this memory, so they are cleared only now
    if (Mr < kTM) {
      const uint32_t zero4[4] = {0u, 0u, 0u, 0u};
      for (int s = 0; s < kSA; ++s) {
        for (uint32_t off = (uint32_t)Mr * 128u + 16u * pt; off < kTile; off += 16u * kPass1Threads)
          st_smem(base + P::kOffA + (uint32_t)s * kTile + off, zero4);
        for (int r = Mr + pt; r < kTM; r += kPass1Threads)
          st_smem_u32(base + P::kOffSfA + (uint32_t)s * kAtom +
                          (uint32_t)((r & 31) * 16 + (r >> 5) * 4),
                      0u);
      }
      tc::fence_async_smem();  // before the MMAs read them
    }
  }
  // all partial sums are in every CTA of the cluster (release / acquire)
  tc::cluster_arrive();
  tc::cluster_wait();

  // ------------------------------------------------ pass 2: the K loop
  if (pass1_failed) {
    *abortp = 1u;  // the streaming producers stop at their next wait
  } else if (warp == kWarpMma && lane == 0) {
    for (int kb = 0; kb < KB; ++kb) {
      const int sa = kb % kSA, sb = kb % P::SB;
      if (!mbar_wait_abortable(smem_addr(&full_a[sa]), (uint32_t)(kb / kSA) & 1u, abortp,
                               a.wait_limit) ||
          !mbar_wait_abortable(smem_addr(&full_b[sb]), (uint32_t)(kb / P::SB) & 1u, abortp,
                               a.wait_limit))
        break;
      tc::fence_after();
      const uint32_t sfa_col = tmem + kSfCol + 8u * (uint32_t)(kb & 3), sfb_col = sfa_col + 4u;
      tc::copy_sf(sfa_col, tc::smem_desc(base + P::kOffSfA + (uint32_t)sa * kAtom, 0, 128,
                                         tc::kLayoutNone));
      tc::copy_sf(sfb_col, tc::smem_desc(base + P::kOffSfB + (uint32_t)sb * kAtom, 0, 128,
                                         tc::kLayoutNone));
#pragma unroll
      for (int kk = 0; kk < kTK / 32; ++kk) {
        const uint64_t ad = tc::smem_desc(base + P::kOffA + (uint32_t)sa * kTile + 32u * kk, 16,
                                          1024, tc::kLayoutSw128);
        const uint64_t bd = tc::smem_desc(base + P::kOffB + (uint32_t)sb * kTile + 32u * kk, 16,
                                          1024, tc::kLayoutSw128);
        tc::mma_mxf8(tmem + kAccCol, ad, bd, tc::mxf8_idesc(kTM, kTN, (uint32_t)kk), sfa_col,
                     sfb_col, (kb | kk) != 0);
      }
      tc::commit(smem_addr(&empty_a[sa]));  // both stages are free once these MMAs are done
      tc::commit(smem_addr(&empty_b[sb]));
    }
  } else if (warp < kProducerWarps) {
    // ---- quantize the block's rows: warp w makes K blocks w, w + 4, ...,
    // so four K blocks are in the making at once and no warp waits for another
    const int t = threadIdx.x;
    if (t < Mr) {
      float ss = part[0][t];
#pragma unroll
      for (int c = 1; c < C; ++c) ss = __fadd_rn(ss, part[c][t]);
      // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))); the mean is RN(ss / K)
      float mean = div_rn(ss, (float)a.K, a.rcp_K);
      if (mean < 0x1p-100f) mean = __fdiv_rn(ss, (float)a.K);
      inv_s[t] = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
    }
    asm volatile("bar.sync %0, %1;" ::"n"(kBarProducers), "n"(kProducers) : "memory");
    const int j = lane & 7;  // 16-column chunk of the K block; rows (lane / 8) + 4 i
    const bool store_q = a.q != nullptr && blockIdx.x == 0;  // one CTA a block writes q
    for (int kb = warp; kb < KB; kb += kProducerWarps) {
      const int sa = kb % kSA, xs = kb % P::XS;
      bool ok = mbar_wait_abortable(smem_addr(&x_full[warp]),
                                    (uint32_t)(kb / kProducerWarps) & 1u, abortp, a.wait_limit);
      if (ok && kb >= kSA)
        ok = mbar_wait_abortable(smem_addr(&empty_a[sa]), (uint32_t)(kb / kSA - 1) & 1u, abortp,
                                 a.wait_limit);
      if (!__all_sync(0xffffffffu, ok)) {  // the warp acts as one
        *abortp = 1u;
        break;
      }
      const uint32_t w_st = base + P::kOffW + 256u * (uint32_t)xs + 32u * (uint32_t)j;
      const uint4 w0 = ld_smem(w_st), w1 = ld_smem(w_st + 16u);
      const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const uint32_t a_st = base + P::kOffA + (uint32_t)sa * kTile;
      const uint32_t sf_st = base + P::kOffSfA + (uint32_t)sa * kAtom;
      const uint32_t x_st = base + P::kOffX + (uint32_t)xs * P::kXStage;
#pragma unroll 4
      for (int i = 0; i < 8 * QB; ++i) {
        const int m = (lane >> 3) + 4 * i;  // tile row
        if (!__any_sync(0xffffffffu, m < Mr)) break;
        // line L of quarter m/32 holds columns 64 h .. 64 h + 63 of row m;
        // 16-byte piece p of a line sits at p ^ (L % 8) (128-byte swizzle)
        const uint32_t L = (uint32_t)(m & 31) * 2u + (uint32_t)(j >> 2);
        const uint32_t sub = x_st + (uint32_t)(m >> 5) * 8192u + L * 128u;
        const uint32_t p0 = (uint32_t)(2 * j) & 7u;
        const uint4 x0 = ld_smem(sub + ((p0 ^ (L & 7u)) << 4));
        const uint4 x1 = ld_smem(sub + (((p0 + 1u) ^ (L & 7u)) << 4));
        uint32_t v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const float iv = m < Mr ? inv_s[m] : 0.f;
        const float2 inv2 = make_float2(iv, iv);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          v[k] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[k]), inv2)), wv[k]);
        // 1x32 group = this chunk and its neighbour (lane ^ 1)
        uint32_t am = absmax_bf2(absmax_bf2(absmax_bf2(v[0], v[1]), absmax_bf2(v[2], v[3])),
                                 absmax_bf2(absmax_bf2(v[4], v[5]), absmax_bf2(v[6], v[7])));
        am &= 0x7fff7fffu;
        am = max_bf2(am, am >> 16);
        am = max_bf2(am, __shfl_xor_sync(0xffffffffu, am, 1)) & 0xffffu;
        const float sc = make_scale(__uint_as_float(am << 16), true);
        const uint32_t e8 = __float_as_uint(sc) >> 23;
        const float rc = __uint_as_float((254u << 23) - __float_as_uint(sc));  // exact
        const float2 rc2 = make_float2(rc, rc);
        uint32_t c4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          c4[k] = f4_to_e4m3x4(__fmul2_rn(bf2_to_f2(v[2 * k]), rc2),
                               __fmul2_rn(bf2_to_f2(v[2 * k + 1]), rc2));
        if (m < Mr) {
          // K-major, 128-byte swizzled A tile: row m, 16-byte chunk j at j ^ (m % 8)
          st_smem(a_st + (uint32_t)m * 128u + (((uint32_t)j ^ ((uint32_t)m & 7u)) << 4), c4);
          if ((j & 1) == 0)
            st_smem_u8(sf_st + (uint32_t)((m & 31) * 16 + (m >> 5) * 4 + (j >> 1)), e8);
          if (store_q) {
            st_stream(a.q + (m0 + m) * a.ldq + kb * kTK + 16 * j, c4);
            if ((j & 1) == 0) a.qs[swizzled_offset(m0 + m, kb * 4 + (j >> 1), KB)] = (uint8_t)e8;
          }
        }
      }
      tc::fence_async_smem();  // the A stage writes come before the MMAs
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_addr(&x_empty[xs]));
        mbar_arrive(smem_addr(&full_a[sa]));
      }
    }
    // the scale rows of the padding past M in the last block, zero in q_scale
    if (store_q && Mr < kTM) {
      for (int m = Mr + t; m < kTM; m += kProducers)
        for (int g = 0; g < 4 * KB; ++g) a.qs[swizzled_offset(m0 + m, g, KB)] = 0;
    }
  }
  }  // warps other than the B producer
  // The MMA thread commits the accumulator once, after its last MMA (or
  // after it stopped); nobody else waits on acc_bar before this point.
  if (warp == kWarpMma && lane == 0) tc::commit(smem_addr(&acc_bar));
  __syncwarp();

  // ------------------------------------------------ epilogue (warps 0-3)
  if (warp < kProducerWarps) {
    // not cut short by an abort: the MMAs must be complete before tensor
    // memory is read or freed
    const bool acc_ok = __all_sync(
        0xffffffffu, mbar_wait_bounded(smem_addr(&acc_bar), 0u, kWaitLimitCycles) && *abortp == 0u);
    if (!acc_ok) *abortp = 1u;
    tc::fence_after();
    const int64_t row = m0 + warp * 32 + lane;
    if (acc_ok && __any_sync(0xffffffffu, row < a.M)) {
#pragma unroll 1
      for (int c = 0; c < kTN; c += 32) {
        uint32_t r[32];
        tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + kAccCol + (uint32_t)c, r);
        uint32_t o[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          o[k] = f2_to_bf2(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])));
        if (row < a.M) {
          uint8_t* p = reinterpret_cast<uint8_t*>(a.d + row * a.ldd + n0 + c);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t vv[4] = {o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]};
            st_stream(p + 16 * k, vv);
          }
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (*abortp != 0u && threadIdx.x == 0) {
    atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
    // this CTA's own loads land before its shared memory goes away
    for (int s = 0; s < P::SB; ++s)
      if (issued_b[s] > 0)
        mbar_wait_bounded(smem_addr(&full_b[s]), (issued_b[s] - 1u) & 1u, kDrainLimitCycles);
    for (int s = 0; s < kProducerWarps; ++s)
      if (issued_x[s] > 0)
        mbar_wait_bounded(smem_addr(&x_full[s]), (issued_x[s] - 1u) & 1u, kDrainLimitCycles);
  }
  __syncthreads();
  if (warp == kWarpMma) tc::tmem_dealloc(tmem, kTmemCols);
}

// x [M, K] bf16 as a 3-D tensor {64 columns, K / 64 column blocks, M rows}
// with boxes of {64, blocks, rows}: swizzled 128-byte lines for the K loop
// (2 blocks x 32 rows), plain rows for pass 1. Zero fill past the last row.
bool encode_x(CUtensorMap* map, const void* x, int64_t M, int64_t K, int64_t ldx, int blocks,
              int rows, bool swizzle) {
  auto fn = tc::encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {64, (cuuint64_t)(K / 64), (cuuint64_t)M};
  const cuuint64_t strides[2] = {128, (cuuint64_t)ldx * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)blocks, (cuuint32_t)rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int C, int QB>
cudaError_t launch_one(const void* x, int64_t M, int64_t K, int64_t ldx, const CUtensorMap& map_b,
                       ProArgs a, int64_t N, cudaStream_t stream, const char** why) {
  using P = Plan<QB>;
  const int64_t slice_bytes = K / C * 2;
  int rows = (int)(P::kStageArea / slice_bytes);
  const int block_rows = M < kTM ? (int)M : kTM;
  if (rows > block_rows) rows = block_rows;
  if (rows > 256) rows = 256;
  a.pass1_rows = rows;
  CUtensorMap map_x, map_xs;
  if (!encode_x(&map_x, x, M, K, ldx, 2, 32, true) ||
      !encode_x(&map_xs, x, M, K, ldx, (int)(K / 64 / C), rows, false)) {
    *why = "cuTensorMapEncodeTiled failed for x";
    return cudaErrorInvalidValue;
  }
  auto kernel = gemm_rmsnorm_mxfp8_kernel<C, QB>;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)P::kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / kTN), (unsigned)((M + kTM - 1) / kTM));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, map_x, map_xs, map_b, a);
}

template <int C>
cudaError_t launch_c(const void* x, int64_t M, int64_t K, int64_t ldx, const CUtensorMap& map_b,
                     const ProArgs& a, int64_t N, cudaStream_t stream, const char** why) {
  switch (M >= kTM ? 4 : (int)((M + 31) / 32)) {
    case 1: return launch_one<C, 1>(x, M, K, ldx, map_b, a, N, stream, why);
    case 2: return launch_one<C, 2>(x, M, K, ldx, map_b, a, N, stream, why);
    case 3: return launch_one<C, 3>(x, M, K, ldx, map_b, a, N, stream, why);
    default: return launch_one<C, 4>(x, M, K, ldx, map_b, a, N, stream, why);
  }
}

}  // namespace

// Cluster size of pass 1: the most CTAs (8, 4, 2, 1) that divide both the
// N tiles and the 64-column blocks of K.
int gemm_rmsnorm_cluster_size(int64_t N, int64_t K) {
  const int64_t nt = N / kTN, kc = K / 64;
  for (int c = 8; c > 1; c >>= 1)
    if (nt % c == 0 && kc % c == 0) return c;
  return 1;
}

int gemm_rmsnorm_mxfp8(const void* x, int64_t ldx, const void* weight, float eps, const void* b,
                       int64_t ldb, const void* b_scale, void* d, int64_t ldd, int64_t M,
                       int64_t N, int64_t K, void* q, int64_t ldq, void* q_scale,
                       long long wait_limit, cudaStream_t stream, const char** why) {
  CUtensorMap map_b;
  if (!tc::encode_e4m3_operand(&map_b, b, N, K, ldb)) {
    *why = "cuTensorMapEncodeTiled failed for b";
    return CUTIE_ERR_CUDA;
  }
  ProArgs a{};
  a.w = static_cast<const uint16_t*>(weight);
  a.sfb = static_cast<const uint8_t*>(b_scale);
  a.d = static_cast<uint16_t*>(d);
  a.ldd = ldd;
  a.q = static_cast<uint8_t*>(q);
  a.ldq = ldq;
  a.qs = static_cast<uint8_t*>(q_scale);
  a.M = (int)M;
  a.K = (int)K;
  a.eps = eps;
  a.rcp_K = 1.0f / (float)K;
  a.wait_limit = wait_limit;
  cudaError_t e;
  switch (gemm_rmsnorm_cluster_size(N, K)) {
    case 8: e = launch_c<8>(x, M, K, ldx, map_b, a, N, stream, why); break;
    case 4: e = launch_c<4>(x, M, K, ldx, map_b, a, N, stream, why); break;
    case 2: e = launch_c<2>(x, M, K, ldx, map_b, a, N, stream, why); break;
    default: e = launch_c<1>(x, M, K, ldx, map_b, a, N, stream, why); break;
  }
  if (e != cudaSuccess) {
    if (**why == '\0') *why = cudaGetErrorString(e);
    return CUTIE_ERR_CUDA;
  }
  return CUTIE_OK;
}

}  // namespace cutie
