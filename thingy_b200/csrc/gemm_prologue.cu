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
// swizzled) writes for x; D is what cutie_gemm_mxfp8 computes from them up
// to the order of the fp32 sums.
//
// Built for decode-size batches, where the N x K weight dominates the bytes
// and one 128 x 128 tile a CTA leaves most SMs idle: the S CTAs of a tile form
// a thread-block cluster and split K (S chosen on the host so that the grid
// fills the SMs once). CTA r of the cluster owns K blocks [r KB / S,
// (r+1) KB / S):
//
//  * pass 1 (sums of squares): warp 6 streams the block's x rows of those K
//    blocks through a TMA ring (128-byte swizzled boxes of 64 columns x 2 x
//    xr rows, xr = 32 or M rounded up to 8, one box per 32-row quarter with
//    data, plus the 128 RMSNorm weights of the K block). When every K block
//    of the CTA fits a stage of its own (decode batches) the ring is
//    resident: each stage is loaded once and read by both passes. Warps 0-3
//    add the squares, reduce each row over its 8 lanes and write the row's
//    partial sum into every CTA of the cluster (distributed shared memory).
//    After a cluster barrier every CTA adds the S partials in rank order:
//    the same inv_rms bits everywhere.
//    The x loads are issued before the first weight tiles, so that pass 1
//    does not queue behind the weight ring.
//  * pass 2: quantizing warp w makes the A tile of every 4th K block
//    (normalise, 1x32 maxima, e8m0 scales, e4m3 codes into a K-major
//    128-byte-swizzled A stage and its 512-byte scale atom), so four K blocks
//    are in the making at once; warp 4 streams the weight tiles and their
//    scale atoms; one thread of warp 5 copies the scale atoms to tensor
//    memory (tcgen05.cp) and issues tcgen05.mma.kind::mxf8f6f4.block_scale
//    into a 128 x 128 fp32 accumulator in tensor memory.
//  * reduction: once every CTA's MMAs are done, the others store their
//    accumulator rows with data straight into the leader's (rank 0) shared
//    memory (or, when they do not fit, keep them for the leader to read
//    over distributed shared memory); after a cluster barrier the leader
//    adds them to its own accumulator in rank order, rounds to bf16 and
//    stores D.
//
// Every load is a plain TMA or bulk copy of this GPU's own memory; nothing is
// multicast. Rows of a block past M are never written in A: row m of D
// depends only on row m of A, and those rows of D are not stored. Every
// mbarrier wait is bounded: one that gives up sets the CTA's abort flag and
// the device error word (code 1), the CTA lets its own copies land, and every
// thread still reaches the cluster barriers (the only unbounded waits, which
// depend on nothing but the other threads reaching them). No barrier is ever
// arrived on while its current phase is incomplete, and no waiter runs more
// than one phase ahead of its barrier (see x_full below).
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
constexpr int kProducerWarps = 4;
constexpr int kMaxSA = kProducerWarps;  // A stages: one per quantizing warp of pass 2
constexpr int kProducers = kProducerWarps * 32;
constexpr int kWarpB = 4, kWarpMma = 5, kWarpX = 6;
constexpr int kThreads = 7 * 32;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kAccCol = 0, kSfCol = 128;  // K block i: kSfCol + 8 (i % 4) (A), + 4 (B)
constexpr int kBarProducers = 1;               // named barrier of the quantizing warps
constexpr int kBarStreams = 2;                 // x warp -> weight warp: first x loads issued
constexpr int kMaxSplits = 8;

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
  int splits;         // S: CTAs of a cluster, each a contiguous range of K blocks
  int xr;             // rows of one x box (8, 16, 24 or 32)
  float eps;
  float rcp_K;
  long long wait_limit;
};

// QB: 32-row quarters of a block with data (1-4), fixed per launch from M.
// An x stage holds one K block of the block's rows: QB boxes of xr rows
// (xr = 32, or M rounded up to 8 when M < 32) x 128 bf16 columns, so a
// decode batch's stages are small and the ring holds up to kMaxXS of them.
constexpr int kMaxXS = 16;
constexpr uint32_t kStaticSmem = 5376;  // the kernel's __shared__ arrays (ptxas: at most 5.2 KB)
// SM (small): a block of at most 16 rows whose every K block has an x stage
// of its own. Pass 2 then writes each K block's A tile over its x stage (the
// 16-row A tile is no larger than the stage), so A needs no ring: the A
// tiles of three K blocks are released together, on one barrier, and the MMA
// thread waits once for those and once for the weight stage of the same
// three blocks. The weight is the MMA's 128-row M side and the block's rows
// its N = 16 side. (A K loop with one A stage a warp and a barrier hand-off
// for every K block ran at about 0.44 us a block; the stand-alone decode
// GEMM, one hand-off a three-block stage, at about 0.29.)
template <int QB, bool SM = false>
struct Plan {
  static_assert(!SM || QB == 1, "the small plan is for one 32-row quarter");
  static constexpr uint32_t kXRegion = SM ? 61440u : QB == 1 ? 32768u : QB == 3 ? 49152u : 65536u;
  // one A stage per quantizing warp (two warps and a 9-stage weight ring
  // measured slower from 16 rows on, and no faster below)
  static constexpr int kSA = kMaxSA;
  static constexpr int SB = SM ? 9 : QB == 1 ? 7 : QB == 3 ? 6 : 5;  // weight slots
  static constexpr int BG = SM ? 3 : 1;  // K blocks a weight stage
  static constexpr int NSB = SB / BG;    // weight stages
  static_assert(SB % BG == 0, "whole stages");
  static constexpr uint32_t kOffA = 0;  // A stages (SM: none, A is made over x)
  static constexpr uint32_t kOffSfA = SM ? kXRegion + kMaxXS * 256u : kSA * kTile;
  static constexpr uint32_t kOffW = SM ? kXRegion : kOffSfA + kSA * kAtom;  // chunks of 128 weights
  static constexpr uint32_t kOffX = SM ? 0u : kOffW + kMaxXS * 256u;
  static constexpr uint32_t kOffB = SM ? kOffSfA + kMaxXS * kAtom : kOffX + kXRegion;
  static constexpr uint32_t kOffSfB = kOffB + SB * kTile;
  static constexpr uint32_t kBytes = kOffSfB + SB * kAtom;
  static constexpr size_t kSmem = kBytes + 1024;  // + alignment of the base to 1 KB
  // after the K loop: the other CTAs' partial tiles (rows with data) fit below
  // kOffSfB (SM: in the x region)
  static constexpr uint32_t kPushArea = SM ? kXRegion : kOffSfB;
  // the partial rows (32 QB of them, 512 bytes each) fit the A stages
  static_assert(kSA * kTile >= 32u * QB * kTN * 4, "the partial tile fits the A stages");
  static_assert(!SM || (kMaxSplits - 1) * 16u * kTN * 4u <= kPushArea, "SM partials fit");
  static_assert(kOffX % 1024 == 0 && kOffB % 1024 == 0, "swizzled tiles on 1 KB boundaries");
  static_assert(kSmem + kStaticSmem <= 227 * 1024, "shared memory (with the static arrays)");
};

__device__ __forceinline__ void st_smem_u8(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Byte offset of (row, 4 columns c4) in the fp32 partial rows (rows < rows_
// with data): column groups outermost, so a warp's consecutive rows fill
// contiguous 16-byte slots (no bank conflicts).
__device__ __forceinline__ uint32_t part_off(int row, int c4, int rows) {
  return ((uint32_t)c4 * (uint32_t)rows + (uint32_t)row) * 16u;
}

template <int QB, bool SM>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_rmsnorm_mxfp8_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_b, const ProArgs a) {
  using P = Plan<QB, SM>;
  extern __shared__ uint8_t smem_raw[];
  constexpr int kSA = P::kSA;
  __shared__ __align__(8) uint64_t full_a[kMaxSA], empty_a[kMaxSA];
  __shared__ __align__(8) uint64_t full_b[P::SB], empty_b[P::SB];
  // x_full: in a resident ring one barrier per stage, each completing once;
  // otherwise indexed by x iteration mod 4 (in pass 2 that is a fixed
  // quantizing warp) with the ring at most 4 stages deep. Either way the
  // producer never arrives on a barrier whose current phase is incomplete,
  // and no waiter is more than one phase ahead of its barrier, although the
  // ring may have fewer stages than there are warps. x_empty by x stage.
  __shared__ __align__(8) uint64_t x_full[kMaxXS], x_empty[kMaxXS];
  __shared__ __align__(8) uint64_t acc_bar;
  // SM: A group g (K blocks 3 g .. 3 g + 2, the blocks of weight stage g) is
  // made when each of its blocks' warps has arrived once
  __shared__ __align__(8) uint64_t a_group[SM ? (kMaxXS + 2) / 3 : 1];
  __shared__ float part[kMaxSplits][kTM];  // row partial sums from every CTA of the cluster
  __shared__ float inv_s[kTM];             // inv_rms of the block's rows
  __shared__ float gsum[16];               // SM: the 8-lane groups' sums of squares
  __shared__ uint32_t tmem_slot, abort_flag;
  __shared__ uint32_t issued_b[P::SB], issued_x[kMaxXS];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int S = a.splits;
  const int rank = (int)blockIdx.z;  // = rank in the cluster (cluster dims 1 x 1 x S)
  const int n0 = blockIdx.x * kTN;
  const int64_t m0 = (int64_t)blockIdx.y * kTM;
  const int Mr = (int)((int64_t)a.M - m0 < kTM ? (int64_t)a.M - m0 : kTM);  // rows with data
  const int nq = (Mr + 31) >> 5;  // quarters with data (<= QB)
  const int KB = a.K / kTK;
  const int kb0 = rank * KB / S, kbs = (rank + 1) * KB / S - kb0;  // this CTA's K blocks
  const int xr = a.xr;
  const uint32_t xstage = (uint32_t)QB * (uint32_t)xr * 256u;
  int XS = (int)(P::kXRegion / xstage);
  if (XS > kMaxXS) XS = kMaxXS;
  // resident: every K block of this CTA has its own x stage, loaded once and
  // read by both passes
  const bool resident = kbs <= XS;
  if (!resident && XS > 4) XS = 4;
  const int x_iters = resident ? kbs : 2 * kbs;
  auto xf = [&](int it) { return resident ? it : (it & 3); };     // x_full index
  auto xp = [&](int it) { return resident ? 0u : (uint32_t)(it >> 2) & 1u; };  // its parity
  volatile uint32_t* abortp = &abort_flag;

  if (threadIdx.x == 0) {
    tc::prefetch_map(&map_x);
    tc::prefetch_map(&map_b);
    for (int s = 0; s < kSA; ++s) {
      mbar_init(smem_addr(&full_a[s]), 1);
      mbar_init(smem_addr(&empty_a[s]), 1);
    }
    for (int s = 0; s < P::SB; ++s) {
      mbar_init(smem_addr(&full_b[s]), 1);
      mbar_init(smem_addr(&empty_b[s]), 1);
      issued_b[s] = 0;
    }
    for (int s = 0; s < kMaxXS; ++s) {
      mbar_init(smem_addr(&x_full[s]), 1);
      issued_x[s] = 0;
    }
    // pass 1: each quantizing warp arrives; pass 2: the one warp, with count 4
    for (int s = 0; s < kMaxXS; ++s) mbar_init(smem_addr(&x_empty[s]), kProducerWarps);
    mbar_init(smem_addr(&acc_bar), 1);
    if constexpr (SM)
      for (int g = 0; g < (kMaxXS + 2) / 3; ++g)
        mbar_init(smem_addr(&a_group[g]), (uint32_t)max(1, min(3, kbs - 3 * g)));
    // the small plan needs every K block resident (the host only picks it then)
    abort_flag = SM && !resident ? 1u : 0u;
    mbar_init_fence();
  }
  if (warp == kWarpMma) tc::tmem_alloc(smem_addr(&tmem_slot), kTmemCols);
  // A rows past M are never written: row m of D depends only on row m of A,
  // and those rows of D are not stored
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_slot;
  // Set-up cluster barrier: every CTA of the cluster has started (its part[]
  // exists) before another writes it. Each thread arrives here and waits
  // only before its next cluster barrier or its first remote write, so the
  // loads into this CTA's own memory do not wait for the other CTAs.
  tc::cluster_arrive();
  griddep_wait();      // x, w and B written by the previous kernel are complete
  griddep_launch_dependents();

  // ---- streaming warps: they arrive on the end-of-pass-1 cluster barrier
  // before they could block (they have no part in pass 1) and wait on it
  // after streaming
  if (warp == kWarpX) {
    // x iterations 0 .. kbs-1 feed pass 1, kbs .. 2 kbs-1 pass 2 (a resident
    // ring keeps pass 1's stages for pass 2: kbs iterations). The first XS
    // need no wait; the weight stream starts once they are issued, so that
    // pass 1's rows are not queued behind a ring of weight tiles.
    const int x_first = x_iters < XS ? x_iters : XS;
    auto issue_x = [&](int it_begin, int it_end) {
      for (int it = it_begin; it < it_end; ++it) {
        const int xs = it % XS;
        if (it >= XS &&
            !mbar_wait_abortable(smem_addr(&x_empty[xs]), (uint32_t)(it / XS - 1) & 1u, abortp,
                                 a.wait_limit))
          break;
        const int kb = kb0 + (it < kbs ? it : it - kbs);
        const uint32_t bar = smem_addr(&x_full[xf(it)]);
        issued_x[xf(it)] = resident ? 1u : (uint32_t)(it >> 2) + 1u;
        mbar_arrive_expect_tx(bar, (uint32_t)nq * (uint32_t)xr * 256u + 256u);
        for (int q = 0; q < nq; ++q)
          tc::tma_load_3d(base + P::kOffX + (uint32_t)xs * xstage + (uint32_t)q * (uint32_t)xr * 256u,
                          &map_x, 0, 2 * kb, (int)(m0 + 32 * q), bar);
        bulk_g2s(base + P::kOffW + 256u * (uint32_t)xs, a.w + kb * kTK, 256u, bar);
      }
    };
    if (lane == 0) issue_x(0, x_first);
    __syncwarp();
    asm volatile("bar.arrive %0, %1;" ::"n"(kBarStreams), "n"(64) : "memory");
    tc::cluster_wait();     // set-up
    tc::cluster_arrive();   // end of pass 1
    if (lane == 0) issue_x(x_first, x_iters);
    __syncwarp();
    tc::cluster_wait();
  } else if (warp == kWarpB) {
    tc::cluster_wait();     // set-up
    tc::cluster_arrive();   // end of pass 1
    asm volatile("bar.sync %0, %1;" ::"n"(kBarStreams), "n"(64) : "memory");
    if (lane == 0) {
      // stage j holds K blocks BG j .. BG j + BG - 1 in slots BG (j % NSB) + ...
      const int nst = (kbs + P::BG - 1) / P::BG;
      for (int j = 0; j < nst; ++j) {
        const int s = j % P::NSB;
        if (j >= P::NSB &&
            !mbar_wait_abortable(smem_addr(&empty_b[s]), (uint32_t)(j / P::NSB - 1) & 1u, abortp,
                                 a.wait_limit))
          break;
        const int first = j * P::BG, nb = min(P::BG, kbs - first);
        const uint32_t bar = smem_addr(&full_b[s]);
        issued_b[s] = (uint32_t)(j / P::NSB) + 1u;
        mbar_arrive_expect_tx(bar, (uint32_t)nb * (kTile + kAtom));
        for (int i = 0; i < nb; ++i) {
          const uint32_t slot = (uint32_t)(s * P::BG + i);
          const int kb = kb0 + first + i;
          tc::tma_load_2d(base + P::kOffB + slot * kTile, &map_b, kb * kTK, n0, bar);
          bulk_g2s(base + P::kOffSfB + slot * kAtom, a.sfb + ((int64_t)blockIdx.x * KB + kb) * kAtom,
                   kAtom, bar);
        }
      }
    }
    __syncwarp();
    tc::cluster_wait();
  } else if (warp == kWarpMma) {
    tc::cluster_wait();     // set-up
    tc::cluster_arrive();   // the MMAs wait for A tiles, which come after pass 1
    tc::cluster_wait();
    if constexpr (SM) {
      // stage j takes weight stage j and A group j (the same three K blocks)
      if (lane == 0) {
        const int nst = (kbs + P::BG - 1) / P::BG;
        for (int j = 0; j < nst; ++j) {
          const int s = j % P::NSB;
          if (!mbar_wait_abortable(smem_addr(&a_group[j]), 0u, abortp, a.wait_limit) ||
              !mbar_wait_abortable(smem_addr(&full_b[s]), (uint32_t)(j / P::NSB) & 1u, abortp,
                                   a.wait_limit))
            break;
          tc::fence_after();
          const int first = j * P::BG, nb = min(P::BG, kbs - first);
          for (int i = 0; i < nb; ++i) {
            const int blk = first + i;  // this CTA's K block: x (now A) stage blk
            const uint32_t slot = (uint32_t)(s * P::BG + i);
            const uint32_t sfa_col = tmem + kSfCol + 8u * slot, sfb_col = sfa_col + 4u;
            tc::copy_sf(sfa_col, tc::smem_desc(base + P::kOffSfA + (uint32_t)blk * kAtom, 0, 128,
                                               tc::kLayoutNone));
            tc::copy_sf(sfb_col, tc::smem_desc(base + P::kOffSfB + slot * kAtom, 0, 128,
                                               tc::kLayoutNone));
#pragma unroll
            for (int kk = 0; kk < kTK / 32; ++kk) {
              const uint64_t ad = tc::smem_desc(base + P::kOffX + (uint32_t)blk * xstage + 32u * kk,
                                                16, 1024, tc::kLayoutSw128);
              const uint64_t bd = tc::smem_desc(base + P::kOffB + slot * kTile + 32u * kk, 16, 1024,
                                                tc::kLayoutSw128);
              // D^T: 128 weight rows x 16 block rows
              tc::mma_mxf8(tmem + kAccCol, bd, ad, tc::mxf8_idesc(kTN, 16, (uint32_t)kk), sfb_col,
                           sfa_col, (blk | kk) != 0);
            }
          }
          tc::commit(smem_addr(&empty_b[s]));  // the weight stage is free after its MMAs
        }
      }
      if (lane == 0) tc::commit(smem_addr(&acc_bar));  // final (or, on abort, quiet)
    } else if (lane == 0) {
      for (int i = 0; i < kbs; ++i) {
        const int sa = i % kSA, sb = i % P::SB;
        if (!mbar_wait_abortable(smem_addr(&full_a[sa]), (uint32_t)(i / kSA) & 1u, abortp,
                                 a.wait_limit) ||
            !mbar_wait_abortable(smem_addr(&full_b[sb]), (uint32_t)(i / P::SB) & 1u, abortp,
                                 a.wait_limit))
          break;
        tc::fence_after();
        const uint32_t sfa_col = tmem + kSfCol + 8u * (uint32_t)(i & 3), sfb_col = sfa_col + 4u;
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
                       sfb_col, (i | kk) != 0);
        }
        tc::commit(smem_addr(&empty_a[sa]));  // both stages are free once these MMAs are done
        tc::commit(smem_addr(&empty_b[sb]));
      }
      tc::commit(smem_addr(&acc_bar));  // the accumulator is final (or, on abort, quiet)
    }
    __syncwarp();
  } else {
    // ---- quantizing warps 0-3
    const int t = threadIdx.x;
    const int j = t & 7;  // 16-column chunk of a K block
    // the 16 columns of chunk j of tile row m in an x stage (line L of the
    // quarter's box holds columns 64 h .. 64 h + 63; piece p sits at p ^ (L % 8))
    auto load_chunk = [&](uint32_t x_st, int m, uint32_t(&v)[8]) {
      const uint32_t L = (uint32_t)(m & 31) * 2u + (uint32_t)(j >> 2);
      const uint32_t sub = x_st + (uint32_t)(m >> 5) * (uint32_t)xr * 256u + L * 128u;
      const uint32_t p0 = (uint32_t)(2 * j) & 7u;
      const uint4 x0 = ld_smem(sub + ((p0 ^ (L & 7u)) << 4));
      const uint4 x1 = ld_smem(sub + (((p0 + 1u) ^ (L & 7u)) << 4));
      v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w;
      v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
    };

    // ---- pass 1: this thread's share of the rows' sums of squares over this
    // CTA's K blocks: rows (t / 8) + 16 u, chunk j, every K block in order
    constexpr int U = 2 * QB;
    const int Mp = Mr <= 1 ? 1 : Mr <= 2 ? 2 : Mr <= 4 ? 4 : Mr <= 8 ? 8 : 16;  // SM
    float2 acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = make_float2(0.f, 0.f);
    bool lost = false;
    auto add_squares = [&](int it) {
      const uint32_t x_st = base + P::kOffX + (uint32_t)(it % XS) * xstage;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int m = (t >> 3) + 16 * u;
        if (m >= Mr) continue;  // its box was not loaded
        uint32_t v[8];
        load_chunk(x_st, m, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) sq_acc(acc[u], v[k]);
      }
    };
    if (resident) {
      // every stage was issued at once: wait for all of them, then add with
      // the loads of several K blocks in flight (nothing is released)
      bool ok = true;
      for (int it = 0; it < kbs && ok; ++it)
        ok = mbar_wait_abortable(smem_addr(&x_full[xf(it)]), xp(it), abortp, a.wait_limit);
      if (!__all_sync(0xffffffffu, ok)) {
        *abortp = 1u;
        lost = true;
      } else if constexpr (SM) {
        // Mr <= 16: row m's K blocks are spread over the 16 / Mp groups of 8
        // lanes g = m + Mp sub (Mp = Mr rounded up to a power of two), group
        // sub taking blocks sub, sub + 16 / Mp, ...: all 128 threads add
        const int g = t >> 3, m = g % Mp, R = 16 / Mp;
        if (m < Mr) {
#pragma unroll 4
          for (int it = g / Mp; it < kbs; it += R) {
            uint32_t v[8];
            load_chunk(base + P::kOffX + (uint32_t)it * xstage, m, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) sq_acc(acc[0], v[k]);
          }
        }
      } else {
#pragma unroll 4
        for (int it = 0; it < kbs; ++it) add_squares(it);
      }
    } else {
      for (int it = 0; it < kbs; ++it) {
        if (!__all_sync(0xffffffffu, mbar_wait_abortable(smem_addr(&x_full[xf(it)]), xp(it),
                                                         abortp, a.wait_limit))) {
          *abortp = 1u;
          lost = true;
          break;
        }
        add_squares(it);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&x_empty[it % XS]));  // this warp has read it
      }
    }
    // one decision for the four warps
    const bool failed = tc::bar_or(kBarProducers, kProducers, lost || *abortp != 0u);
    tc::cluster_wait();  // set-up: every CTA has started before the partials go out
    // row partials: the 8 lanes of a row add their chunks (a symmetric
    // butterfly: all 8 get the same bits), then lane j of the row writes it
    // into part[rank][row] of CTA j (and j + 8) of the cluster
    if (!failed && SM) {
      // a group's 8 lanes add their chunks, then the groups of a row add in
      // the order of their K blocks' residue (sub = 0, 1, ...), and thread m
      // writes row m's partial into part[rank][m] of every CTA of the cluster
      float v = __fadd_rn(acc[0].x, acc[0].y);
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
      if (j == 0) gsum[t >> 3] = v;
      asm volatile("bar.sync %0, %1;" ::"n"(kBarProducers), "n"(kProducers) : "memory");
      if (t < Mr) {
        float tot = gsum[t];
        for (int sub = 1; sub < 16 / Mp; ++sub) tot = __fadd_rn(tot, gsum[sub * Mp + t]);
        for (int c = 0; c < S; ++c) tc::st_cluster_f32(tc::mapa(smem_addr(&part[rank][t]), (uint32_t)c), tot);
      }
    } else if (!failed) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float v = __fadd_rn(acc[u].x, acc[u].y);
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        const int m = (t >> 3) + 16 * u;
        if (m < Mr)
          for (int c = j; c < S; c += 8)
            tc::st_cluster_f32(tc::mapa(smem_addr(&part[rank][m]), (uint32_t)c), v);
      }
    }
    tc::cluster_arrive();  // all partial sums are in every CTA (release / acquire)
    tc::cluster_wait();

    if (!failed) {
      if (t < Mr) {
        float ss = part[0][t];
        for (int c = 1; c < S; ++c) ss = __fadd_rn(ss, part[c][t]);
        // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))); the mean is RN(ss / K)
        float mean = div_rn(ss, (float)a.K, a.rcp_K);
        if (mean < 0x1p-100f) mean = __fdiv_rn(ss, (float)a.K);
        inv_s[t] = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
      }
      asm volatile("bar.sync %0, %1;" ::"n"(kBarProducers), "n"(kProducers) : "memory");

      // ---- pass 2: warp w < kSA makes the A tiles of this CTA's K blocks
      // w, w + kSA, ... (x_full slot it % 4 then always belongs to one warp)
      const bool store_q = a.q != nullptr && blockIdx.x == 0;  // one tile column writes q
      // normalise, quantize and store chunk j of tile row m of K block kb
      auto finish_item = [&](uint32_t(&v)[8], const uint32_t(&wv)[8], uint32_t a_st,
                             uint32_t sf_st, int kb, int m) {
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
      };
      for (int i = warp; i < kbs; i += kSA) {
        const int it = kbs + i, kb = kb0 + i;
        const int sa = i % kSA, xs = resident ? i : it % XS;
        bool ok = resident || mbar_wait_abortable(smem_addr(&x_full[xf(it)]), xp(it), abortp,
                                                  a.wait_limit);
        if (!SM && ok && i >= kSA)
          ok = mbar_wait_abortable(smem_addr(&empty_a[sa]), (uint32_t)(i / kSA - 1) & 1u, abortp,
                                   a.wait_limit);
        if (!__all_sync(0xffffffffu, ok)) {  // the warp acts as one
          *abortp = 1u;
          break;
        }
        const uint32_t w_st = base + P::kOffW + 256u * (uint32_t)xs + 32u * (uint32_t)j;
        const uint4 w0 = ld_smem(w_st), w1 = ld_smem(w_st + 16u);
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint32_t x_st = base + P::kOffX + (uint32_t)xs * xstage;
        // SM: the A tile goes over its own x stage (row m writes 128 bytes at
        // 128 m, over x lines that rows before m / 2 + 1 held: those rows have
        // been read, by this warp, in this or an earlier step of the loop below)
        const uint32_t a_st = SM ? x_st : base + P::kOffA + (uint32_t)sa * kTile;
        const uint32_t sf_st = base + P::kOffSfA + (uint32_t)(SM ? i : sa) * kAtom;
#pragma unroll 2
        for (int r = 0; r < 8 * QB; ++r) {
          const int m = (lane >> 3) + 4 * r;  // tile row
          if (!__any_sync(0xffffffffu, m < Mr)) break;
          uint32_t v[8];
          load_chunk(x_st, m, v);
          finish_item(v, wv, a_st, sf_st, kb, m);
        }
        tc::fence_async_smem();  // the A stage writes come before the MMAs
        __syncwarp();
        if (SM && lane == 0) mbar_arrive(smem_addr(&a_group[i / 3]));
        if (!SM && lane == 0) {
          if (!resident)  // counts for all four warps
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(
                             smem_addr(&x_empty[xs])),
                         "r"(kProducerWarps)
                         : "memory");
          mbar_arrive(smem_addr(&full_a[sa]));
        }
      }
      // the scale rows of the padding past M in the last block (this CTA's K
      // blocks), zero in q_scale
      if (store_q && Mr < kTM)
        for (int m = Mr + t; m < kTM; m += kProducers)
          for (int g = 4 * kb0; g < 4 * (kb0 + kbs); ++g) a.qs[swizzled_offset(m0 + m, g, KB)] = 0;
    }
  }

  // ------------------------------------------------ reduction and epilogue
  // Warps 0-3 hold accumulator lanes 32 w .. 32 w + 31 (tile rows). The
  // acc_bar wait is not cut short by an abort: the MMAs must be complete
  // before tensor memory is read or freed.
  bool acc_ok = false;
  if (warp < kProducerWarps) {
    acc_ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&acc_bar), 0u, kWaitLimitCycles) &&
                                         *abortp == 0u);
    tc::fence_after();
  }
  if constexpr (SM) {
    // D^T in tensor memory: warp w (< 4) holds weight rows n0 + 32 w + lane,
    // one column a block row. Reduce-scatter over the cluster: every CTA
    // stores its partial tile into its own (idle) x region, weight row n at
    // 80 n bytes with its Mr columns contiguous; after a cluster barrier CTA q
    // adds, for its share of the block rows, the S partials in rank order
    // (16-byte distributed shared memory loads) and stores D; a second barrier
    // keeps every CTA's memory until the others are done reading it.
    constexpr uint32_t kRowBytes = (16 + 4) * 4;
    static_assert(kTM * kRowBytes <= P::kXRegion, "the partial tile fits the x region");
    const int n = warp * 32 + lane;  // weight row of the tile = column of D
    const uint32_t prow = base + P::kOffX + (uint32_t)n * kRowBytes;
    if (acc_ok) {
      uint32_t r[32];
      tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + kAccCol, r);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (4 * k < Mr) {
          const uint32_t v4[4] = {r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]};
          st_smem(prow + 16u * (uint32_t)k, v4);
        }
    }
    if (S > 1) tc::cluster_sync();  // every partial is in its CTA's memory
    if (acc_ok) {
      const int share = ((Mr + S - 1) / S + 3) & ~3, m_lo = rank * share;
      const int m_hi = m_lo + share < Mr ? m_lo + share : Mr;
      for (int m4 = m_lo; m4 < m_hi; m4 += 4) {
        const uint32_t off = prow + (uint32_t)m4 * 4u;
        // every CTA's 16 bytes are requested before the first is added
        uint4 o[kMaxSplits];
#pragma unroll
        for (int p = 0; p < kMaxSplits; ++p)
          if (p < S) o[p] = ld_cluster_v4(tc::mapa(off, (uint32_t)p));
        float v[4] = {__uint_as_float(o[0].x), __uint_as_float(o[0].y), __uint_as_float(o[0].z),
                      __uint_as_float(o[0].w)};
#pragma unroll
        for (int p = 1; p < kMaxSplits; ++p) {
          if (p < S) {  // the other CTAs' partials, in rank order
            v[0] = __fadd_rn(v[0], __uint_as_float(o[p].x));
            v[1] = __fadd_rn(v[1], __uint_as_float(o[p].y));
            v[2] = __fadd_rn(v[2], __uint_as_float(o[p].z));
            v[3] = __fadd_rn(v[3], __uint_as_float(o[p].w));
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (m4 + e < m_hi)
            a.d[(m0 + m4 + e) * a.ldd + n0 + n] =
                (uint16_t)(f2_to_bf2(make_float2(v[e], 0.f)) & 0xffffu);
      }
    }
    if (S > 1) tc::cluster_sync();  // the others are done reading this CTA's partial
  } else {
    const int row = warp * 32 + lane;  // tile row of this thread (warps 0-3)
    const bool row_live = warp < kProducerWarps && row < Mr;
    const uint32_t tm_row = tmem + ((uint32_t)(warp * 32) << 16) + kAccCol;
    // Push: the others store their rows with data straight into the leader's
    // shared memory (remote stores, no round trip) once every CTA's MMAs are
    // done; pull, when they do not fit: each keeps its rows and the leader
    // reads them. Both use two cluster barriers.
    const bool push = (uint32_t)(S - 1) * (uint32_t)Mr * 512u <= P::kPushArea;
    // slot of rank p's partial rows in the leader: column groups outermost
    auto push_off = [&](int p, int rw, int c4) {
      return (uint32_t)(p - 1) * (uint32_t)Mr * 512u + ((uint32_t)c4 * (uint32_t)Mr + (uint32_t)rw) * 16u;
    };
    if (S > 1) {
      if (push) tc::cluster_sync();  // every CTA's MMAs are done: the leader's memory is free
      if (rank > 0 && acc_ok && __any_sync(0xffffffffu, row_live)) {
        for (int c = 0; c < kTN; c += 32) {
          uint32_t r[32];
          tc::tmem_ld32(tm_row + (uint32_t)c, r);
          if (row_live) {
  #pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t v4[4] = {r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]};
              if (push) {
                const uint32_t dst = tc::mapa(base + push_off(rank, row, c / 4 + k), 0u);
                asm volatile("st.shared::cluster.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst),
                             "r"(v4[0]), "r"(v4[1]), "r"(v4[2]), "r"(v4[3])
                             : "memory");
              } else {
                st_smem(base + P::kOffA + part_off(row, c / 4 + k, Mr), v4);
              }
            }
          }
        }
      }
      tc::cluster_sync();  // every partial tile is in place
    }
    if ((S == 1 || rank == 0) && acc_ok && __any_sync(0xffffffffu, row_live)) {
      for (int c = 0; c < kTN; c += 32) {
        uint32_t r[32];
        tc::tmem_ld32(tm_row + (uint32_t)c, r);
        if (row_live) {
          for (int p = 1; p < S; ++p) {  // the other CTAs' partials, in rank order
  #pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint4 o =
                  push ? ld_smem(base + push_off(p, row, c / 4 + k))
                       : ld_cluster_v4(tc::mapa(base + P::kOffA + part_off(row, c / 4 + k, Mr),
                                                (uint32_t)p));
              const uint32_t ov[4] = {o.x, o.y, o.z, o.w};
  #pragma unroll
              for (int e = 0; e < 4; ++e)
                r[4 * k + e] =
                    __float_as_uint(__fadd_rn(__uint_as_float(r[4 * k + e]), __uint_as_float(ov[e])));
            }
          }
          uint32_t o16[16];
  #pragma unroll
          for (int k = 0; k < 16; ++k)
            o16[k] = f2_to_bf2(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])));
          uint8_t* dp = reinterpret_cast<uint8_t*>(a.d + (m0 + row) * a.ldd + n0 + c);
  #pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t vv[4] = {o16[4 * k], o16[4 * k + 1], o16[4 * k + 2], o16[4 * k + 3]};
            st_stream(dp + 16 * k, vv);
          }
        }
      }
    }
    if (S > 1 && !push) tc::cluster_sync();  // the leader has read every partial tile
  }
  tc::fence_before();
  __syncthreads();
  if (*abortp != 0u && threadIdx.x == 0) {
    atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
    // this CTA's own loads land before its shared memory goes away
    for (int s = 0; s < P::SB; ++s)
      if (issued_b[s] > 0)
        mbar_wait_bounded(smem_addr(&full_b[s]), (issued_b[s] - 1u) & 1u, kDrainLimitCycles);
    for (int s = 0; s < kMaxXS; ++s)
      if (issued_x[s] > 0)
        mbar_wait_bounded(smem_addr(&x_full[s]), (issued_x[s] - 1u) & 1u, kDrainLimitCycles);
  }
  __syncthreads();
  if (warp == kWarpMma) tc::tmem_dealloc(tmem, kTmemCols);
}

// x [M, K] bf16 as a 3-D tensor {64 columns, K / 64 column blocks, M rows}
// with boxes of 64 columns x 2 blocks x `rows` rows, each 128-byte line
// swizzled; zero fill past the last row.
bool encode_x(CUtensorMap* map, const void* x, int64_t M, int64_t K, int64_t ldx, int rows) {
  auto fn = tc::encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {64, (cuuint64_t)(K / 64), (cuuint64_t)M};
  const cuuint64_t strides[2] = {128, (cuuint64_t)ldx * 2};
  const cuuint32_t box[3] = {64, 2, (cuuint32_t)rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int QB, bool SM = false>
cudaError_t launch_one(const CUtensorMap& map_x, const CUtensorMap& map_b, const ProArgs& a,
                       int64_t N, int64_t M, cudaStream_t stream) {
  using P = Plan<QB, SM>;
  auto kernel = gemm_rmsnorm_mxfp8_kernel<QB, SM>;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)P::kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / kTN), (unsigned)((M + kTM - 1) / kTM), (unsigned)a.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)a.splits;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, map_x, map_b, a);
}

}  // namespace

// K split: the most CTAs a tile (up to 8 and up to its K blocks) that still
// fit the grid on the SMs in one wave, one CTA an SM.
int gemm_rmsnorm_splits(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = (N / kTN) * ((M + kTM - 1) / kTM);
  int64_t s = device_sm_count() / (tiles > 0 ? tiles : 1);
  if (s > kMaxSplits) s = kMaxSplits;
  if (s > K / kTK) s = K / kTK;
  return s < 1 ? 1 : (int)s;
}

int gemm_rmsnorm_mxfp8(const void* x, int64_t ldx, const void* weight, float eps, const void* b,
                       int64_t ldb, const void* b_scale, void* d, int64_t ldd, int64_t M,
                       int64_t N, int64_t K, void* q, int64_t ldq, void* q_scale,
                       long long wait_limit, cudaStream_t stream, const char** why) {
  CUtensorMap map_b, map_x;
  if (!tc::encode_e4m3_operand(&map_b, b, N, K, ldb)) {
    *why = "cuTensorMapEncodeTiled failed for b";
    return CUTIE_ERR_CUDA;
  }
  const int xr = M >= 32 ? 32 : (int)((M + 7) / 8 * 8);
  if (!encode_x(&map_x, x, M, K, ldx, xr)) {
    *why = "cuTensorMapEncodeTiled failed for x";
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
  a.splits = gemm_rmsnorm_splits(M, N, K);
  a.xr = xr;
  a.eps = eps;
  a.rcp_K = 1.0f / (float)K;
  a.wait_limit = wait_limit;
  // the small plan: at most 16 rows, and every K block of a CTA resident in
  // an x stage of its own
  const int64_t kbs_max = (K / kTK + a.splits - 1) / a.splits;
  const int64_t xs_small = Plan<1, true>::kXRegion / ((uint32_t)xr * 256u);
  const bool small = M <= 16 && kbs_max <= (xs_small < kMaxXS ? xs_small : kMaxXS);
  cudaError_t e;
  switch (small ? 0 : M >= kTM ? 4 : (int)((M + 31) / 32)) {
    case 0: e = launch_one<1, true>(map_x, map_b, a, N, M, stream); break;
    case 1: e = launch_one<1>(map_x, map_b, a, N, M, stream); break;
    case 2: e = launch_one<2>(map_x, map_b, a, N, M, stream); break;
    case 3: e = launch_one<3>(map_x, map_b, a, N, M, stream); break;
    default: e = launch_one<4>(map_x, map_b, a, N, M, stream); break;
  }
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return CUTIE_ERR_CUDA;
  }
  return CUTIE_OK;
}

}  // namespace cutie
