// MXFP8 block-scaled GEMM on the 5th-generation tensor cores (sm_100a):
// the downstream consumer of this library's FP8 codes and their swizzled
// e8m0 scales.
//
//   D[M, N] (bf16) = sum_k (A[m, k] * 2^(sA[m, k/32] - 127)) * (B[n, k] * 2^(sB[n, k/32] - 127))
//
// A: e4m3 [M, K], K contiguous (the q of cutie_rms_norm_fp8 with 1x32 groups);
// sA: its e8m0 scales in the Blackwell block-scaled layout
// (CUTIE_LAYOUT_MX_SWIZZLED: 128x4 atoms of 512 bytes); B: e4m3 [N, K] (the
// weight, K contiguous) with scales sB in the same layout; fp32 accumulation
// in tensor memory, bf16 out.
//
// One CTA computes one 128 x BN tile of D with 4 warps (BN = 256 when N is a
// multiple of 256 and the grid still has a tile for every SM, else 128; a
// 256-wide tile reads each A tile once for twice the columns, which halves
// the shared-memory bytes an MMA reads per flop):
//  * warp 0, one thread: the producer. Per 128-wide K block it loads the A
//    tile (16 KB) and the B tile (BN rows, one 128-row TMA box each) into a
//    4-stage shared-memory ring, 128-byte swizzled rows (the canonical
//    K-major operand layout of tcgen05.mma), and the scale atoms of the block
//    (one for A, BN / 128 for B) with plain bulk copies: in the swizzled
//    layout the scales of 128 rows x 4 groups are one contiguous atom,
//    already in the order tcgen05.cp.32x128b.warpx4 takes (row i of the copy
//    holds rows i, i+32, i+64, i+96), so nothing is rearranged.
//  * warp 1, one thread: the MMA issuer. Per stage it copies the scale atoms
//    into tensor memory (4 columns each; every stage has its own columns, so
//    a copy never overwrites scales an earlier MMA still reads) and issues
//    four tcgen05.mma.kind::mxf8f6f4.block_scale of 128 x BN x 32 (scale id
//    k selects byte k of each 32-bit scale cell); tcgen05.commit releases the
//    stage.
//  * all warps: the epilogue. Warp w reads accumulator lanes 32w..32w+31
//    (tcgen05.ld 32x32b, 32 columns at a time), rounds to bf16 and stores.
// Tensor memory: the BN accumulator columns, then the scale columns of the 4
// stages (256 or 512 columns allocated by warp 2, freed by it at the end).
// No cluster, no multicast. Batches of at most 32 rows, and of at most 128
// when N leaves SMs idle, take the decode kernel below instead (swapped
// operands, K split over a cluster).
//
// Every wait is bounded (kWaitLimitCycles): a wait that gives up sets the
// CTA's abort flag and the device error word; the producer stops issuing and
// lets its copies in flight land, the MMA thread commits what it issued and
// the epilogue waits for that before tensor memory is freed.
#include "cutie.h"
#include "launch.cuh"
#include "tcgen05.cuh"

namespace cutie {

static __device__ int g_gemm_device_error = 0;

namespace {

constexpr int kBM = 128, kBK = 128;  // tile rows; K in e4m3 elements (= bytes)
constexpr int kStages = 4;
constexpr uint32_t kTileBytes = kBM * kBK;  // one 128-row operand box: 16 KB
constexpr uint32_t kSfBytes = 512;          // one 128 x 4 scale atom
constexpr int kThreads = 128;

template <int BN>
struct GemmPlan {
  static constexpr int kNB = BN / 128;  // 128-row boxes (and scale atoms) of B
  static constexpr uint32_t kOffB = kTileBytes;
  static constexpr uint32_t kOffSfA = kOffB + kNB * kTileBytes;
  static constexpr uint32_t kOffSfB = kOffSfA + kSfBytes;
  // a stage is a multiple of 1 KB, so every swizzled tile starts on one
  static constexpr uint32_t kStageBytes = (kOffSfB + kNB * kSfBytes + 1023u) & ~1023u;
  static constexpr size_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment to 1 KB
  static constexpr uint32_t kAccCol = 0;
  static constexpr uint32_t kSfCol = BN;                 // stage s: kSfCol + kSfStride s
  static constexpr uint32_t kSfStride = 4 * (1 + kNB);   // A atom, then the B atoms
  static constexpr uint32_t kTmemCols = BN + kStages * kSfStride <= 256 ? 256 : 512;
  static_assert(BN + kStages * kSfStride <= kTmemCols, "tensor memory columns");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

using tc::kLayoutNone;
using tc::kLayoutSw128;
using tc::smem_desc;

// Waits that give up after `limit` cycles or at once when the abort flag is
// set; giving up sets the flag.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity,
                                              volatile uint32_t* abort_flag) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  while (!*abort_flag && clock64() - t0 <= kWaitLimitCycles)
    if (mbar_try_wait(bar, parity)) return true;
  *abort_flag = 1u;
  return false;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_mxfp8_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, const uint8_t* sfa,
                      const uint8_t* sfb, uint16_t* d, int64_t ldd, int M, int K) {
  using P = GemmPlan<BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t tmem_base_slot;
  __shared__ uint32_t abort_flag;
  __shared__ uint32_t issued[kStages];  // copies issued into each stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;  // 1 KB aligned stages
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
  const int KB = K / kBK;  // K blocks = scale atoms along K (4 groups of 32 each)
  volatile uint32_t* abortp = &abort_flag;

  if (threadIdx.x == 0) {
    tc::prefetch_map(&map_a);
    tc::prefetch_map(&map_b);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), 1);
      issued[s] = 0;
    }
    mbar_init(smem_addr(&acc_bar), 1);
    abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 2) tc::tmem_alloc(smem_addr(&tmem_base_slot), P::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base_slot;
  griddep_wait();  // operands written by the previous kernel are complete
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---- producer
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kStages;
      const uint32_t use = (uint32_t)(kb / kStages);
      if (use > 0 && !wait_or_abort(smem_addr(&empty_bar[s]), (use - 1u) & 1u, abortp)) break;
      const uint32_t st = base + (uint32_t)s * P::kStageBytes;
      const uint32_t bar = smem_addr(&full_bar[s]);
      issued[s] = use + 1u;
      mbar_arrive_expect_tx(bar, (1 + P::kNB) * (kTileBytes + kSfBytes));
      tc::tma_load_2d(st, &map_a, kb * kBK, m0, bar);
      bulk_g2s(st + P::kOffSfA, sfa + ((int64_t)blockIdx.y * KB + kb) * kSfBytes, kSfBytes, bar);
#pragma unroll
      for (int h = 0; h < P::kNB; ++h) {
        tc::tma_load_2d(st + P::kOffB + (uint32_t)h * kTileBytes, &map_b, kb * kBK, n0 + 128 * h,
                        bar);
        bulk_g2s(st + P::kOffSfB + (uint32_t)h * kSfBytes,
                 sfb + ((int64_t)(blockIdx.x * P::kNB + h) * KB + kb) * kSfBytes, kSfBytes, bar);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kStages;
      const uint32_t use = (uint32_t)(kb / kStages);
      if (!wait_or_abort(smem_addr(&full_bar[s]), use & 1u, abortp)) break;
      tc::fence_after();
      const uint32_t st = base + (uint32_t)s * P::kStageBytes;
      const uint32_t sfa_col = tmem + P::kSfCol + P::kSfStride * (uint32_t)s, sfb_col = sfa_col + 4u;
      // scale atoms: 32 rows of 16 bytes, rows 16 bytes apart (8-row groups 128 bytes apart)
      tc::copy_sf(sfa_col, smem_desc(st + P::kOffSfA, 0, 128, kLayoutNone));
#pragma unroll
      for (int h = 0; h < P::kNB; ++h)
        tc::copy_sf(sfb_col + 4u * (uint32_t)h,
                    smem_desc(st + P::kOffSfB + (uint32_t)h * kSfBytes, 0, 128, kLayoutNone));
#pragma unroll
      for (int kk = 0; kk < kBK / 32; ++kk) {
        // 32 bytes of K a step inside the 128-byte swizzled rows; 8-row groups 1 KB apart
        const uint64_t ad = smem_desc(st + 32u * kk, 16, 1024, kLayoutSw128);
        const uint64_t bd = smem_desc(st + P::kOffB + 32u * kk, 16, 1024, kLayoutSw128);
        tc::mma_mxf8(tmem + P::kAccCol, ad, bd, tc::mxf8_idesc(kBM, BN, (uint32_t)kk), sfa_col,
                     sfb_col, (kb | kk) != 0);
      }
      tc::commit(smem_addr(&empty_bar[s]));  // the stage is free once these MMAs are done
    }
    tc::commit(smem_addr(&acc_bar));  // the accumulator is final (or, on abort, quiet)
  }
  __syncwarp();

  // ---- epilogue: every warp, its 32 accumulator lanes. The wait is not cut
  // short by an abort: the MMA thread always commits, and its MMAs must have
  // finished before tensor memory is read or freed.
  const bool acc_ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&acc_bar), 0u,
                                                                kWaitLimitCycles) &&
                                                  *abortp == 0u);
  if (!acc_ok) *abortp = 1u;
  tc::fence_after();
  const int row = m0 + warp * 32 + lane;
  if (acc_ok && __any_sync(0xffffffffu, row < M)) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + P::kAccCol + (uint32_t)c, r);
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        o[j] = f2_to_bf2(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])));
      if (row < M) {
        uint8_t* p = reinterpret_cast<uint8_t*>(d + (int64_t)row * ldd + n0 + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t v[4] = {o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]};
          st_stream(p + 16 * j, v);
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (*abortp) {
    if (threadIdx.x == 0) {
      atomicCAS(&g_gemm_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
      // let the copies in flight land before the shared memory goes away
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0)
          mbar_wait_bounded(smem_addr(&full_bar[s]), (issued[s] - 1u) & 1u, kDrainLimitCycles);
    }
    __syncthreads();
  }
  if (warp == 2) tc::tmem_dealloc(tmem, P::kTmemCols);
}

// ---------------------------------------------------------------- decode
//
// Batches of at most 128 rows: the weight is the 128-row M side of the MMA
// and the batch the BR-wide N side (D^T = B A^T; BR = 32, 64 or 128, the
// smallest that holds the batch), so a CTA streams 16 KB of weight a K block
// with a batch box of BR rows (rows past M zero-filled): up to 32 rows, 4 KB
// instead of a 16 KB A box that is nearly all zero.
//
// The grid has only N / 128 tiles, so K is split over a cluster of S CTAs
// (grid z) to put more SMs on the weight stream. Every rank accumulates its
// K range in its own tensor memory and keeps its partial tile in its own
// shared memory; each rank then adds, for its share of the batch rows, the
// partials of all ranks in rank order over distributed shared memory (no
// multicast), so the result does not depend on timing.
//
// Two or three K blocks share one ring stage and one pair of barriers: at
// decode sizes the per-stage hand-off, not the bytes, set the time of
// one-block stages.
constexpr int kDecodeRows = 32;     // batch rows of the narrow plan (the MMA's N)
constexpr int kDecodeMidRows = 64;    // of the middle one
constexpr int kDecodeWideRows = 128;  // and of the wide one
constexpr int kDecodeMaxRanks = 8;    // a portable cluster

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int BR>
struct DecodePlan {
  static constexpr int kStages = 3;
  static constexpr int kBlocks = BR == kDecodeWideRows ? 2 : 3;  // K blocks a stage
  static constexpr uint32_t kOffA = kTileBytes;  // batch box: BR rows x 128 bytes
  static constexpr uint32_t kOffSfW = kOffA + BR * kBK;
  static constexpr uint32_t kOffSfA = kOffSfW + kSfBytes;
  static constexpr uint32_t kBlockBytes = (kOffSfA + kSfBytes + 1023u) & ~1023u;  // 21 or 33 KB
  static constexpr uint32_t kStageBytes = kBlocks * kBlockBytes;
  static constexpr size_t kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr uint32_t kTxBytes = kTileBytes + BR * kBK + 2 * kSfBytes;
  // tensor memory: BR accumulator columns, then 8 scale columns a block slot
  static constexpr uint32_t kSfCol = BR;
  static constexpr uint32_t kTmemCols = BR + 8 * kStages * kBlocks <= 128 ? 128 : 256;
  // a rank's partial tile (in its idle ring after the K loop): 128 weight
  // rows of BR fp32 batch columns, rows kRowStride floats apart
  static constexpr uint32_t kRowStride = BR + 4;
  static constexpr uint32_t kPartBytes = kBM * kRowStride * 4;
  static constexpr int kMaxSplit = kDecodeMaxRanks;
  static_assert(kSfCol + 8 * kStages * kBlocks <= kTmemCols, "tensor memory columns");
  static_assert(kPartBytes <= kStages * kStageBytes, "the partial tile fits the ring");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

template <int BR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_mxfp8_decode_kernel(const __grid_constant__ CUtensorMap map_a,
                             const __grid_constant__ CUtensorMap map_b, const uint8_t* sfa,
                             const uint8_t* sfb, uint16_t* d, int64_t ldd, int M, int K) {
  using P = DecodePlan<BR>;
  constexpr int kDecodeStages = P::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kDecodeStages];
  __shared__ __align__(8) uint64_t empty_bar[kDecodeStages];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t tmem_base_slot;
  __shared__ uint32_t abort_flag;
  __shared__ float peer_bad;  // the leader's: non-zero once a rank gave up
  __shared__ uint32_t issued[kDecodeStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
  const int n0 = blockIdx.x * kBM;  // 128 columns of D = 128 rows of the weight
  const int KB = K / kBK, S = (int)gridDim.z;
  const uint32_t rank = tc::cluster_ctarank();  // = blockIdx.z: the cluster spans z
  const int kb0 = (int)((int64_t)KB * rank / S), kb1 = (int)((int64_t)KB * (rank + 1) / S);
  const int NS = (kb1 - kb0 + P::kBlocks - 1) / P::kBlocks;  // ring stages used
  volatile uint32_t* abortp = &abort_flag;

  if (threadIdx.x == 0) {
    tc::prefetch_map(&map_a);
    tc::prefetch_map(&map_b);
    for (int s = 0; s < kDecodeStages; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), 1);
      issued[s] = 0;
    }
    mbar_init(smem_addr(&acc_bar), 1);
    abort_flag = 0;
    peer_bad = 0.f;
    mbar_init_fence();
  }
  if (warp == 2) tc::tmem_alloc(smem_addr(&tmem_base_slot), P::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = tmem_base_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    for (int j = 0; j < NS; ++j) {
      const int s = j % kDecodeStages;
      const uint32_t use = (uint32_t)(j / kDecodeStages);
      if (use > 0 && !wait_or_abort(smem_addr(&empty_bar[s]), (use - 1u) & 1u, abortp)) break;
      const uint32_t bar = smem_addr(&full_bar[s]);
      const int first = kb0 + j * P::kBlocks, nb = min(P::kBlocks, kb1 - first);
      issued[s] = use + 1u;
      mbar_arrive_expect_tx(bar, (uint32_t)nb * P::kTxBytes);
      for (int i = 0; i < nb; ++i) {
        const int kb = first + i;
        const uint32_t st = base + (uint32_t)s * P::kStageBytes + (uint32_t)i * P::kBlockBytes;
        tc::tma_load_2d(st, &map_b, kb * kBK, n0, bar);
        tc::tma_load_2d(st + P::kOffA, &map_a, kb * kBK, 0, bar);  // zero past row M
        bulk_g2s(st + P::kOffSfW, sfb + ((int64_t)blockIdx.x * KB + kb) * kSfBytes, kSfBytes,
                 bar);
        bulk_g2s(st + P::kOffSfA, sfa + (int64_t)kb * kSfBytes, kSfBytes, bar);
      }
    }
  } else if (warp == 1 && lane == 0) {
    for (int j = 0; j < NS; ++j) {
      const int s = j % kDecodeStages;
      const uint32_t use = (uint32_t)(j / kDecodeStages);
      if (!wait_or_abort(smem_addr(&full_bar[s]), use & 1u, abortp)) break;
      tc::fence_after();
      const int first = kb0 + j * P::kBlocks, nb = min(P::kBlocks, kb1 - first);
      for (int i = 0; i < nb; ++i) {
        const uint32_t st = base + (uint32_t)s * P::kStageBytes + (uint32_t)i * P::kBlockBytes;
        const uint32_t sfw_col = tmem + P::kSfCol + 8u * (uint32_t)(s * P::kBlocks + i);
        const uint32_t sfa_col = sfw_col + 4u;
        tc::copy_sf(sfw_col, smem_desc(st + P::kOffSfW, 0, 128, kLayoutNone));
        tc::copy_sf(sfa_col, smem_desc(st + P::kOffSfA, 0, 128, kLayoutNone));
#pragma unroll
        for (int kk = 0; kk < kBK / 32; ++kk) {
          const uint64_t wd = smem_desc(st + 32u * kk, 16, 1024, kLayoutSw128);
          const uint64_t ad = smem_desc(st + P::kOffA + 32u * kk, 16, 1024, kLayoutSw128);
          tc::mma_mxf8(tmem, wd, ad, tc::mxf8_idesc(kBM, BR, (uint32_t)kk), sfw_col,
                       sfa_col, (j | i | kk) != 0);
        }
      }
      tc::commit(smem_addr(&empty_bar[s]));
    }
    tc::commit(smem_addr(&acc_bar));
  }
  __syncwarp();

  // ---- this rank's partial tile: warp w holds D^T rows n0 + 32 w + lane, one
  // column a batch row
  const bool acc_ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&acc_bar), 0u,
                                                                kWaitLimitCycles) &&
                                                  *abortp == 0u);
  if (!acc_ok) *abortp = 1u;
  tc::fence_after();
  __syncthreads();
  const bool ok = *abortp == 0u;  // the same in every thread after the barrier
  if (!ok) {
    if (threadIdx.x == 0) {
      atomicCAS(&g_gemm_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
      // let the copies in flight land before other ranks write this ring
      for (int s = 0; s < kDecodeStages; ++s)
        if (issued[s] > 0)
          mbar_wait_bounded(smem_addr(&full_bar[s]), (issued[s] - 1u) & 1u, kDrainLimitCycles);
    }
    __syncthreads();
  }
  // Reduce-scatter over the cluster. Every rank stores its partial tile into
  // its own (idle) ring as [M batch rows][128 weight rows] fp32; after a
  // cluster barrier rank q adds, for the batch rows it owns (a contiguous
  // share of the M), the S partials in rank order, reading the others over
  // distributed shared memory, and stores D; a second barrier keeps every
  // rank's memory until the others are done reading it. A rank that gave up
  // marks every rank's peer_bad first, so that none stores.
  const int row = warp * 32 + lane;
  const uint32_t tm_row = tmem + ((uint32_t)(warp * 32) << 16);
  // weight row `row` keeps its batch columns contiguous, rows 16 bytes more
  // than BR floats apart (16-byte vector stores and loads, at most 4-way bank
  // conflicts)
  const uint32_t prow = base + (uint32_t)row * P::kRowStride * 4u;
  if (ok) {
    for (int c = 0; c < BR && c < M; c += 32) {
      uint32_t r[32];
      tc::tmem_ld32(tm_row + (uint32_t)c, r);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (c + 4 * k < M) {
          const uint32_t v4[4] = {r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]};
          st_smem(prow + (uint32_t)(c + 4 * k) * 4u, v4);
        }
    }
  } else if (threadIdx.x == 0) {
    for (int q = 0; q < S; ++q) tc::st_cluster_f32(tc::mapa(smem_addr(&peer_bad), (uint32_t)q), 1.f);
  }
  tc::cluster_sync();  // every partial is in its rank's memory
  if (peer_bad == 0.f) {
    // this rank's share of the batch rows, a multiple of 4
    const int share = ((M + S - 1) / S + 3) & ~3, m_lo = (int)rank * share;
    const int m_hi = m_lo + share < M ? m_lo + share : M;
    uint16_t* dp = d + n0 + row;
#pragma unroll 2
    for (int m4 = m_lo; m4 < m_hi; m4 += 4) {
      const uint32_t off = prow + (uint32_t)m4 * 4u;
      // every rank's 16 bytes are requested before the first is added
      float4 o[kDecodeMaxRanks];
#pragma unroll
      for (int q = 0; q < kDecodeMaxRanks; ++q)
        if (q < S) o[q] = ld_cluster_f4(tc::mapa(off, (uint32_t)q));
      float4 acc = o[0];
#pragma unroll
      for (int q = 1; q < kDecodeMaxRanks; ++q)
        if (q < S)  // rank order: the sum does not depend on timing
          acc.x += o[q].x, acc.y += o[q].y, acc.z += o[q].z, acc.w += o[q].w;
      const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (m4 + e < m_hi)
          dp[(int64_t)(m4 + e) * ldd] = (uint16_t)(f2_to_bf2(make_float2(v[e], 0.f)) & 0xffffu);
    }
  } else if (threadIdx.x == 0) {
    atomicCAS(&g_gemm_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
  }
  tc::cluster_sync();  // the others are done reading this rank's partial
  tc::fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, P::kTmemCols);
}

// Ranks a tile's K range is split over: enough CTAs for the SMs, at most
// max_split (the partial tiles fit the leader's ring; 8 at most, a portable
// cluster), at least one K block a rank.
int decode_splits(int64_t N, int64_t K, int max_split) {
  const int64_t tiles = N / kBM, kb = K / kBK;
  int64_t s = device_sm_count() / tiles;
  if (s > max_split) s = max_split;
  if (s > kb) s = kb;
  return s < 1 ? 1 : (int)s;
}

template <int BR>
cudaError_t launch_decode(const CUtensorMap& map_a, const CUtensorMap& map_b, const void* a_scale,
                          const void* b_scale, void* d, int64_t ldd, int64_t M, int64_t N,
                          int64_t K, cudaStream_t stream) {
  using P = DecodePlan<BR>;
  auto kernel = gemm_mxfp8_decode_kernel<BR>;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)P::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int S = decode_splits(N, K, P::kMaxSplit);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / kBM), 1, (unsigned)S);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = (unsigned)S;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, static_cast<const uint8_t*>(a_scale),
                            static_cast<const uint8_t*>(b_scale), static_cast<uint16_t*>(d), ldd,
                            (int)M, (int)K);
}

template <int BN>
cudaError_t launch_gemm(const CUtensorMap& map_a, const CUtensorMap& map_b, const void* a_scale,
                        const void* b_scale, void* d, int64_t ldd, int64_t M, int64_t N,
                        int64_t K, cudaStream_t stream) {
  using P = GemmPlan<BN>;
  auto kernel = gemm_mxfp8_kernel<BN>;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P::kSmemBytes);
  if (e != cudaSuccess) return e;
  // one CTA a 128 x BN tile of D, with programmatic stream serialization
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / BN), (unsigned)((M + kBM - 1) / kBM));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, static_cast<const uint8_t*>(a_scale),
                            static_cast<const uint8_t*>(b_scale), static_cast<uint16_t*>(d), ldd,
                            (int)M, (int)K);
}

}  // namespace

cudaError_t device_error_gemm(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_gemm_device_error, &zero, sizeof(int));
  }
  *out = v;
  return e;
}

int gemm_mxfp8(const void* a, int64_t lda, const void* a_scale, const void* b, int64_t ldb,
               const void* b_scale, void* d, int64_t ldd, int64_t M, int64_t N, int64_t K,
               cudaStream_t stream, const char** why) {
  // decode plans: up to 32 rows, and up to 128 rows when the 128-wide tiles
  // leave SMs for a K split of at least 2
  const int box_rows =
      M <= kDecodeRows ? kDecodeRows : M <= kDecodeMidRows ? kDecodeMidRows : kDecodeWideRows;
  const bool decode =
      M <= kDecodeRows ||
      (M <= kDecodeWideRows &&
       decode_splits(N, K, DecodePlan<kDecodeWideRows>::kMaxSplit) >= 2);
  CUtensorMap map_a, map_b;
  if (!tc::encode_e4m3_operand(&map_a, a, M, K, lda, decode ? box_rows : kBM) ||
      !tc::encode_e4m3_operand(&map_b, b, N, K, ldb)) {
    *why = "cuTensorMapEncodeTiled failed for an operand";
    return CUTIE_ERR_CUDA;
  }
  // decode batches: swapped operands, K split over a cluster. Otherwise
  // 256-wide tiles when N allows them and there are still enough of them to
  // give every SM one, else 128-wide tiles, twice as many CTAs
  const bool wide = N % 256 == 0 && (N / 256) * ((M + kBM - 1) / kBM) >= device_sm_count();
  const cudaError_t e =
      decode ? (M <= kDecodeRows
                    ? launch_decode<kDecodeRows>(map_a, map_b, a_scale, b_scale, d, ldd, M, N, K,
                                                 stream)
                : M <= kDecodeMidRows
                    ? launch_decode<kDecodeMidRows>(map_a, map_b, a_scale, b_scale, d, ldd, M, N,
                                                    K, stream)
                    : launch_decode<kDecodeWideRows>(map_a, map_b, a_scale, b_scale, d, ldd, M,
                                                     N, K, stream))
      : wide ? launch_gemm<256>(map_a, map_b, a_scale, b_scale, d, ldd, M, N, K, stream)
             : launch_gemm<128>(map_a, map_b, a_scale, b_scale, d, ldd, M, N, K, stream);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return CUTIE_ERR_CUDA;
  }
  return CUTIE_OK;
}

}  // namespace cutie
