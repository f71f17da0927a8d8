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
// One CTA computes one 128 x 128 tile of D with 4 warps:
//  * warp 0, one thread: the producer. Per 128-wide K block it loads the A and
//    B tiles (16 KB each) with TMA into a 4-stage shared-memory ring, 128-byte
//    swizzled rows (the canonical K-major operand layout of tcgen05.mma), and
//    the two 512-byte scale atoms of the block with plain bulk copies: in the
//    swizzled layout the scales of 128 rows x 4 groups are one contiguous
//    atom, already in the order tcgen05.cp.32x128b.warpx4 takes (row i of the
//    copy holds rows i, i+32, i+64, i+96), so nothing is rearranged.
//  * warp 1, one thread: the MMA issuer. Per stage it copies both scale atoms
//    into tensor memory (4 columns each, a column pair per stage, so a copy
//    never overwrites scales an earlier MMA still reads) and issues four
//    tcgen05.mma.kind::mxf8f6f4.block_scale of K = 32 (scale id k selects
//    byte k of each 32-bit scale cell); tcgen05.commit releases the stage.
//  * all warps: the epilogue. Warp w reads accumulator lanes 32w..32w+31
//    (tcgen05.ld 32x32b, 32 columns at a time), rounds to bf16 and stores.
// Tensor memory: 256 columns (128 accumulator + 8 scale columns per stage),
// allocated by warp 2 and freed by it at the end. No cluster, no multicast.
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

constexpr int kBM = 128, kBN = 128, kBK = 128;  // tile; K in e4m3 elements (= bytes)
constexpr int kStages = 4;
constexpr uint32_t kTileBytes = kBM * kBK;         // 16 KB (A) = kBN * kBK (B)
constexpr uint32_t kSfBytes = 512;                 // one 128 x 4 scale atom
constexpr uint32_t kStageBytes = 2 * kTileBytes + 2 * kSfBytes;  // 33 KB, a multiple of 1 KB
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kAccCol = 0, kSfCol = 128;  // scales of stage s: kSfCol + 8 s (A), + 4 (B)
constexpr int kThreads = 128;
constexpr size_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment to 1 KB

using tc::kLayoutNone;
using tc::kLayoutSw128;
using tc::mma_mxf8;
using tc::smem_desc;
using tc::tma_load_2d;
__device__ __forceinline__ void fence_tc_before() { tc::fence_before(); }
__device__ __forceinline__ void fence_tc_after() { tc::fence_after(); }
__device__ __forceinline__ uint32_t instr_desc(uint32_t sf_id) {
  return tc::mxf8_idesc(kBM, kBN, sf_id);
}
__device__ __forceinline__ void tc_copy_sf(uint32_t col, uint64_t desc) { tc::copy_sf(col, desc); }
__device__ __forceinline__ void tc_commit(uint32_t bar) { tc::commit(bar); }

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

__global__ void __launch_bounds__(kThreads, 1)
    gemm_mxfp8_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, const uint8_t* sfa,
                      const uint8_t* sfb, uint16_t* d, int64_t ldd, int M, int K) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t tmem_base_slot;
  __shared__ uint32_t abort_flag;
  __shared__ uint32_t issued[kStages];  // copies issued into each stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;  // 1 KB aligned stages
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int KB = K / kBK;
  const int sf_tiles_k = K / kBK;  // scale atoms along K (4 groups of 32 each)
  volatile uint32_t* abortp = &abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), 1);
      issued[s] = 0;
    }
    mbar_init(smem_addr(&acc_bar), 1);
    abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&tmem_base_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_tc_before();
  __syncthreads();
  fence_tc_after();
  const uint32_t tmem = tmem_base_slot;
  griddep_wait();  // operands written by the previous kernel are complete
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---- producer
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kStages;
      const uint32_t use = (uint32_t)(kb / kStages);
      if (use > 0 && !wait_or_abort(smem_addr(&empty_bar[s]), (use - 1u) & 1u, abortp)) break;
      const uint32_t st = base + (uint32_t)s * kStageBytes;
      const uint32_t bar = smem_addr(&full_bar[s]);
      issued[s] = use + 1u;
      mbar_arrive_expect_tx(bar, kStageBytes);
      tma_load_2d(st, &map_a, kb * kBK, m0, bar);
      tma_load_2d(st + kTileBytes, &map_b, kb * kBK, n0, bar);
      bulk_g2s(st + 2 * kTileBytes, sfa + ((int64_t)blockIdx.y * sf_tiles_k + kb) * kSfBytes,
               kSfBytes, bar);
      bulk_g2s(st + 2 * kTileBytes + kSfBytes,
               sfb + ((int64_t)blockIdx.x * sf_tiles_k + kb) * kSfBytes, kSfBytes, bar);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kStages;
      const uint32_t use = (uint32_t)(kb / kStages);
      if (!wait_or_abort(smem_addr(&full_bar[s]), use & 1u, abortp)) break;
      fence_tc_after();
      const uint32_t st = base + (uint32_t)s * kStageBytes;
      const uint32_t sfa_col = tmem + kSfCol + 8u * (uint32_t)s, sfb_col = sfa_col + 4u;
      // scale atoms: 32 rows of 16 bytes, rows 16 bytes apart (8-row groups 128 bytes apart)
      tc_copy_sf(sfa_col, smem_desc(st + 2 * kTileBytes, 0, 128, kLayoutNone));
      tc_copy_sf(sfb_col, smem_desc(st + 2 * kTileBytes + kSfBytes, 0, 128, kLayoutNone));
#pragma unroll
      for (int kk = 0; kk < kBK / 32; ++kk) {
        // 32 bytes of K a step inside the 128-byte swizzled rows; 8-row groups 1 KB apart
        const uint64_t ad = smem_desc(st + 32u * kk, 16, 1024, kLayoutSw128);
        const uint64_t bd = smem_desc(st + kTileBytes + 32u * kk, 16, 1024, kLayoutSw128);
        mma_mxf8(tmem + kAccCol, ad, bd, instr_desc((uint32_t)kk), sfa_col, sfb_col,
                 (kb | kk) != 0);
      }
      tc_commit(smem_addr(&empty_bar[s]));  // the stage is free once these MMAs are done
    }
    tc_commit(smem_addr(&acc_bar));  // the accumulator is final (or, on abort, quiet)
  }
  __syncwarp();

  // ---- epilogue: every warp, its 32 accumulator lanes. The wait is not cut
  // short by an abort: the MMA thread always commits, and its MMAs must have
  // finished before tensor memory is read or freed.
  const bool acc_ok = mbar_wait_bounded(smem_addr(&acc_bar), 0u, kWaitLimitCycles) && !*abortp;
  if (!acc_ok) *abortp = 1u;
  fence_tc_after();
  const int row = m0 + warp * 32 + lane;
  if (acc_ok) {
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t r[32];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
          "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
            "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
            "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
            "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
            "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
            "=r"(r[31])
          : "r"(tmem + ((uint32_t)(warp * 32) << 16) + kAccCol + (uint32_t)c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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
  fence_tc_before();
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
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
}

bool encode_operand(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int64_t ld) {
  return tc::encode_e4m3_operand(map, ptr, rows, K, ld);
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
  CUtensorMap map_a, map_b;
  if (!encode_operand(&map_a, a, M, K, lda) || !encode_operand(&map_b, b, N, K, ldb)) {
    *why = "cuTensorMapEncodeTiled failed for an operand";
    return CUTIE_ERR_CUDA;
  }
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_mxfp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemBytes);
  });
  if (attr_err != cudaSuccess) {
    *why = cudaGetErrorString(attr_err);
    return CUTIE_ERR_CUDA;
  }
  // one CTA a 128 x 128 tile of D, with programmatic stream serialization
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / kBN), (unsigned)((M + kBM - 1) / kBM));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, gemm_mxfp8_kernel, map_a, map_b, static_cast<const uint8_t*>(a_scale),
      static_cast<const uint8_t*>(b_scale), static_cast<uint16_t*>(d), ldd, (int)M, (int)K);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return CUTIE_ERR_CUDA;
  }
  return CUTIE_OK;
}

}  // namespace cutie
