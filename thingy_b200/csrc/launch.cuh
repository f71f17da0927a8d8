// Launch plumbing shared by the per-mode translation units. Each mode's
// kernels are instantiated in their own .cu file so nvcc builds them in
// parallel; capi.cu only sees the launch_fused_* entry points below.
#pragma once

#include "fused_kernel.cuh"
#include "pipe_kernel.cuh"
#include "rowstage_kernel.cuh"

namespace cutie {

// Defined in capi.cu; cached per device / per (kernel, block size, bytes).
int device_sm_count();
int cached_blocks_per_sm(const void* kernel, int threads, int dyn_smem);

// Ring plan: the most CTAs per SM (up to what registers allow) that still
// leave room for >= 2 stages each, and up to `max_stages` stages. Raises the
// kernel's dynamic shared-memory limit when needed. stages < 2: no plan.
struct BulkPlan {
  int stages;
  int blocks_per_sm;
  int smem_bytes;
};
BulkPlan plan_bulk(const void* kernel, int threads, int stage_bytes, int max_stages);

// Raise the kernel's dynamic shared-memory limit to `smem` (never lowers it)
// and return the resident CTAs per SM at that size (0 on failure).
int set_smem_and_occupancy(const void* kernel, int threads, int smem);

constexpr int kMaxStages = 4;

// Launch with programmatic stream serialization (see griddep_wait in
// fused_kernel.cuh): the kernel's prologue may overlap the previous kernel's
// tail; its global accesses still wait for that kernel to complete.
template <class... P, class... A>
cudaError_t launch_pdl(void (*kernel)(P...), unsigned grid, unsigned block, size_t smem,
                       cudaStream_t stream, A&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// Plan of the pipelined kernel: 2 or 3 stages a CTA, the most stages an SM
// (CTAs x stages), deeper rings first on a tie. stages < 2: no plan.
BulkPlan plan_pipe(const void* kernel, int threads, int stage_bytes);

// Persistent grid: as many CTAs as can be resident, never more than rows.
template <int NCH, int QM, int LPG, bool RES, bool NORM, bool FULL>
cudaError_t launch_fused_one(FusedArgs a, int threads, cudaStream_t stream) {
  auto kernel = fused_rmsnorm_fp8_kernel<NCH, QM, LPG, RES, NORM, FULL>;
  const int row_pad = (a.V * 16 + 63) / 64 * 64 + 64;  // whole chunks + one zero chunk
  const int stage_bytes = row_pad * (RES ? 2 : 1);
  const BulkPlan p =
      plan_bulk(reinterpret_cast<const void*>(kernel), threads, stage_bytes, kMaxStages);
  if (p.stages < 1) return cudaErrorInvalidConfiguration;
  a.stages = p.stages;
  int64_t grid = (int64_t)p.blocks_per_sm * device_sm_count();
  if (grid > a.M_pad) grid = a.M_pad;
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kernel, (unsigned)grid, (unsigned)threads, (size_t)p.smem_bytes, stream, a);
}

// Warp-per-row kernel: kRowwarpWarps warps per CTA, a private ring of
// `stages` 2 KB piece slots per warp; persistent grid over rows.
int rowwarp_stages();
template <int QM, int LPG, bool RES, bool NORM, bool FULL>
cudaError_t launch_rowwarp_one(FusedArgs a, cudaStream_t stream) {
  auto kernel = rowwarp_rmsnorm_fp8_kernel<QM, LPG, RES, NORM, FULL>;
  constexpr int kThreads = kRowwarpWarps * 32;
  const int P = rowwarp_stages();
  const int slot = (int)kPieceBytes * (RES ? 2 : 1);
  const int smem = kRowwarpWarps * P * (slot + 8);
  const int per_sm = set_smem_and_occupancy(reinterpret_cast<const void*>(kernel), kThreads, smem);
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  a.stages = P;
  int64_t grid = (int64_t)per_sm * device_sm_count();
  const int64_t need = (a.M_pad + kRowwarpWarps - 1) / kRowwarpWarps;
  if (grid > need) grid = need;
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kernel, (unsigned)grid, (unsigned)kThreads, (size_t)smem, stream, a);
}

// Pipelined kernel (pipe_kernel.cuh); *launched = false when two stages of
// the row do not fit a CTA (the caller then runs the single-pass kernel).
template <int QM, int LPG, bool RES, bool FULL, int SK, int MAXT>
cudaError_t launch_pipe_one(FusedArgs a, int threads, cudaStream_t stream, bool* launched) {
  auto kernel = pipe_rmsnorm_fp8_kernel<QM, LPG, RES, FULL, SK, MAXT>;
  const int row_pad = (int)pipe_row_pad(a.V, threads, PipeLayout<QM, LPG>::kInterleaved);
  const int stage_bytes = row_pad * (RES ? 2 : 1);
  const BulkPlan p = plan_pipe(reinterpret_cast<const void*>(kernel), threads, stage_bytes);
  *launched = false;
  if (p.stages < 2) return cudaSuccess;
  a.stages = p.stages;
  int64_t grid = (int64_t)p.blocks_per_sm * device_sm_count();
  if (grid > a.M_pad) grid = a.M_pad;
  if (grid > 0 && (a.M + grid - 1) / grid > INT32_MAX) return cudaSuccess;  // 32-bit row counter
  *launched = true;
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kernel, (unsigned)grid, (unsigned)threads, (size_t)p.smem_bytes, stream, a);
}

template <int QM, int LPG, bool RES, int SK>
cudaError_t launch_pipe_sk(const FusedArgs& a, int threads, cudaStream_t stream, bool* launched) {
  const bool full = (int64_t)threads * 4 == a.V;
  if (threads <= 224)
    return full ? launch_pipe_one<QM, LPG, RES, true, SK, 224>(a, threads, stream, launched)
                : launch_pipe_one<QM, LPG, RES, false, SK, 224>(a, threads, stream, launched);
  return full ? launch_pipe_one<QM, LPG, RES, true, SK, 1024>(a, threads, stream, launched)
              : launch_pipe_one<QM, LPG, RES, false, SK, 1024>(a, threads, stream, launched);
}

template <int QM, int LPG, bool RES>
cudaError_t launch_pipe(const FusedArgs& a, int threads, cudaStream_t stream, bool* launched) {
  if constexpr (QM == kQNone) {
    return launch_pipe_sk<QM, LPG, RES, kSkF32>(a, threads, stream, launched);
  } else {
    if (a.scale_layout == kLaySwizzled)
      return launch_pipe_sk<QM, LPG, RES, kSkE8Swz>(a, threads, stream, launched);
    switch (a.scale_fmt) {
      case kFmtE8M0: return launch_pipe_sk<QM, LPG, RES, kSkE8>(a, threads, stream, launched);
      case kFmtPow2: return launch_pipe_sk<QM, LPG, RES, kSkF32Pow2>(a, threads, stream, launched);
      default: return launch_pipe_sk<QM, LPG, RES, kSkF32>(a, threads, stream, launched);
    }
  }
}

// Plan of the row-staged kernel: one CTA an SM of `warps` warps, each with
// one row slot of `row_pad` bytes, plus one slot for the weights. warps == 0:
// no plan (fewer than kRowstageMinWarps fit in one CTA's shared memory).
struct RowstagePlan {
  int warps;
  int smem_bytes;
};
constexpr int kRowstageMinWarps = 4;
// Batches of fewer rows keep the CTA-per-row kernels: with about one row a
// warp the row-staged kernel cannot hide its per-row latency (measured on a
// B200 at H = 7168: 2048 rows 14.8 vs 13.9 us, 4096 rows 21.6 vs 21.9 us).
constexpr int64_t kRowstageMinRows = 4096;
RowstagePlan plan_rowstage(const void* kernel, int row_pad, int max_warps);

template <int QM, int NB, int SK>
cudaError_t launch_rowstage_one(FusedArgs a, cudaStream_t stream, bool* launched) {
  auto kernel = rowstage_rmsnorm_fp8_kernel<QM, NB, SK>;
  const RowstagePlan p = plan_rowstage(reinterpret_cast<const void*>(kernel),
                                       NB * (int)kRowstageBlockBytes, rowstage_max_warps(NB));
  *launched = false;
  if (p.warps < kRowstageMinWarps) return cudaSuccess;
  int64_t grid = device_sm_count();
  const int64_t need = (a.M + p.warps - 1) / p.warps;
  if (grid > need) grid = need;
  *launched = true;
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kernel, (unsigned)grid, (unsigned)(p.warps * 32), (size_t)p.smem_bytes,
                    stream, a);
}

template <int QM, int SK>
cudaError_t launch_rowstage_sk(const FusedArgs& a, cudaStream_t stream, bool* launched) {
  switch ((a.V + 127) / 128) {
    case 1: return launch_rowstage_one<QM, 1, SK>(a, stream, launched);
    case 2: return launch_rowstage_one<QM, 2, SK>(a, stream, launched);
    case 3: return launch_rowstage_one<QM, 3, SK>(a, stream, launched);
    case 4: return launch_rowstage_one<QM, 4, SK>(a, stream, launched);
    case 5: return launch_rowstage_one<QM, 5, SK>(a, stream, launched);
    case 6: return launch_rowstage_one<QM, 6, SK>(a, stream, launched);
    case 7: return launch_rowstage_one<QM, 7, SK>(a, stream, launched);
    case 8: return launch_rowstage_one<QM, 8, SK>(a, stream, launched);
    default: *launched = false; return cudaSuccess;  // wider rows: the other kernels
  }
}

template <int QM>
cudaError_t launch_rowstage(const FusedArgs& a, cudaStream_t stream, bool* launched) {
  if constexpr (QM == kQNone) {
    return launch_rowstage_sk<QM, kSkF32>(a, stream, launched);
  } else {
    if (QM == kQGroup && a.scale_layout == kLaySwizzled)
      return launch_rowstage_sk<QM, kSkE8Swz>(a, stream, launched);
    switch (a.scale_fmt) {
      case kFmtE8M0: return launch_rowstage_sk<QM, kSkE8>(a, stream, launched);
      case kFmtPow2: return launch_rowstage_sk<QM, kSkF32Pow2>(a, stream, launched);
      default: return launch_rowstage_sk<QM, kSkF32>(a, stream, launched);
    }
  }
}

template <int QM, int LPG, bool RES, bool NORM>
cudaError_t launch_fused_nch(const FusedArgs& a, LaunchShape sh, cudaStream_t stream) {
  // Residual-free batches of many rows: the row-staged kernel (1x128 groups,
  // one scale a row, or no quantization).
  if constexpr (NORM && !RES && (QM == kQToken || QM == kQNone || (QM == kQGroup && LPG == 4))) {
    if (sh.rowstage && a.M >= kRowstageMinRows) {
      bool launched = false;
      const cudaError_t e = launch_rowstage<QM>(a, stream, &launched);
      if (e != cudaSuccess || launched) return e;
    }
  }
  if constexpr (NORM && QM != kQToken) {
    if (sh.pipe) {
      bool launched = false;
      const cudaError_t e = launch_pipe<QM, LPG, RES>(a, sh.threads, stream, &launched);
      if (e != cudaSuccess || launched) return e;
    }
  }
  if (sh.rowwarp) {
    // no bounds predicates when the row is whole 2 KB pieces
    const bool full = a.V % 128 == 0;
    return full ? launch_rowwarp_one<QM, LPG, RES, NORM, true>(a, stream)
                : launch_rowwarp_one<QM, LPG, RES, NORM, false>(a, stream);
  }
  // Rows that fill every thread's chunks exactly take the kernel without
  // store predicates.
  const bool full = (int64_t)sh.threads * sh.nch * 4 == a.V;
  switch (sh.nch * 2 + (full ? 1 : 0)) {
    case 2: return launch_fused_one<1, QM, LPG, RES, NORM, false>(a, sh.threads, stream);
    case 3: return launch_fused_one<1, QM, LPG, RES, NORM, true>(a, sh.threads, stream);
    case 4: return launch_fused_one<2, QM, LPG, RES, NORM, false>(a, sh.threads, stream);
    case 5: return launch_fused_one<2, QM, LPG, RES, NORM, true>(a, sh.threads, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int QM, int LPG>
cudaError_t launch_fused_mode(const FusedArgs& a, LaunchShape sh, bool res, bool norm,
                              cudaStream_t stream) {
  if (!norm) {
    if constexpr (QM != kQNone) return launch_fused_nch<QM, LPG, false, false>(a, sh, stream);
    return cudaErrorInvalidValue;
  }
  return res ? launch_fused_nch<QM, LPG, true, true>(a, sh, stream)
             : launch_fused_nch<QM, LPG, false, true>(a, sh, stream);
}

// Read (and optionally clear) this translation unit's device error word.
inline cudaError_t read_device_error(int* out, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_cutie_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_cutie_device_error, &zero, sizeof(int));
  }
  *out = v;
  return e;
}

#define CUTIE_DECLARE_MODE(name)                                                          \
  cudaError_t launch_fused_##name(const FusedArgs& a, LaunchShape sh, bool res, bool norm, \
                                  cudaStream_t stream);                                   \
  cudaError_t device_error_##name(int* out, bool clear);

CUTIE_DECLARE_MODE(none)
CUTIE_DECLARE_MODE(token)
CUTIE_DECLARE_MODE(g32)
CUTIE_DECLARE_MODE(g64)
CUTIE_DECLARE_MODE(g128)

// Backward of the fused path (backward.cu).
struct BwdArgs {
  const uint16_t* dn;   // d normalized, bf16 [M, H]
  int64_t lddn;
  const uint16_t* r;    // forward RMSNorm input (x + residual), bf16 [M, H]
  int64_t ldr;
  const uint16_t* w;    // weight [H]
  const uint16_t* dro;  // d residual_out (may be null)
  int64_t lddro;
  uint16_t* dx;         // d x (= d residual), bf16 [M, H]
  int64_t lddx;
  float* partial;       // [gridDim.x, H] fp32 partial sums of dw (null: no dw)
  FusedArgs qa;         // quantization of dx: q, ldq, scale, s_row, s_grp, n_groups(_pad),
                        // scale_fmt, scale_layout, M, M_pad, H, V (q == null: none)
};

// Threads of a row and CTAs of a backward launch (the CTAs are also the rows
// of dw partial sums the workspace holds).
void backward_shape(int64_t M, int64_t H, int* threads, int* grid);
// Floats of the d_weight scratch the allocation-free backward keeps in a
// device array of the library (backward.cu), and that array's address in the
// current context (resolved on every call).
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 20;
cudaError_t noalloc_scratch(float** out);

// Device error word of backward.cu (see read_device_error).
cudaError_t device_error_bwd(int* out, bool clear);

// MXFP8 block-scaled GEMM (gemm_mxfp8.cu): arguments checked by the caller;
// returns a CUTIE_* status and, on failure, points *why at a message.
int gemm_mxfp8(const void* a, int64_t lda, const void* a_scale, const void* b, int64_t ldb,
               const void* b_scale, void* d, int64_t ldd, int64_t M, int64_t N, int64_t K,
               cudaStream_t stream, const char** why);
cudaError_t device_error_gemm(int* out, bool clear);

// Fused RMSNorm -> MXFP8 -> block-scaled GEMM (gemm_prologue.cu): arguments
// checked by the caller (q and q_scale both null or both set); same status
// convention as gemm_mxfp8.
int gemm_rmsnorm_mxfp8(const void* x, int64_t ldx, const void* weight, float eps, const void* b,
                       int64_t ldb, const void* b_scale, void* d, int64_t ldd, int64_t M,
                       int64_t N, int64_t K, void* q, int64_t ldq, void* q_scale,
                       long long wait_limit, cudaStream_t stream, const char** why);
cudaError_t device_error_prologue(int* out, bool clear);

// max_grid > 0 caps the CTAs (and so the rows of partial sums in a.partial).
cudaError_t launch_backward(const BwdArgs& a, float eps, bool dw_wanted, uint16_t* dw,
                            int max_grid, cudaStream_t st);

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

// The fp32 kernel keeps its own register layout (NV vectors a thread).
struct F32Shape {
  int nv;
  int threads;
};
cudaError_t launch_rmsnorm_f32(const F32Args& a, F32Shape sh, cudaStream_t stream);

}  // namespace cutie
