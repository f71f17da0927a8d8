/*
 * cutie.h — C ABI of the B200 (sm_100a) residual-add + RMSNorm + FP8 (e4m3)
 * activation-quantization path.
 *
 * Every entry point is destination-passing: the caller owns and preallocates
 * all device buffers, nothing is allocated inside, and the work is enqueued
 * asynchronously on the caller's CUDA stream (`stream` is a cudaStream_t; NULL
 * means the legacy default stream) on the calling thread's current device.
 * No C++ exception crosses this boundary: every function returns a status code
 * (CUTIE_OK == 0) and, on failure, a message readable through
 * cutie_last_error() on the same thread.
 *
 * Reference interfaces replaced (paths within the S1ro1/thingy project):
 *   cutie_rms_norm_fp8          <- RMSNorm.__call__ / rms_norm_kernel
 *                                  (src/cutie/rms_norm/rms_norm.py:50-311),
 *                                  compiled and bound through cute.compile at
 *                                  src/cutie/rms_norm/bench.py:278-301, and the
 *                                  functional reference it must agree with,
 *                                  residual_rms_norm_fp8_reference
 *                                  (src/cutie/rms_norm/bench.py:83-100).
 *   cutie_per_token_cast_to_fp8 <- per_token_cast_to_fp8_triton /
 *                                  _per_token_fp8_kernel
 *                                  (src/cutie/vendor/prime_rl/fp8_utils.py:21-89),
 *                                  the op behind the custom op
 *                                  cutie::per_token_fp8_quant
 *                                  (src/cutie/rms_norm/bench.py:68-80).
 *   cutie_rms_norm              <- rms_norm / rms_norm_on_stream
 *                                  (src/cutie/rms_norm/rms_norm.py:11-33, fp32)
 *                                  and rms_norm_reference
 *                                  (src/cutie/rms_norm/bench.py:58-65, bf16).
 */
#ifndef CUTIE_H_
#define CUTIE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUTIE_ABI_VERSION 1

#if defined(__GNUC__)
#define CUTIE_API __attribute__((visibility("default")))
#else
#define CUTIE_API
#endif

/* ---- status codes ------------------------------------------------------- */
enum cutie_status {
  CUTIE_OK = 0,
  CUTIE_ERR_INVALID_ARGUMENT = -1, /* bad shape, null pointer, bad enum      */
  CUTIE_ERR_UNSUPPORTED = -2,      /* valid request this build cannot serve  */
  CUTIE_ERR_ALIGNMENT = -3,        /* pointer / leading dim not 16-B aligned */
  CUTIE_ERR_CUDA = -4,             /* a CUDA runtime call failed             */
};

/* ---- quantization granularity (who shares one scale) -------------------- */
enum cutie_quant_mode {
  CUTIE_QUANT_NONE = 0,  /* no FP8 output (plain RMSNorm)                    */
  CUTIE_QUANT_TOKEN = 1, /* one scale per row (group = H)                    */
  CUTIE_QUANT_GROUP = 2, /* one scale per `group_size` contiguous elements   */
};

/* ---- how a scale is encoded --------------------------------------------- */
enum cutie_scale_fmt {
  CUTIE_SCALE_FP32 = 0,      /* fp32 s = max(amax/448, 1e-4)                 */
  CUTIE_SCALE_FP32_POW2 = 1, /* fp32 s = 2^ceil(log2(max(amax/448, 1e-4)))   */
                             /* (the reference's use_ue8m0=True rule)        */
  CUTIE_SCALE_E8M0 = 2,      /* one byte: biased exponent of the POW2 scale  */
};

/* ---- where scale (row m, group g) lives --------------------------------- */
enum cutie_scale_layout {
  CUTIE_LAYOUT_ROW_MAJOR = 0,   /* scale[m * ld_scale + g], ld >= n_groups   */
  CUTIE_LAYOUT_COL_MAJOR = 1,   /* scale[g * ld_scale + m], ld >= M          */
  CUTIE_LAYOUT_MX_SWIZZLED = 2, /* Blackwell block-scaled-GEMM layout:       */
  /* 128x4 tiles of 512 bytes, tile (m/128, g/4) at ((m/128)*ceil(G/4)+g/4)*512,
   * inside a tile (m%32)*16 + ((m%128)/32)*4 + g%4. Rows are padded to a
   * multiple of 128 and groups to a multiple of 4; padding bytes are written
   * as 0. Requires CUTIE_SCALE_E8M0. ld_scale is ignored.                   */
  CUTIE_LAYOUT_COL_MAJOR_PACKED = 3, /* e8m0 exponents packed four to a     */
  /* little-endian 32-bit word along the groups, words M-major: scale (m, g) is
   * byte g%4 of word (g/4)*ld_scale + m, i.e. byte offset
   * (g/4)*4*ld_scale + 4*m + g%4 (the packed UE8M0 scale tensor that
   * DeepGEMM-style SM100 FP8 GEMMs take: int32 [M, ceil(G/4)], stride
   * (1, ld_scale)). ld_scale counts words, >= M; 0 means M rounded up to a
   * multiple of 4 (16-byte aligned columns). Bytes of groups past the last
   * one in the final word are not written. Requires CUTIE_SCALE_E8M0.
   * No counterpart in the reference, which writes fp32 row-major scales.  */
};

/* ---- element types for cutie_rms_norm ----------------------------------- */
enum cutie_dtype {
  CUTIE_DTYPE_BF16 = 0,
  CUTIE_DTYPE_F32 = 1,
};

/*
 * Fused [residual add] -> RMSNorm -> [FP8 e4m3 quantization].
 *
 *   r   = bf16(x + residual)                (or r = x when residual is NULL)
 *   inv = 1 / RN(sqrt(RN(sum(r^2) / H) + eps))            (fp32 statistics)
 *   n   = bf16( bf16(r * inv) * weight )    (cast before the weight multiply)
 *   per group: amax = max|n|, s = max(amax / 448, 1e-4) [, rounded up to 2^k]
 *   q   = e4m3_rne(RN(n / s))
 *
 * x, residual, weight, residual_out, normalized_out: bf16. q: e4m3 bytes.
 * M >= 0 rows, H > 0 columns, H % 8 == 0; in CUTIE_QUANT_GROUP mode
 * group_size is 32, 64 or 128 and the last group of a row may be partial
 * (n_groups = ceil(H / group_size)). Leading dimensions are in elements; every
 * row must start 16-byte aligned. residual_out / normalized_out may be NULL
 * (not written); residual_out requires residual. q and scale may be NULL only
 * when quant_mode == CUTIE_QUANT_NONE. ld_scale == 0 selects the dense leading
 * dimension (n_groups for row-major, M for column-major).
 * threads_per_row: 0 picks the launch shape; otherwise a multiple of 32 in
 * [32, 1024] that must cover the row with at most 8 16-byte vectors a thread.
 */
CUTIE_API int cutie_rms_norm_fp8(const void* x, int64_t ldx,
                       const void* residual, int64_t ldr,
                       const void* weight, float eps,
                       int64_t M, int64_t H,
                       int quant_mode, int group_size,
                       int scale_fmt, int scale_layout, int64_t ld_scale,
                       void* q, int64_t ldq, void* scale,
                       void* residual_out, int64_t ldro,
                       void* normalized_out, int64_t ldn,
                       int threads_per_row, void* stream);

/*
 * Quantization alone: bf16 x [M, H] -> e4m3 q [M, H] + scales, one scale per
 * (row, group). Same scale rules, formats and layouts as above; group_size 0
 * means one scale per row. Mirrors per_token_cast_to_fp8_triton(x, use_ue8m0,
 * gran_k) (src/cutie/vendor/prime_rl/fp8_utils.py:63-89), whose defaults are
 * group_size 128, CUTIE_SCALE_FP32 (use_ue8m0=False) or CUTIE_SCALE_FP32_POW2
 * (use_ue8m0=True), row-major [M, ceil(H/128)] scales.
 */
CUTIE_API int cutie_per_token_cast_to_fp8(const void* x, int64_t ldx,
                                int64_t M, int64_t H, int group_size,
                                int scale_fmt, int scale_layout,
                                int64_t ld_scale,
                                void* q, int64_t ldq, void* scale,
                                int threads_per_row, void* stream);

/*
 * Standalone RMSNorm, out = f(x) [M, H].
 *   dtype == CUTIE_DTYPE_BF16: out = bf16(bf16(x * inv) * w), inv as above
 *     (rms_norm_reference, src/cutie/rms_norm/bench.py:58-65).
 *   dtype == CUTIE_DTYPE_F32:  out = RN(RN(x / RN(sqrt(RN(mean(RN(x^2))) + eps))) * w)
 *     (rms_norm, src/cutie/rms_norm/rms_norm.py:11-20).
 * x, weight and out share `dtype`. H % 8 == 0 (bf16) or H % 4 == 0 (f32).
 */
CUTIE_API int cutie_rms_norm(const void* x, int64_t ldx, const void* weight, float eps,
                   int64_t M, int64_t H, int dtype,
                   void* out, int64_t ldo, int threads_per_row, void* stream);

/*
 * Backward of cutie_rms_norm_fp8 (bf16, with or without a residual). The
 * reference has no backward pass (src/cutie/rms_norm/bench.py is forward
 * only); these are the gradients torch autograd gives its PyTorch forward
 * (bench.py:58-65 and the residual add of bench.py:97), op for op in fp32:
 *   inv = the forward's inv_rms of r;  dt = bf16(dn * w);  b = sum(dt * r)
 *   dx  = bf16(bf16(dt * inv + ((-0.5 * b) * inv^3 / H) * (2 * r)) + dro)
 *   dw  = bf16(sum over rows of bf16(dn * bf16(r * inv)))
 * d_normalized (dn): bf16 [M, H] gradient of the normalized output;
 * r: bf16 [M, H], the forward's RMSNorm input (x + residual, i.e.
 * residual_out, or x); d_residual_out (dro): gradient of residual_out, or
 * NULL; dx: bf16 [M, H], the gradient of x and of residual; d_weight: bf16
 * [H] or NULL. The weight gradient is summed per CTA into `workspace` (fp32,
 * at least cutie_rms_norm_backward_workspace(M, H) bytes, 16-byte aligned,
 * caller-owned, contents need not be initialised) and reduced over CTAs in a
 * fixed order, so it is deterministic. quant_mode CUTIE_QUANT_GROUP with
 * group_size 128 also writes dx as FP8 codes q + scales (formats and layouts
 * as in cutie_rms_norm_fp8); CUTIE_QUANT_NONE writes none. H % 8 == 0,
 * H <= 32768. Asynchronous on `stream`; nothing is allocated.
 */
CUTIE_API int cutie_rms_norm_backward(const void* d_normalized, int64_t ldd,
                                      const void* r, int64_t ldr, const void* weight,
                                      const void* d_residual_out, int64_t lddr,
                                      float eps, int64_t M, int64_t H,
                                      void* dx, int64_t lddx, void* d_weight,
                                      void* workspace, size_t workspace_bytes,
                                      int quant_mode, int group_size, int scale_fmt,
                                      int scale_layout, int64_t ld_scale,
                                      void* q, int64_t ldq, void* scale, void* stream);

/* Workspace bytes cutie_rms_norm_backward needs for d_weight on the current
 * device (one fp32 row of H partial sums per CTA of its grid). */
CUTIE_API size_t cutie_rms_norm_backward_workspace(int64_t M, int64_t H);

/*
 * cutie_rms_norm_backward without a workspace argument: it allocates nothing
 * and needs no device memory from the caller beyond inputs and outputs. It
 * has no counterpart in the reference. It is for callers that cannot
 * allocate device memory: code that runs where a cudaMalloc is not allowed
 * or must not happen (inside an allocator's or a framework's callbacks, a
 * plug-in whose host owns every device buffer, a memory pool that must not
 * grow), or that cannot hold a workspace between calls.
 *
 * The partial sums of d_weight go to a device array of the library instead:
 * 2^20 floats (4 MiB), present on every GPU that loads the library until the
 * process exits. Its CTAs are capped so that their rows of H partial sums
 * fit (2^20 / H CTAs, e.g. 146 at H = 7168), so d_weight is summed in a
 * different grouping than cutie_rms_norm_backward's (the same bound on the
 * error; dx, q and scale are identical). The cap costs time where it is
 * below the regular grid: measured on a B200 (residual gradient, 1x128 FP8
 * copy of dx) 210.6 against 183.4 us at 16384 x 7168 (146 CTAs), 122.8
 * against 116.6 us at 16384 x 4096, 881 against 236 us at 2048 x 32768
 * (32 CTAs). Sizes: as cutie_rms_norm_backward
 * (H <= 32768, which always fits the array); a larger H is refused with
 * CUTIE_ERR_UNSUPPORTED. Every row of the array that a call reads was
 * written by that call, so nothing needs clearing between calls.
 *
 * Every call resolves the array's device address in the calling thread's
 * current context (cudaGetSymbolAddress; nothing is cached, so the address
 * stays right after cudaDeviceReset or under another driver context). The
 * first call in a context also loads the library's device code there: make
 * that first call before any stream capture. All calls on a device share the
 * one array, so calls that may run at the same time on the GPU (other
 * streams, other host threads) race on it and give wrong d_weight: order
 * them on one stream.
 */
CUTIE_API int cutie_rms_norm_backward_noalloc(const void* d_normalized, int64_t ldd,
                                              const void* r, int64_t ldr, const void* weight,
                                              const void* d_residual_out, int64_t lddr,
                                              float eps, int64_t M, int64_t H,
                                              void* dx, int64_t lddx, void* d_weight,
                                              int quant_mode, int group_size, int scale_fmt,
                                              int scale_layout, int64_t ld_scale,
                                              void* q, int64_t ldq, void* scale, void* stream);

/*
 * MXFP8 block-scaled GEMM on the tensor cores, the consumer of this path's
 * 1x32 codes and swizzled e8m0 scales (no counterpart in the reference, whose
 * bench stops before the GEMM, src/cutie/rms_norm/bench.py:4-7):
 *   D[m, n] = bf16( sum_k A[m, k] 2^(sA[m, k/32] - 127) * B[n, k] 2^(sB[n, k/32] - 127) )
 * with fp32 accumulation. a: e4m3 [M, K] (K contiguous, lda bytes between
 * rows), a_scale: its e8m0 scales in CUTIE_LAYOUT_MX_SWIZZLED for [M, K/32]
 * (rows padded to 128, as cutie_rms_norm_fp8 writes them); b: e4m3 [N, K]
 * (ldb) with b_scale likewise for [N, K/32]; d: bf16 [M, N] (ldd elements).
 * N and K multiples of 128, any M >= 0; a, b, d rows and both scale buffers
 * 16-byte aligned. Asynchronous on `stream`; nothing is allocated.
 */
CUTIE_API int cutie_gemm_mxfp8(const void* a, int64_t lda, const void* a_scale,
                               const void* b, int64_t ldb, const void* b_scale,
                               void* d, int64_t ldd, int64_t M, int64_t N, int64_t K,
                               void* stream);

/*
 * RMSNorm -> MXFP8 quantization -> block-scaled GEMM in ONE kernel: the
 * norm-and-quantize step becomes the GEMM's A-operand prologue, so the FP8
 * codes and scales of the activation never leave the chip (no counterpart in
 * the reference; it composes rms_norm_reference, src/cutie/rms_norm/bench.py:
 * 58-65, the 1x32 UE8M0 quantizer rule of src/cutie/vendor/prime_rl/
 * fp8_utils.py:50-57 with gran_k 32, and the GEMM its output feeds):
 *   A = cutie_rms_norm_fp8(x, weight, eps, group 32, e8m0, swizzled) codes,
 *   D[m, n] = bf16( sum_k A[m, k] 2^(sA[m, k/32] - 127) * b[n, k] 2^(sB[n, k/32] - 127) )
 * x: bf16 [M, K] (ldx elements, 16-byte aligned rows), weight: bf16 [K];
 * b / b_scale / d as cutie_gemm_mxfp8. q / q_scale: both NULL, or an e4m3
 * [M, K] buffer (ldq bytes) and a swizzled e8m0 scale buffer that receive A
 * and its scales as cutie_rms_norm_fp8 would write them (for a backward pass
 * that keeps the quantized activation). N and K multiples of 128,
 * K <= 65536. The CTAs that share 128 rows of x run as a thread-block cluster
 * (8, 4, 2 or 1 CTAs along N, the largest that divides N / 128) and quantize
 * each A tile once between them. Asynchronous on `stream`; nothing is
 * allocated.
 */
CUTIE_API int cutie_rms_norm_mxfp8_gemm(const void* x, int64_t ldx, const void* weight,
                                        float eps, const void* b, int64_t ldb,
                                        const void* b_scale, void* d, int64_t ldd, int64_t M,
                                        int64_t N, int64_t K, void* q, int64_t ldq,
                                        void* q_scale, void* stream);

/*
 * Device-side status of this library's kernels on the current device: 0 when
 * no kernel has hit a failure since the last clear; otherwise the first error
 * code recorded (1 = a bulk-copy wait ran out: a row never arrived in shared
 * memory within ~2 s and the kernel stopped early, leaving outputs
 * incomplete, see cutie_set_wait_limit; 2 = a kernel was launched with a
 * shared-memory ring depth it does not hold and wrote nothing). Synchronises with the device; `clear` != 0
 * resets the word.
 * A negative return is a CUDA failure (see cutie_last_error()).
 */
CUTIE_API int cutie_device_error(int clear);

/*
 * Limit, in SM clock cycles, on every wait that the kernels launched later
 * by the calling thread make for their own bulk copies and row exchanges
 * (the default, about 2 s, bounds a copy that never lands). A wait that runs
 * out stops the kernel early with device error 1 (cutie_device_error); the
 * kernel first lets the copies it issued land, so the GPU stays usable.
 * cycles == 0 restores the default; cycles < 0 makes every wait that would
 * have to block give up at once, which exercises that failure path with
 * valid inputs (the outputs of such a launch are incomplete). Affects this
 * thread only; returns the previous limit. No counterpart in the reference,
 * whose kernels have no waits that can run out.
 */
CUTIE_API int64_t cutie_set_wait_limit(int64_t cycles);

/* Message of the last failing call on this thread ("" if none). */
CUTIE_API const char* cutie_last_error(void);

/* CUTIE_ABI_VERSION of the loaded library. */
CUTIE_API int cutie_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CUTIE_H_ */
