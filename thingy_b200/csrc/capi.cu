// extern "C" entry points declared in include/cutie.h: argument validation,
// launch-shape choice and dispatch to the per-mode launchers. No allocation,
// no host synchronisation; errors come back as status codes plus a
// thread-local message.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "cutie.h"
#include "launch.cuh"

namespace cutie {

namespace {

thread_local char g_err[512] = "";

// Limit (SM cycles) on every wait of the kernels this thread launches; set
// through cutie_set_wait_limit, kWaitLimitCycles by default.
thread_local long long g_wait_limit = kWaitLimitCycles;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CUTIE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

}  // namespace

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < kMaxDevices) {
    const int cached = g_sm_count[dev].load(std::memory_order_relaxed);
    if (cached > 0) return cached;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < kMaxDevices) g_sm_count[dev].store(n, std::memory_order_relaxed);
  return n;
}

int cached_blocks_per_sm(const void* kernel, int threads, int dyn_smem) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) * 0x9E3779B97F4A7C15ull) ^
                       (static_cast<uint64_t>(threads) << 40) ^
                       (static_cast<uint64_t>(dyn_smem) << 8) ^ static_cast<uint64_t>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, dyn_smem) != cudaSuccess)
    return 0;
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

namespace {
std::mutex g_attr_mu;
std::unordered_map<const void*, int> g_attr_raised;  // kernel -> dynamic smem limit set
}  // namespace

int set_smem_and_occupancy(const void* kernel, int threads, int smem) {
  {
    std::lock_guard<std::mutex> lock(g_attr_mu);
    int& have = g_attr_raised[kernel];
    if (smem > have) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess)
        return 0;
      have = smem;
    }
  }
  return cached_blocks_per_sm(kernel, threads, smem);
}

// Ring depth of the warp-per-row kernel (2 KB slots per warp).
int rowwarp_stages() { return 3; }

BulkPlan plan_bulk(const void* kernel, int threads, int stage_bytes, int max_stages) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, BulkPlan> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) * 0x9E3779B97F4A7C15ull) ^
                       (static_cast<uint64_t>(threads) << 44) ^
                       (static_cast<uint64_t>(stage_bytes) << 12) ^
                       (static_cast<uint64_t>(max_stages) << 6) ^ static_cast<uint64_t>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  BulkPlan plan{0, 0, 0};
  int sm_smem = 0, block_smem = 0, reserved = 0;
  cudaFuncAttributes attr{};
  if (cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&block_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) !=
          cudaSuccess ||
      cudaFuncGetAttributes(&attr, kernel) != cudaSuccess)
    return plan;
  const int by_regs = cached_blocks_per_sm(kernel, threads, 0);
  // Prefer >= 2 stages (prefetch two rows ahead); rows too wide for that on
  // one SM still run with one stage (its refill overlaps the row's compute).
  for (int b = by_regs; b >= 1 && plan.stages < 2; --b) {
    int room = sm_smem / b - reserved - (int)attr.sharedSizeBytes;
    if (room > block_smem - (int)attr.sharedSizeBytes) room = block_smem - (int)attr.sharedSizeBytes;
    int stages = room / (stage_bytes + 8);
    if (stages > max_stages) stages = max_stages;
    if (stages >= 2) {
      plan.stages = stages;
      plan.blocks_per_sm = b;
      plan.smem_bytes = stages * (stage_bytes + 8);
    }
  }
  if (plan.stages < 2) {
    int room = block_smem - (int)attr.sharedSizeBytes - reserved;
    if (room >= stage_bytes + 8) plan = BulkPlan{1, 1, stage_bytes + 8};
  }
  if (plan.stages >= 1) {
    // The limit is a property of the kernel, shared by every plan of it:
    // it is only ever raised, so plans cached for larger rows stay launchable.
    const int n = set_smem_and_occupancy(kernel, threads, plan.smem_bytes);
    if (n <= 0) plan = BulkPlan{0, 0, 0};
    else plan.blocks_per_sm = n;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = plan;
  return plan;
}

BulkPlan plan_pipe(const void* kernel, int threads, int stage_bytes) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, BulkPlan> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) * 0x9E3779B97F4A7C15ull) ^
                       (static_cast<uint64_t>(threads) << 44) ^
                       (static_cast<uint64_t>(stage_bytes) << 12) ^ static_cast<uint64_t>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  BulkPlan plan{0, 0, 0};
  int sm_smem = 0, block_smem = 0, reserved = 0;
  cudaFuncAttributes attr{};
  if (cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&block_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) !=
          cudaSuccess ||
      cudaFuncGetAttributes(&attr, kernel) != cudaSuccess)
    return plan;
  const int by_regs = cached_blocks_per_sm(kernel, threads, 0);
  int best = 0;
  for (int stages = 3; stages >= 2; --stages) {
    const int dyn = stages * stage_bytes;
    if (dyn + (int)attr.sharedSizeBytes > block_smem) continue;
    int b = sm_smem / (dyn + (int)attr.sharedSizeBytes + reserved);
    if (b > by_regs) b = by_regs;
    if (b * stages > best) {
      best = b * stages;
      plan = BulkPlan{stages, b, dyn};
    }
  }
  if (plan.stages >= 2) {
    const int n = set_smem_and_occupancy(kernel, threads, plan.smem_bytes);
    if (n <= 0) plan = BulkPlan{0, 0, 0};
    else plan.blocks_per_sm = n;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = plan;
  return plan;
}

RowstagePlan plan_rowstage(const void* kernel, int row_pad, int max_warps) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, RowstagePlan> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) * 0x9E3779B97F4A7C15ull) ^
                       (static_cast<uint64_t>(row_pad) << 12) ^ static_cast<uint64_t>(dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  RowstagePlan plan{0, 0};
  int block_smem = 0;
  cudaFuncAttributes attr{};
  if (cudaDeviceGetAttribute(&block_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
          cudaSuccess ||
      cudaFuncGetAttributes(&attr, kernel) != cudaSuccess)
    return plan;
  // one slot a warp plus the weights' slot, as many warps as fit (and as the
  // kernel's register budget allows)
  int warps = (block_smem - (int)attr.sharedSizeBytes) / row_pad - 1;
  if (warps > max_warps) warps = max_warps;
  if (warps >= kRowstageMinWarps) {
    plan = RowstagePlan{warps, (warps + 1) * row_pad};
    if (set_smem_and_occupancy(kernel, warps * 32, plan.smem_bytes) <= 0) plan = RowstagePlan{0, 0};
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = plan;
  return plan;
}

namespace {


// Launch shape for a row of V 16-byte vectors (NC 64-byte chunks).
//  * threads_per_row == 32: one warp per row, the two-pass kernel (any H).
//  * larger requests, and the automatic choice: the single-pass kernel with
//    one CTA per row, one chunk per thread (two when the row is wider than
//    1024 chunks); rows wider than that stream through the warp-per-row
//    kernel (unless an output aliases an input: it re-reads its inputs).
int pick_shape(int64_t V, int64_t M, int requested, bool aliased, LaunchShape* out) {
  const int64_t NC = (V + 3) / 4;
  if (requested == 32) {
    if (aliased)
      return fail(CUTIE_ERR_UNSUPPORTED,
                  "threads_per_row=32 (one warp per row) re-reads its inputs and cannot run "
                  "with an output that aliases an input");
    *out = {1, 32, true};
    return CUTIE_OK;
  }
  if (requested != 0) {
    if (requested < 32 || requested > 1024 || requested % 32 != 0)
      return fail(CUTIE_ERR_INVALID_ARGUMENT,
                  "threads_per_row must be 0 or a multiple of 32 in [32, 1024], got %d",
                  requested);
    const int64_t nch = (NC + requested - 1) / requested;
    if (nch > 2 || (nch == 2 && requested > 512))
      return fail(CUTIE_ERR_UNSUPPORTED,
                  "threads_per_row=%d leaves %lld 64-byte chunks per thread for a %lld-chunk "
                  "row (at most 1, or 2 with at most 512 threads)",
                  requested, (long long)nch, (long long)NC);
    *out = {nch < 1 ? 1 : (int)nch, requested, false, nch <= 1};
    return CUTIE_OK;
  }
  int64_t T = (NC + 31) / 32 * 32;
  if (T < 32) T = 32;
  if (T <= 1024) {
    *out = {1, (int)T, false, true, true};
    return CUTIE_OK;
  }
  T = ((NC + 1) / 2 + 31) / 32 * 32;
  if (T <= 512) {
    *out = {2, (int)T, false, false, true};
    return CUTIE_OK;
  }
  if (!aliased) {  // wider rows than one CTA can hold: stream them per warp
    *out = {1, 32, true};
    return CUTIE_OK;
  }
  return fail(CUTIE_ERR_UNSUPPORTED,
              "H=%lld with an output aliasing an input is wider than the single-pass kernel "
              "supports (32768)",
              (long long)V * 8);
}

// fp32 kernel: NV 16-byte vectors (4 floats) a thread, least idle lanes.
int pick_f32_shape(int64_t V, int64_t M, int requested, F32Shape* out) {
  auto max_threads_for = [](int nv) { return nv > 4 ? 512 : 1024; };
  if (requested != 0) {
    if (requested < 32 || requested > 1024 || requested % 32 != 0)
      return fail(CUTIE_ERR_INVALID_ARGUMENT,
                  "threads_per_row must be 0 or a multiple of 32 in [32, 1024], got %d",
                  requested);
    int64_t nv = (V + requested - 1) / requested;
    if (nv < 1) nv = 1;
    if (nv > 8 || requested > max_threads_for((int)nv))
      return fail(CUTIE_ERR_UNSUPPORTED,
                  "threads_per_row=%d leaves %lld vectors per thread for a %lld-vector row",
                  requested, (long long)nv, (long long)V);
    *out = {(int)nv, requested};
    return CUTIE_OK;
  }
  static const int kPrefMany[8] = {4, 3, 5, 2, 6, 7, 8, 1};
  static const int kPrefFew[8] = {1, 2, 3, 4, 5, 6, 7, 8};
  const int sms = device_sm_count();
  const int* pref = (M < 2 * (int64_t)(sms > 0 ? sms : 148)) ? kPrefFew : kPrefMany;
  int64_t best_waste = -1;
  for (int i = 0; i < 8; ++i) {
    const int nv = pref[i];
    int64_t T = (V + nv - 1) / nv;
    T = ((T + 31) / 32) * 32;
    if (T < 32) T = 32;
    if (T > max_threads_for(nv)) continue;
    const int64_t waste = T * nv - V;
    if (best_waste < 0 || waste < best_waste) {
      best_waste = waste;
      *out = {nv, (int)T};
    }
  }
  if (best_waste < 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld is wider than this build supports (16384)",
                (long long)V * 4);
  return CUTIE_OK;
}

int check_matrix(const char* name, const void* p, int64_t ld, int64_t H, uintptr_t align,
                 int64_t ld_multiple) {
  if (p == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "%s is NULL", name);
  if (ld < H)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "%s: leading dimension %lld < H=%lld", name,
                (long long)ld, (long long)H);
  if (!aligned(p, align) || ld % ld_multiple != 0)
    return fail(CUTIE_ERR_ALIGNMENT,
                "%s: rows must start %d-byte aligned (pointer %p, leading dimension %lld)",
                name, (int)align, p, (long long)ld);
  return CUTIE_OK;
}

// Strides of a strided scale layout: element offset of (row m, group g) =
// m*s_row + (g/4)*s_grp4 + (g%4)*s_grp. Row- and column-major take ld_scale
// elements (0: dense); the packed layout takes ld_scale 32-bit words (0: M
// rounded up to 4, 16-byte aligned columns) and e8m0 scales only.
int strided_scale(int layout, int fmt, int64_t ld_scale, int64_t M, int64_t n_groups,
                  int64_t* s_row, int64_t* s_grp, int64_t* s_grp4) {
  if (layout == CUTIE_LAYOUT_ROW_MAJOR) {
    const int64_t ld = ld_scale == 0 ? n_groups : ld_scale;
    if (ld < n_groups)
      return fail(CUTIE_ERR_INVALID_ARGUMENT, "ld_scale %lld < %lld groups",
                  (long long)ld_scale, (long long)n_groups);
    *s_row = ld;
    *s_grp = 1;
  } else if (layout == CUTIE_LAYOUT_COL_MAJOR) {
    const int64_t ld = ld_scale == 0 ? M : ld_scale;
    if (ld < M)
      return fail(CUTIE_ERR_INVALID_ARGUMENT, "ld_scale %lld < M=%lld", (long long)ld_scale,
                  (long long)M);
    *s_row = 1;
    *s_grp = ld;
  } else if (layout == CUTIE_LAYOUT_COL_MAJOR_PACKED) {
    if (fmt != CUTIE_SCALE_E8M0)
      return fail(CUTIE_ERR_INVALID_ARGUMENT, "the packed scale layout needs E8M0 scales");
    const int64_t ld = ld_scale == 0 ? (M + 3) / 4 * 4 : ld_scale;
    if (ld < M)
      return fail(CUTIE_ERR_INVALID_ARGUMENT, "ld_scale %lld words < M=%lld",
                  (long long)ld_scale, (long long)M);
    *s_row = 4;  // bytes: one 32-bit word a row
    *s_grp = 1;
    *s_grp4 = 4 * ld;
    return CUTIE_OK;
  } else {
    return CUTIE_OK;  // swizzled: addressed by its own map
  }
  *s_grp4 = 4 * *s_grp;
  return CUTIE_OK;
}

int run_fused(bool norm, const void* x, int64_t ldx, const void* residual, int64_t ldr,
              const void* weight, float eps, int64_t M, int64_t H, int quant_mode,
              int group_size, int scale_fmt, int scale_layout, int64_t ld_scale, void* q,
              int64_t ldq, void* scale, void* residual_out, int64_t ldro, void* normalized_out,
              int64_t ldn, int threads_per_row, void* stream) {
  g_err[0] = '\0';
  if (M < 0 || H <= 0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "need M >= 0 and H > 0 (got M=%lld, H=%lld)",
                (long long)M, (long long)H);
  if (H % 8 != 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld must be a multiple of 8 (16-byte rows)",
                (long long)H);
  if (H > (int64_t)1 << 30) return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld too large", (long long)H);
  if (!(eps >= 0.0f) || std::isinf(eps))
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
  if (quant_mode < CUTIE_QUANT_NONE || quant_mode > CUTIE_QUANT_GROUP)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown quant_mode %d", quant_mode);
  if (scale_fmt < CUTIE_SCALE_FP32 || scale_fmt > CUTIE_SCALE_E8M0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown scale_fmt %d", scale_fmt);
  if (scale_layout < CUTIE_LAYOUT_ROW_MAJOR || scale_layout > CUTIE_LAYOUT_COL_MAJOR_PACKED)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown scale_layout %d", scale_layout);
  const bool quant = quant_mode != CUTIE_QUANT_NONE;
  if (!norm && !quant)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "quantization-only call without quantization");
  if (quant_mode == CUTIE_QUANT_GROUP && group_size != 32 && group_size != 64 &&
      group_size != 128)
    return fail(CUTIE_ERR_UNSUPPORTED, "group_size must be 32, 64 or 128 (got %d)", group_size);
  if (residual_out != nullptr && residual == nullptr)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "residual_out requires residual");
  if (!quant && normalized_out == nullptr && residual_out == nullptr)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "no output requested");
  if (scale_layout == CUTIE_LAYOUT_MX_SWIZZLED && quant &&
      (quant_mode != CUTIE_QUANT_GROUP || scale_fmt != CUTIE_SCALE_E8M0))
    return fail(CUTIE_ERR_INVALID_ARGUMENT,
                "the swizzled scale layout needs group quantization with E8M0 scales");

  const int64_t n_groups = quant_mode == CUTIE_QUANT_GROUP ? (H + group_size - 1) / group_size : 1;
  const bool swz = quant && scale_layout == CUTIE_LAYOUT_MX_SWIZZLED;
  const int64_t n_groups_pad = swz ? (n_groups + 3) / 4 * 4 : n_groups;
  const int64_t M_pad = swz ? (M + 127) / 128 * 128 : M;
  if (M_pad == 0) return CUTIE_OK;

  int rc;
  if ((rc = check_matrix("x", x, ldx, H, 16, 8)) != CUTIE_OK) return rc;
  if (residual != nullptr && (rc = check_matrix("residual", residual, ldr, H, 16, 8)) != CUTIE_OK)
    return rc;
  if (residual_out != nullptr &&
      (rc = check_matrix("residual_out", residual_out, ldro, H, 16, 8)) != CUTIE_OK)
    return rc;
  if (normalized_out != nullptr &&
      (rc = check_matrix("normalized_out", normalized_out, ldn, H, 16, 8)) != CUTIE_OK)
    return rc;
  if (norm) {
    if (weight == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "weight is NULL");
    if (!aligned(weight, 16)) return fail(CUTIE_ERR_ALIGNMENT, "weight must be 16-byte aligned");
  }
  int64_t s_row = 0, s_grp = 0, s_grp4 = 0;
  if (quant) {
    if ((rc = check_matrix("q", q, ldq, H, 8, 8)) != CUTIE_OK) return rc;
    if (scale == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "scale is NULL");
    if (scale_fmt != CUTIE_SCALE_E8M0 && !aligned(scale, 4))
      return fail(CUTIE_ERR_ALIGNMENT, "fp32 scales must be 4-byte aligned");
    if ((rc = strided_scale(scale_layout, scale_fmt, ld_scale, M, n_groups, &s_row, &s_grp,
                            &s_grp4)) != CUTIE_OK)
      return rc;
  }

  const int64_t V = H / 8;
  LaunchShape sh{};
  const bool aliased =
      (residual_out != nullptr && (residual_out == x || residual_out == residual)) ||
      (normalized_out != nullptr && (normalized_out == x || normalized_out == residual));
  if ((rc = pick_shape(V, M, threads_per_row, aliased, &sh)) != CUTIE_OK) return rc;

  FusedArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.ldx = ldx;
  a.res = static_cast<const uint16_t*>(residual);
  a.ldr = ldr;
  a.w = static_cast<const uint16_t*>(weight);
  a.res_out = static_cast<uint16_t*>(residual_out);
  a.ldro = ldro;
  a.norm_out = static_cast<uint16_t*>(normalized_out);
  a.ldn = ldn;
  a.q = static_cast<uint8_t*>(q);
  a.ldq = ldq;
  a.scale = scale;
  a.s_row = s_row;
  a.s_grp = s_grp;
  a.s_grp4 = s_grp4;
  a.M = M;
  a.M_pad = M_pad;
  a.H = (int)H;
  a.V = (int)V;
  a.n_groups = (int)n_groups;
  a.n_groups_pad = (int)n_groups_pad;
  a.eps = eps;
  a.rcp_H = 1.0f / (float)H;
  a.scale_fmt = scale_fmt;
  a.scale_layout = swz ? kLaySwizzled : kLayStrided;
  a.stages = 0;
  a.wait_limit = g_wait_limit;

  const bool res = residual != nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (quant_mode) {
    case CUTIE_QUANT_NONE: e = launch_fused_none(a, sh, res, norm, st); break;
    case CUTIE_QUANT_TOKEN: e = launch_fused_token(a, sh, res, norm, st); break;
    default:
      e = group_size == 32   ? launch_fused_g32(a, sh, res, norm, st)
          : group_size == 64 ? launch_fused_g64(a, sh, res, norm, st)
                             : launch_fused_g128(a, sh, res, norm, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "fused rmsnorm/fp8 launch");
  return CUTIE_OK;
}

}  // namespace
}  // namespace cutie

using namespace cutie;

extern "C" int cutie_rms_norm_fp8(const void* x, int64_t ldx, const void* residual, int64_t ldr,
                                  const void* weight, float eps, int64_t M, int64_t H,
                                  int quant_mode, int group_size, int scale_fmt,
                                  int scale_layout, int64_t ld_scale, void* q, int64_t ldq,
                                  void* scale, void* residual_out, int64_t ldro,
                                  void* normalized_out, int64_t ldn, int threads_per_row,
                                  void* stream) {
  return run_fused(true, x, ldx, residual, ldr, weight, eps, M, H, quant_mode, group_size,
                   scale_fmt, scale_layout, ld_scale, q, ldq, scale, residual_out, ldro,
                   normalized_out, ldn, threads_per_row, stream);
}

extern "C" int cutie_per_token_cast_to_fp8(const void* x, int64_t ldx, int64_t M, int64_t H,
                                           int group_size, int scale_fmt, int scale_layout,
                                           int64_t ld_scale, void* q, int64_t ldq, void* scale,
                                           int threads_per_row, void* stream) {
  const int mode = group_size == 0 ? CUTIE_QUANT_TOKEN : CUTIE_QUANT_GROUP;
  return run_fused(false, x, ldx, nullptr, 0, nullptr, 0.0f, M, H, mode, group_size, scale_fmt,
                   scale_layout, ld_scale, q, ldq, scale, nullptr, 0, nullptr, 0,
                   threads_per_row, stream);
}

extern "C" int cutie_rms_norm(const void* x, int64_t ldx, const void* weight, float eps,
                              int64_t M, int64_t H, int dtype, void* out, int64_t ldo,
                              int threads_per_row, void* stream) {
  if (dtype == CUTIE_DTYPE_BF16) {
    if (out == nullptr) {
      g_err[0] = '\0';
      return fail(CUTIE_ERR_INVALID_ARGUMENT, "out is NULL");
    }
    return run_fused(true, x, ldx, nullptr, 0, weight, eps, M, H, CUTIE_QUANT_NONE, 0,
                     CUTIE_SCALE_FP32, CUTIE_LAYOUT_ROW_MAJOR, 0, nullptr, 0, nullptr, nullptr,
                     0, out, ldo, threads_per_row, stream);
  }
  g_err[0] = '\0';
  if (dtype != CUTIE_DTYPE_F32) return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (M < 0 || H <= 0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "need M >= 0 and H > 0 (got M=%lld, H=%lld)",
                (long long)M, (long long)H);
  if (H % 4 != 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld must be a multiple of 4 (16-byte rows)",
                (long long)H);
  if (H > (int64_t)1 << 30) return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld too large", (long long)H);
  if (!(eps >= 0.0f) || std::isinf(eps))
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
  if (M == 0) return CUTIE_OK;
  int rc;
  if ((rc = check_matrix("x", x, ldx, H, 16, 4)) != CUTIE_OK) return rc;
  if ((rc = check_matrix("out", out, ldo, H, 16, 4)) != CUTIE_OK) return rc;
  if (weight == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "weight is NULL");
  if (!aligned(weight, 16)) return fail(CUTIE_ERR_ALIGNMENT, "weight must be 16-byte aligned");
  F32Shape sh{};
  if ((rc = pick_f32_shape(H / 4, M, threads_per_row, &sh)) != CUTIE_OK) return rc;
  F32Args a{static_cast<const float*>(x), ldx, static_cast<const float*>(weight),
            static_cast<float*>(out), ldo, M, (int)H, (int)(H / 4), eps};
  const cudaError_t e = launch_rmsnorm_f32(a, sh, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp32 rmsnorm launch");
  return CUTIE_OK;
}

extern "C" size_t cutie_rms_norm_backward_workspace(int64_t M, int64_t H) {
  if (M < 0 || H <= 0) return 0;
  int T = 0, grid = 0;
  backward_shape(M, H, &T, &grid);
  return (size_t)grid * (size_t)H * sizeof(float);
}

namespace cutie {
namespace {

// Checks the backward's arguments and fills `a`; returns CUTIE_OK, or the
// status of the first bad argument (the workspace is checked by the caller).
int prepare_backward(const void* d_normalized, int64_t ldd, const void* r, int64_t ldr,
                     const void* weight, const void* d_residual_out, int64_t lddr, float eps,
                     int64_t M, int64_t H, void* dx, int64_t lddx, void* d_weight,
                     int quant_mode, int group_size, int scale_fmt, int scale_layout,
                     int64_t ld_scale, void* q, int64_t ldq, void* scale, BwdArgs* a) {
  if (M < 0 || H <= 0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "need M >= 0 and H > 0 (got M=%lld, H=%lld)",
                (long long)M, (long long)H);
  if (H % 8 != 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "H=%lld must be a multiple of 8 (16-byte rows)",
                (long long)H);
  if (H > 32768)
    return fail(CUTIE_ERR_UNSUPPORTED, "the backward kernel holds rows of up to 32768 (H=%lld)",
                (long long)H);
  if (!(eps >= 0.0f) || std::isinf(eps))
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
  if (quant_mode != CUTIE_QUANT_NONE &&
      !(quant_mode == CUTIE_QUANT_GROUP && group_size == 128))
    return fail(CUTIE_ERR_UNSUPPORTED,
                "the backward quantizes its gradient in 1x128 groups only (quant_mode %d, "
                "group_size %d)",
                quant_mode, group_size);
  if (scale_fmt < CUTIE_SCALE_FP32 || scale_fmt > CUTIE_SCALE_E8M0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown scale_fmt %d", scale_fmt);
  if (scale_layout < CUTIE_LAYOUT_ROW_MAJOR || scale_layout > CUTIE_LAYOUT_COL_MAJOR_PACKED)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "unknown scale_layout %d", scale_layout);
  const bool quant = quant_mode != CUTIE_QUANT_NONE;
  if (quant && scale_layout == CUTIE_LAYOUT_MX_SWIZZLED && scale_fmt != CUTIE_SCALE_E8M0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "the swizzled scale layout needs E8M0 scales");
  const int64_t n_groups = quant ? (H + 127) / 128 : 0;
  const bool swz = quant && scale_layout == CUTIE_LAYOUT_MX_SWIZZLED;
  const int64_t n_groups_pad = swz ? (n_groups + 3) / 4 * 4 : n_groups;
  const int64_t M_pad = swz ? (M + 127) / 128 * 128 : M;

  int rc;
  if (M > 0) {
    if ((rc = check_matrix("d_normalized", d_normalized, ldd, H, 16, 8)) != CUTIE_OK) return rc;
    if ((rc = check_matrix("r", r, ldr, H, 16, 8)) != CUTIE_OK) return rc;
    if ((rc = check_matrix("dx", dx, lddx, H, 16, 8)) != CUTIE_OK) return rc;
    if (d_residual_out != nullptr &&
        (rc = check_matrix("d_residual_out", d_residual_out, lddr, H, 16, 8)) != CUTIE_OK)
      return rc;
  }
  if (weight == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "weight is NULL");
  if (!aligned(weight, 16)) return fail(CUTIE_ERR_ALIGNMENT, "weight must be 16-byte aligned");
  if (d_weight != nullptr && !aligned(d_weight, 2))
    return fail(CUTIE_ERR_ALIGNMENT, "d_weight must be 2-byte aligned");
  int64_t s_row = 0, s_grp = 0, s_grp4 = 0;
  if (quant && M > 0) {
    if ((rc = check_matrix("q", q, ldq, H, 8, 8)) != CUTIE_OK) return rc;
    if (scale == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "scale is NULL");
    if (scale_fmt != CUTIE_SCALE_E8M0 && !aligned(scale, 4))
      return fail(CUTIE_ERR_ALIGNMENT, "fp32 scales must be 4-byte aligned");
  }
  if (quant) {
    if ((rc = strided_scale(scale_layout, scale_fmt, ld_scale, M, n_groups, &s_row, &s_grp,
                            &s_grp4)) != CUTIE_OK)
      return rc;
  }
  *a = BwdArgs{};
  a->dn = static_cast<const uint16_t*>(d_normalized);
  a->lddn = ldd;
  a->r = static_cast<const uint16_t*>(r);
  a->ldr = ldr;
  a->w = static_cast<const uint16_t*>(weight);
  a->dro = static_cast<const uint16_t*>(d_residual_out);
  a->lddro = lddr;
  a->dx = static_cast<uint16_t*>(dx);
  a->lddx = lddx;
  FusedArgs& qa = a->qa;
  qa.q = quant ? static_cast<uint8_t*>(q) : nullptr;
  qa.ldq = ldq;
  qa.scale = scale;
  qa.s_row = s_row;
  qa.s_grp = s_grp;
  qa.s_grp4 = s_grp4;
  qa.M = M;
  qa.M_pad = M_pad;
  qa.H = (int)H;
  qa.V = (int)(H / 8);
  qa.n_groups = (int)n_groups;
  qa.n_groups_pad = (int)n_groups_pad;
  qa.scale_fmt = scale_fmt;
  qa.scale_layout = swz ? kLaySwizzled : kLayStrided;
  qa.wait_limit = g_wait_limit;
  return CUTIE_OK;
}

}  // namespace
}  // namespace cutie

extern "C" int cutie_rms_norm_backward(const void* d_normalized, int64_t ldd, const void* r,
                                       int64_t ldr, const void* weight,
                                       const void* d_residual_out, int64_t lddr, float eps,
                                       int64_t M, int64_t H, void* dx, int64_t lddx,
                                       void* d_weight, void* workspace, size_t workspace_bytes,
                                       int quant_mode, int group_size, int scale_fmt,
                                       int scale_layout, int64_t ld_scale, void* q, int64_t ldq,
                                       void* scale, void* stream) {
  g_err[0] = '\0';
  BwdArgs a{};
  int rc = prepare_backward(d_normalized, ldd, r, ldr, weight, d_residual_out, lddr, eps, M, H,
                            dx, lddx, d_weight, quant_mode, group_size, scale_fmt, scale_layout,
                            ld_scale, q, ldq, scale, &a);
  if (rc != CUTIE_OK) return rc;
  const bool want_dw = d_weight != nullptr;
  if (a.qa.M_pad == 0 && !want_dw) return CUTIE_OK;
  if (want_dw) {
    const size_t need = cutie_rms_norm_backward_workspace(M, H);
    if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))
      return fail(CUTIE_ERR_INVALID_ARGUMENT,
                  "d_weight needs a 16-byte aligned workspace of %zu bytes (got %zu at %p)", need,
                  workspace_bytes, workspace);
    a.partial = static_cast<float*>(workspace);
  }
  const cudaError_t e = launch_backward(a, eps, want_dw, static_cast<uint16_t*>(d_weight), 0,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm backward launch");
  return CUTIE_OK;
}

extern "C" int cutie_rms_norm_backward_noalloc(const void* d_normalized, int64_t ldd,
                                               const void* r, int64_t ldr, const void* weight,
                                               const void* d_residual_out, int64_t lddr,
                                               float eps, int64_t M, int64_t H, void* dx,
                                               int64_t lddx, void* d_weight, int quant_mode,
                                               int group_size, int scale_fmt, int scale_layout,
                                               int64_t ld_scale, void* q, int64_t ldq,
                                               void* scale, void* stream) {
  g_err[0] = '\0';
  BwdArgs a{};
  int rc = prepare_backward(d_normalized, ldd, r, ldr, weight, d_residual_out, lddr, eps, M, H,
                            dx, lddx, d_weight, quant_mode, group_size, scale_fmt, scale_layout,
                            ld_scale, q, ldq, scale, &a);
  if (rc != CUTIE_OK) return rc;
  const bool want_dw = d_weight != nullptr;
  if (a.qa.M_pad == 0 && !want_dw) return CUTIE_OK;
  int max_grid = 0;
  if (want_dw) {
    // each CTA writes one row of H partial sums into the scratch
    if (H > kNoAllocScratchFloats)
      return fail(CUTIE_ERR_UNSUPPORTED,
                  "H=%lld exceeds the %lld-float device scratch of the allocation-free backward",
                  (long long)H, (long long)kNoAllocScratchFloats);
    float* scratch = nullptr;
    const cudaError_t e = noalloc_scratch(&scratch);
    if (e != cudaSuccess) return cuda_fail(e, "resolving the backward's device scratch");
    a.partial = scratch;
    max_grid = (int)(kNoAllocScratchFloats / H);
  }
  const cudaError_t e = launch_backward(a, eps, want_dw, static_cast<uint16_t*>(d_weight),
                                        max_grid, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm backward launch");
  return CUTIE_OK;
}

extern "C" int cutie_gemm_mxfp8(const void* a, int64_t lda, const void* a_scale, const void* b,
                                int64_t ldb, const void* b_scale, void* d, int64_t ldd,
                                int64_t M, int64_t N, int64_t K, void* stream) {
  g_err[0] = '\0';
  if (M < 0 || N <= 0 || K <= 0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "need M >= 0, N > 0 and K > 0 (got %lld, %lld, %lld)",
                (long long)M, (long long)N, (long long)K);
  if (N % 128 != 0 || K % 128 != 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "N and K must be multiples of 128 (got N=%lld, K=%lld)",
                (long long)N, (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(CUTIE_ERR_UNSUPPORTED, "M, N and K must be below 2^31");
  if (M == 0) return CUTIE_OK;
  int rc;
  if ((rc = check_matrix("a", a, lda, K, 16, 16)) != CUTIE_OK) return rc;
  if ((rc = check_matrix("b", b, ldb, K, 16, 16)) != CUTIE_OK) return rc;
  if ((rc = check_matrix("d", d, ldd, N, 16, 8)) != CUTIE_OK) return rc;
  if (a_scale == nullptr || b_scale == nullptr)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "a_scale and b_scale must not be NULL");
  if (!aligned(a_scale, 16) || !aligned(b_scale, 16))
    return fail(CUTIE_ERR_ALIGNMENT, "the swizzled scale buffers must be 16-byte aligned");
  const char* why = "";
  rc = gemm_mxfp8(a, lda, a_scale, b, ldb, b_scale, d, ldd, M, N, K,
                  static_cast<cudaStream_t>(stream), &why);
  if (rc != CUTIE_OK) return fail(rc, "mxfp8 gemm: %s", why);
  return CUTIE_OK;
}

extern "C" int cutie_rms_norm_mxfp8_gemm(const void* x, int64_t ldx, const void* weight,
                                         float eps, const void* b, int64_t ldb,
                                         const void* b_scale, void* d, int64_t ldd, int64_t M,
                                         int64_t N, int64_t K, void* q, int64_t ldq,
                                         void* q_scale, void* stream) {
  g_err[0] = '\0';
  if (M < 0 || N <= 0 || K <= 0)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "need M >= 0, N > 0 and K > 0 (got %lld, %lld, %lld)",
                (long long)M, (long long)N, (long long)K);
  if (N % 128 != 0 || K % 128 != 0)
    return fail(CUTIE_ERR_UNSUPPORTED, "N and K must be multiples of 128 (got N=%lld, K=%lld)",
                (long long)N, (long long)K);
  if (K > 65536)
    return fail(CUTIE_ERR_UNSUPPORTED, "K must be at most 65536 (got %lld)", (long long)K);
  if (M > INT32_MAX || N > INT32_MAX)
    return fail(CUTIE_ERR_UNSUPPORTED, "M and N must be below 2^31");
  if (!std::isfinite(eps) || eps < 0.0f)
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
  if ((q == nullptr) != (q_scale == nullptr))
    return fail(CUTIE_ERR_INVALID_ARGUMENT, "q and q_scale must be given together");
  if (M == 0) return CUTIE_OK;
  int rc;
  if ((rc = check_matrix("x", x, ldx, K, 16, 8)) != CUTIE_OK) return rc;
  if (weight == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "weight is NULL");
  if (!aligned(weight, 16)) return fail(CUTIE_ERR_ALIGNMENT, "weight must be 16-byte aligned");
  if ((rc = check_matrix("b", b, ldb, K, 16, 16)) != CUTIE_OK) return rc;
  if ((rc = check_matrix("d", d, ldd, N, 16, 8)) != CUTIE_OK) return rc;
  if (b_scale == nullptr) return fail(CUTIE_ERR_INVALID_ARGUMENT, "b_scale is NULL");
  if (!aligned(b_scale, 16))
    return fail(CUTIE_ERR_ALIGNMENT, "the swizzled scale buffers must be 16-byte aligned");
  if (q != nullptr) {
    if ((rc = check_matrix("q", q, ldq, K, 16, 16)) != CUTIE_OK) return rc;
    if (!aligned(q_scale, 16))
      return fail(CUTIE_ERR_ALIGNMENT, "the swizzled scale buffers must be 16-byte aligned");
  }
  const char* why = "";
  rc = gemm_rmsnorm_mxfp8(x, ldx, weight, eps, b, ldb, b_scale, d, ldd, M, N, K, q, ldq, q_scale,
                          g_wait_limit, static_cast<cudaStream_t>(stream), &why);
  if (rc != CUTIE_OK) return fail(rc, "rms_norm mxfp8 gemm: %s", why);
  return CUTIE_OK;
}

extern "C" int cutie_device_error(int clear) {
  g_err[0] = '\0';
  int any = 0;
  cudaError_t (*readers[])(int*, bool) = {device_error_none, device_error_token, device_error_g32,
                                          device_error_g64, device_error_g128,
                                          device_error_bwd,  device_error_gemm,
                                          device_error_prologue};
  for (auto read : readers) {
    int v = 0;
    const cudaError_t e = read(&v, clear != 0);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    if (any == 0) any = v;
  }
  return any;
}

extern "C" int64_t cutie_set_wait_limit(int64_t cycles) {
  const long long prev = g_wait_limit;
  g_wait_limit = cycles == 0 ? kWaitLimitCycles : (long long)cycles;
  return prev;
}

extern "C" const char* cutie_last_error(void) { return g_err; }

extern "C" int cutie_abi_version(void) { return CUTIE_ABI_VERSION; }
