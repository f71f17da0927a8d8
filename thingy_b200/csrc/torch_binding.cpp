// Thin torch binding over the C ABI in include/cutie.h (no kernels here).
//
// Python could call the C ABI through ctypes, but marshalling 22 arguments and
// checking tensors from Python costs ~15 us a call, several times the kernel
// at decode sizes. This module takes at::Tensor arguments, derives pointers,
// leading dimensions and the current CUDA stream in C++, and calls the same
// extern "C" entry points. Argument errors raise ValueError, CUDA failures
// RuntimeError (the status codes of cutie.h).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>

#include "cutie.h"

namespace {

void check_status(int status) {
  if (status == CUTIE_OK) return;
  const std::string msg = cutie_last_error();
  if (status == CUTIE_ERR_CUDA) throw std::runtime_error(msg);
  throw std::invalid_argument(msg);
}

[[noreturn]] void bad(const std::string& msg) { throw std::invalid_argument(msg); }

// Leading dimension of a row-major [M, H] view (contiguous along H).
int64_t rows_ld(const at::Tensor& t, const char* name, int64_t M, int64_t H,
                at::ScalarType dtype, const at::Device& dev) {
  if (t.dim() != 2 || t.size(0) != M || t.size(1) != H)
    bad(std::string(name) + " must have shape (" + std::to_string(M) + ", " + std::to_string(H) +
        ")");
  if (t.scalar_type() != dtype) bad(std::string(name) + " has the wrong dtype");
  if (t.device() != dev) bad(std::string(name) + " is on the wrong device");
  if (H > 1 && t.stride(1) != 1) bad(std::string(name) + " must be contiguous along its last dimension");
  return M > 0 ? std::max<int64_t>(t.stride(0), H) : H;
}

const void* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr() : nullptr;
}

// ld_scale for (layout, groups) from the scale tensor's shape and strides;
// mirrors thingy_b200.ops._scale_args.
int64_t scale_ld(const at::Tensor& s, int64_t M, int64_t G, int64_t layout) {
  if (layout == CUTIE_LAYOUT_COL_MAJOR_PACKED) {  // int32 words, four groups a word
    const int64_t W = (G + 3) / 4;
    if (s.dim() == 1 && W == 1) {
      if (s.size(0) != M || (M > 1 && s.stride(0) != 1)) bad("packed per-row scales must be a contiguous [M] tensor");
      return M;
    }
    if (s.dim() != 2) bad("packed scales must be 2-D");
    const int64_t a = s.size(0), b = s.size(1);
    if (a == M && b == W && (M <= 1 || s.stride(0) == 1)) return W > 1 ? std::max<int64_t>(s.stride(1), M) : M;
    if (a == W && b == M && (M <= 1 || s.stride(1) == 1)) return W > 1 ? std::max<int64_t>(s.stride(0), M) : M;
    bad("packed scales must be an int32 [M, ceil(n_groups/4)] tensor contiguous along M (or its transpose)");
  }
  if (layout == CUTIE_LAYOUT_MX_SWIZZLED) {
    if (!s.is_contiguous()) bad("swizzled scales need a contiguous buffer");
    const int64_t need = (M + 127) / 128 * 128 * ((G + 3) / 4 * 4);
    if (s.numel() < need) bad("swizzled scale buffer too small");
    return 0;
  }
  if (s.dim() == 1 && G == 1) {
    if (s.size(0) != M || (M > 1 && s.stride(0) != 1)) bad("per-token scale must be a contiguous [M] tensor");
    return layout == CUTIE_LAYOUT_COL_MAJOR ? M : 1;
  }
  if (s.dim() != 2) bad("scale must be 2-D");
  const int64_t a = s.size(0), b = s.size(1);
  if (layout == CUTIE_LAYOUT_ROW_MAJOR) {
    if (a != M || b != G) bad("row-major scale must have shape (M, n_groups)");
    if (G > 1 && s.stride(1) != 1) bad("row-major scale must be contiguous along groups");
    return M > 1 ? std::max<int64_t>(s.stride(0), G) : G;
  }
  if (a == G && b == M && (M <= 1 || s.stride(1) == 1)) return G > 1 ? std::max<int64_t>(s.stride(0), M) : M;
  if (a == M && b == G && (M <= 1 || s.stride(0) == 1)) return G > 1 ? std::max<int64_t>(s.stride(1), M) : M;
  bad("column-major scale must be a [n_groups, M] tensor contiguous along M (or its transpose)");
}

// Fused [residual add] -> RMSNorm -> [FP8 quantization]; normalize=false is
// the quantizer alone. q / scale absent: no quantization.
void rms_norm_fp8(const at::Tensor& x, const c10::optional<at::Tensor>& weight, double eps,
                  const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& q,
                  const c10::optional<at::Tensor>& scale,
                  const c10::optional<at::Tensor>& residual_out,
                  const c10::optional<at::Tensor>& normalized_out, int64_t group_size,
                  int64_t scale_fmt, int64_t scale_layout, int64_t threads_per_row,
                  bool normalize) {
  if (x.dim() != 2) bad("x must be 2-D [M, H]");
  if (!x.is_cuda()) bad("x must be a CUDA tensor (this library has no CPU path)");
  if (x.scalar_type() != at::kBFloat16) bad("x must be bfloat16");
  const int64_t M = x.size(0), H = x.size(1);
  const at::Device dev = x.device();
  const int64_t ldx = rows_ld(x, "x", M, H, at::kBFloat16, dev);
  const int64_t ldr = residual ? rows_ld(*residual, "residual", M, H, at::kBFloat16, dev) : 0;
  const int64_t ldro =
      residual_out ? rows_ld(*residual_out, "residual_out", M, H, at::kBFloat16, dev) : 0;
  const int64_t ldn =
      normalized_out ? rows_ld(*normalized_out, "normalized_out", M, H, at::kBFloat16, dev) : 0;
  if (normalize) {
    if (!weight) bad("weight is required");
    if (weight->dim() != 1 || weight->size(0) != H || weight->scalar_type() != at::kBFloat16 ||
        weight->device() != dev || !weight->is_contiguous())
      bad("weight must be a contiguous bf16 [H] tensor on x's device");
  }
  const bool quant = q.has_value() || scale.has_value();
  int64_t ldq = 0, lds = 0;
  int mode = CUTIE_QUANT_NONE;
  if (quant) {
    if (!q || !scale) bad("q and scale must be given together");
    if (q->scalar_type() != at::kFloat8_e4m3fn && q->scalar_type() != at::kByte)
      bad("q must be float8_e4m3fn");
    ldq = rows_ld(*q, "q", M, H, q->scalar_type(), dev);
    const int64_t G = group_size > 0 ? (H + group_size - 1) / group_size : 1;
    if (scale_layout == CUTIE_LAYOUT_COL_MAJOR_PACKED) {
      if (scale->scalar_type() != at::kInt) bad("packed e8m0 scales must be int32 words");
    } else if (scale_fmt == CUTIE_SCALE_E8M0) {
      if (scale->element_size() != 1) bad("e8m0 scales must be 1-byte elements");
    } else if (scale->scalar_type() != at::kFloat) {
      bad("fp32 / pow2 scales must be float32");
    }
    if (scale->device() != dev) bad("scale is on the wrong device");
    lds = scale_ld(*scale, M, G, scale_layout);
    mode = group_size > 0 ? CUTIE_QUANT_GROUP : CUTIE_QUANT_TOKEN;
  }
  const c10::cuda::CUDAGuard guard(dev);
  void* stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  int status;
  if (normalize) {
    status = cutie_rms_norm_fp8(
        x.data_ptr(), ldx, ptr_or_null(residual), ldr, weight->data_ptr(), (float)eps, M, H, mode,
        (int)group_size, (int)scale_fmt, (int)scale_layout, lds,
        quant ? q->data_ptr() : nullptr, ldq, quant ? scale->data_ptr() : nullptr,
        const_cast<void*>(ptr_or_null(residual_out)), ldro,
        const_cast<void*>(ptr_or_null(normalized_out)), ldn, (int)threads_per_row, stream);
  } else {
    if (!quant) bad("quantization-only call needs q and scale");
    status = cutie_per_token_cast_to_fp8(x.data_ptr(), ldx, M, H, (int)group_size, (int)scale_fmt,
                                         (int)scale_layout, lds, q->data_ptr(), ldq,
                                         scale->data_ptr(), (int)threads_per_row, stream);
  }
  check_status(status);
}

void rms_norm(const at::Tensor& x, const at::Tensor& weight, double eps, const at::Tensor& out,
              int64_t threads_per_row) {
  if (x.dim() != 2) bad("x must be 2-D [M, H]");
  if (!x.is_cuda()) bad("x must be a CUDA tensor (this library has no CPU path)");
  const auto dt = x.scalar_type();
  if (dt != at::kBFloat16 && dt != at::kFloat) bad("x must be bfloat16 or float32");
  const int64_t M = x.size(0), H = x.size(1);
  const at::Device dev = x.device();
  const int64_t ldx = rows_ld(x, "x", M, H, dt, dev);
  const int64_t ldo = rows_ld(out, "out", M, H, dt, dev);
  if (weight.dim() != 1 || weight.size(0) != H || weight.scalar_type() != dt ||
      weight.device() != dev || !weight.is_contiguous())
    bad("weight must be a contiguous [H] tensor of x's dtype on x's device");
  const c10::cuda::CUDAGuard guard(dev);
  void* stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  check_status(cutie_rms_norm(x.data_ptr(), ldx, weight.data_ptr(), (float)eps, M, H,
                              dt == at::kBFloat16 ? CUTIE_DTYPE_BF16 : CUTIE_DTYPE_F32,
                              out.data_ptr(), ldo, (int)threads_per_row, stream));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch binding of the cutie C ABI (thingy_b200)";
  m.def("rms_norm_fp8", &rms_norm_fp8, py::arg("x"), py::arg("weight"), py::arg("eps"),
        py::arg("residual"), py::arg("q"), py::arg("scale"), py::arg("residual_out"),
        py::arg("normalized_out"), py::arg("group_size"), py::arg("scale_fmt"),
        py::arg("scale_layout"), py::arg("threads_per_row"), py::arg("normalize"));
  m.def("rms_norm", &rms_norm, py::arg("x"), py::arg("weight"), py::arg("eps"), py::arg("out"),
        py::arg("threads_per_row"));
  m.def("abi_version", []() { return cutie_abi_version(); });
}
