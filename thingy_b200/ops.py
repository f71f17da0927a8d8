"""Tensor-level launchers over the C ABI (include/cutie.h).

These are the destination-passing primitives every public entry point uses:
the caller passes preallocated CUDA tensors, the work is enqueued on the
current torch stream of the tensors' device (or on ``stream``), nothing is
synchronised. Argument errors raise ValueError, CUDA failures RuntimeError.

Calls go through the compiled torch binding (thingy_b200/_C, built next to
the library) when it is present: it reads tensor metadata and the current
stream in C++ and costs a few microseconds. Without it, or for a raw stream
handle, the same C ABI is called through ctypes with the checks done here.
"""

from __future__ import annotations

import torch

from . import _lib

_UNSET = object()
_binding_mod = _UNSET


def _binding():
    """The torch binding, imported on first use (None if it was not built).

    Importing it maps libcutie_b200.so too, so it is deferred until an op
    runs: importing the package (or a pure-Python submodule such as
    ``workloads``) loads no native code."""
    global _binding_mod
    if _binding_mod is _UNSET:
        try:
            from . import _C as mod
        except ImportError:  # the ctypes path below covers the same entry points
            mod = None
        _binding_mod = mod
    return _binding_mod
from .layouts import SCALE_FORMATS, SCALE_LAYOUTS, mx_swizzled_size, n_groups

_FMT_CODE = {"fp32": _lib.SCALE_FP32, "ue8m0": _lib.SCALE_FP32_POW2, "e8m0": _lib.SCALE_E8M0}
_LAYOUT_CODE = {"row": _lib.LAYOUT_ROW_MAJOR, "col": _lib.LAYOUT_COL_MAJOR,
                "mx": _lib.LAYOUT_MX_SWIZZLED, "packed": _lib.LAYOUT_COL_MAJOR_PACKED}

E8M0_DTYPES = tuple(
    d for d in (getattr(torch, "float8_e8m0fnu", None), torch.uint8) if d is not None
)
FP8_DTYPE = torch.float8_e4m3fn


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device, stream) -> int:
    if stream is None:
        return torch.cuda.current_stream(device).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)  # a raw cudaStream_t / CUstream handle


def _rows(name: str, t: torch.Tensor, M: int, H: int, dtype: torch.dtype, device) -> int:
    """Validate a row-major [M, H] matrix view; return its leading dimension."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dim() != 2 or tuple(t.shape) != (M, H):
        raise ValueError(f"{name} must have shape ({M}, {H}), got {tuple(t.shape)}")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if H > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must be contiguous along its last dimension")
    return max(t.stride(0), H) if M > 0 else H


def _check_x(x: torch.Tensor, dtype=torch.bfloat16) -> tuple[int, int]:
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, H], got {x.dim()}-D")
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor (this library has no CPU path)")
    if x.dtype != dtype:
        raise ValueError(f"x must be {dtype}, got {x.dtype}")
    return x.shape[0], x.shape[1]


def _packed_scale_ld(scale: torch.Tensor, M: int, G: int, fmt: str, device) -> int:
    """ld_scale (in int32 words) of a packed UE8M0 scale tensor."""
    if fmt != "e8m0":
        raise ValueError("the packed scale layout needs e8m0 scales")
    if scale.dtype != torch.int32:
        raise ValueError(f"packed e8m0 scales must be int32 words, got {scale.dtype}")
    if scale.device != device:
        raise ValueError(f"scale is on {scale.device}, expected {device}")
    W = (G + 3) // 4
    if scale.dim() == 1 and W == 1:
        if scale.shape[0] != M or (M > 1 and scale.stride(0) != 1):
            raise ValueError(f"packed per-row scales must be a contiguous [{M}] tensor")
        return M
    if scale.dim() == 2:
        shape = tuple(scale.shape)
        if shape == (M, W) and (M <= 1 or scale.stride(0) == 1):
            return max(scale.stride(1), M) if W > 1 else M
        if shape == (W, M) and (M <= 1 or scale.stride(1) == 1):
            return max(scale.stride(0), M) if W > 1 else M
    raise ValueError(
        f"packed scales must be an int32 [{M}, {W}] tensor contiguous along M (or its transpose)"
    )


def _scale_args(scale: torch.Tensor, M: int, H: int, group_size: int | None, fmt: str,
                layout: str, device) -> int:
    """Validate the scale tensor for (fmt, layout); return ld_scale."""
    G = n_groups(H, group_size)
    if layout == "packed":
        return _packed_scale_ld(scale, M, G, fmt, device)
    if fmt == "e8m0":
        if scale.dtype not in E8M0_DTYPES:
            raise ValueError(f"e8m0 scales must be uint8 or float8_e8m0fnu, got {scale.dtype}")
    elif scale.dtype != torch.float32:
        raise ValueError(f"{fmt} scales must be float32, got {scale.dtype}")
    if scale.device != device:
        raise ValueError(f"scale is on {scale.device}, expected {device}")
    if layout == "mx":
        if not scale.is_contiguous() or scale.numel() < mx_swizzled_size(M, G):
            raise ValueError(
                f"swizzled scales need a contiguous buffer of {mx_swizzled_size(M, G)} bytes"
            )
        return 0
    if scale.dim() == 1 and G == 1:
        if scale.shape[0] != M or (M > 1 and scale.stride(0) != 1):
            raise ValueError(f"per-token scale must be a contiguous [{M}] tensor")
        return M if layout == "col" else 1
    if scale.dim() != 2:
        raise ValueError("scale must be 2-D")
    shape = tuple(scale.shape)
    if layout == "row":
        if shape != (M, G):
            raise ValueError(f"row-major scale must have shape ({M}, {G}), got {shape}")
        if G > 1 and scale.stride(1) != 1:
            raise ValueError("row-major scale must be contiguous along groups")
        return max(scale.stride(0), G) if M > 1 else G
    # column-major: a [G, M] tensor, or its transposed [M, G] view
    if shape == (G, M) and (M <= 1 or scale.stride(1) == 1):
        return max(scale.stride(0), M) if G > 1 else M
    if shape == (M, G) and (M <= 1 or scale.stride(0) == 1):
        return max(scale.stride(1), M) if G > 1 else M
    raise ValueError(
        f"column-major scale must be a [{G}, {M}] tensor contiguous along M (or its transpose)"
    )


def launch_rms_norm_fp8(
    x: torch.Tensor,
    weight: torch.Tensor | None,
    eps: float,
    *,
    residual: torch.Tensor | None = None,
    q: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    normalized_out: torch.Tensor | None = None,
    group_size: int | None = 128,
    scale_format: str = "fp32",
    scale_layout: str = "row",
    threads_per_row: int = 0,
    normalize: bool = True,
    stream=None,
) -> None:
    """Enqueue one fused [residual add] -> RMSNorm -> [FP8 quant] launch.

    ``q`` and ``scale`` both None means no quantization. ``group_size`` None
    (or 0) means one scale per row. ``normalize=False`` quantizes ``x`` as is.
    """
    if scale_format not in SCALE_FORMATS:
        raise ValueError(f"scale_format must be one of {SCALE_FORMATS}")
    if scale_layout not in SCALE_LAYOUTS:
        raise ValueError(f"scale_layout must be one of {SCALE_LAYOUTS}")
    binding = _binding() if not isinstance(stream, int) else None
    if binding is not None:
        if not isinstance(x, torch.Tensor):
            raise TypeError("x must be a torch.Tensor")
        args = (x, weight, float(eps), residual, q, scale, residual_out, normalized_out,
                int(group_size or 0), _FMT_CODE[scale_format], _LAYOUT_CODE[scale_layout],
                int(threads_per_row), bool(normalize))
        if stream is None:
            binding.rms_norm_fp8(*args)
        else:
            with torch.cuda.stream(stream):
                binding.rms_norm_fp8(*args)
        return
    M, H = _check_x(x)
    device = x.device
    ldx = _rows("x", x, M, H, torch.bfloat16, device)
    ldr = _rows("residual", residual, M, H, torch.bfloat16, device) if residual is not None else 0
    ldro = (
        _rows("residual_out", residual_out, M, H, torch.bfloat16, device)
        if residual_out is not None
        else 0
    )
    ldn = (
        _rows("normalized_out", normalized_out, M, H, torch.bfloat16, device)
        if normalized_out is not None
        else 0
    )
    if normalize:
        if weight is None:
            raise ValueError("weight is required")
        if weight.shape != (H,) or weight.dtype != torch.bfloat16 or weight.device != device:
            raise ValueError(f"weight must be a bf16 [{H}] tensor on {device}")
        if not weight.is_contiguous():
            raise ValueError("weight must be contiguous")
    quant = q is not None or scale is not None
    if quant:
        if q is None or scale is None:
            raise ValueError("q and scale must be given together")
        if q.dtype not in (FP8_DTYPE, torch.uint8):
            raise ValueError(f"q must be float8_e4m3fn, got {q.dtype}")
        ldq = _rows("q", q, M, H, q.dtype, device)
        ld_scale = _scale_args(scale, M, H, group_size, scale_format, scale_layout, device)
        mode = _lib.QUANT_GROUP if group_size else _lib.QUANT_TOKEN
    else:
        ldq, ld_scale, mode = 0, 0, _lib.QUANT_NONE
    lib = _lib.load()
    with torch.cuda.device(device):
        handle = _stream_handle(device, stream)
        if normalize:
            status = lib.cutie_rms_norm_fp8(
                _ptr(x), ldx, _ptr(residual), ldr, _ptr(weight), float(eps), M, H,
                mode, int(group_size or 0), _FMT_CODE[scale_format],
                _LAYOUT_CODE[scale_layout], ld_scale, _ptr(q), ldq, _ptr(scale),
                _ptr(residual_out), ldro, _ptr(normalized_out), ldn,
                int(threads_per_row), handle,
            )
        else:
            if not quant:
                raise ValueError("quantization-only call needs q and scale")
            status = lib.cutie_per_token_cast_to_fp8(
                _ptr(x), ldx, M, H, int(group_size or 0), _FMT_CODE[scale_format],
                _LAYOUT_CODE[scale_layout], ld_scale, _ptr(q), ldq, _ptr(scale),
                int(threads_per_row), handle,
            )
    _lib.check(status)


def launch_rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    out: torch.Tensor,
    *,
    threads_per_row: int = 0,
    stream=None,
) -> None:
    """Enqueue a standalone RMSNorm (bf16 or fp32, see include/cutie.h)."""
    binding = _binding() if not isinstance(stream, int) else None
    if binding is not None:
        if stream is None:
            binding.rms_norm(x, weight, float(eps), out, int(threads_per_row))
        else:
            with torch.cuda.stream(stream):
                binding.rms_norm(x, weight, float(eps), out, int(threads_per_row))
        return
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"x must be bfloat16 or float32, got {x.dtype}")
    M, H = _check_x(x, x.dtype)
    device = x.device
    ldx = _rows("x", x, M, H, x.dtype, device)
    ldo = _rows("out", out, M, H, x.dtype, device)
    if weight.shape != (H,) or weight.dtype != x.dtype or weight.device != device:
        raise ValueError(f"weight must be a {x.dtype} [{H}] tensor on {device}")
    if not weight.is_contiguous():
        raise ValueError("weight must be contiguous")
    code = _lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_F32
    lib = _lib.load()
    with torch.cuda.device(device):
        status = lib.cutie_rms_norm(
            _ptr(x), ldx, _ptr(weight), float(eps), M, H, code, _ptr(out), ldo,
            int(threads_per_row), _stream_handle(device, stream),
        )
    _lib.check(status)


def backward_workspace_bytes(M: int, H: int, device=None) -> int:
    """Bytes of fp32 workspace the backward needs for the weight gradient on ``device``."""
    lib = _lib.load()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        return int(lib.cutie_rms_norm_backward_workspace(int(M), int(H)))


def launch_rms_norm_backward(
    d_normalized: torch.Tensor,
    r: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    dx: torch.Tensor,
    d_residual_out: torch.Tensor | None = None,
    d_weight: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    q: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    scale_format: str = "fp32",
    scale_layout: str = "row",
    stream=None,
) -> None:
    """Enqueue the backward of [residual add] -> RMSNorm (cutie_rms_norm_backward).

    d_normalized: bf16 [M, H] gradient of the normalized output; r: the
    forward's RMSNorm input (x + residual, i.e. residual_out, or x);
    d_residual_out: gradient of residual_out, or None. Writes dx (the
    gradient of x and of residual), d_weight (bf16 [H], needs ``workspace``,
    a CUDA tensor of at least backward_workspace_bytes(M, H) bytes) and, with
    q and scale, the 1x128 FP8 quantization of dx.
    """
    if scale_format not in SCALE_FORMATS:
        raise ValueError(f"scale_format must be one of {SCALE_FORMATS}")
    if scale_layout not in SCALE_LAYOUTS:
        raise ValueError(f"scale_layout must be one of {SCALE_LAYOUTS}")
    M, H = _check_x(d_normalized)
    device = d_normalized.device
    ldd = _rows("d_normalized", d_normalized, M, H, torch.bfloat16, device)
    ldr = _rows("r", r, M, H, torch.bfloat16, device)
    lddx = _rows("dx", dx, M, H, torch.bfloat16, device)
    lddr = (_rows("d_residual_out", d_residual_out, M, H, torch.bfloat16, device)
            if d_residual_out is not None else 0)
    if weight.shape != (H,) or weight.dtype != torch.bfloat16 or weight.device != device:
        raise ValueError(f"weight must be a bf16 [{H}] tensor on {device}")
    if not weight.is_contiguous():
        raise ValueError("weight must be contiguous")
    ws_bytes = 0
    if d_weight is not None:
        if d_weight.shape != (H,) or d_weight.dtype != torch.bfloat16 or d_weight.device != device:
            raise ValueError(f"d_weight must be a bf16 [{H}] tensor on {device}")
        if not d_weight.is_contiguous():
            raise ValueError("d_weight must be contiguous")
        if workspace is None or workspace.device != device or not workspace.is_contiguous():
            raise ValueError("d_weight needs a contiguous CUDA workspace tensor")
        ws_bytes = workspace.numel() * workspace.element_size()
    quant = q is not None or scale is not None
    if quant:
        if q is None or scale is None:
            raise ValueError("q and scale must be given together")
        if q.dtype not in (FP8_DTYPE, torch.uint8):
            raise ValueError(f"q must be float8_e4m3fn, got {q.dtype}")
        ldq = _rows("q", q, M, H, q.dtype, device)
        ld_scale = _scale_args(scale, M, H, 128, scale_format, scale_layout, device)
        mode = _lib.QUANT_GROUP
    else:
        ldq, ld_scale, mode = 0, 0, _lib.QUANT_NONE
    lib = _lib.load()
    with torch.cuda.device(device):
        status = lib.cutie_rms_norm_backward(
            _ptr(d_normalized), ldd, _ptr(r), ldr, _ptr(weight), _ptr(d_residual_out), lddr,
            float(eps), M, H, _ptr(dx), lddx, _ptr(d_weight), _ptr(workspace), ws_bytes,
            mode, 128, _FMT_CODE[scale_format], _LAYOUT_CODE[scale_layout], ld_scale,
            _ptr(q), ldq, _ptr(scale), _stream_handle(device, stream),
        )
    _lib.check(status)
