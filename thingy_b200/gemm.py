"""The downstream consumer of the path's MXFP8 output: a block-scaled FP8 GEMM,
and the same GEMM with RMSNorm + MXFP8 quantization fused in as its prologue.

``mxfp8_gemm(a, a_scale, b, b_scale)`` multiplies e4m3 codes with 1x32 e8m0
scales in the Blackwell swizzled layout (what ``rms_norm_fp8(...,
group_size=32, scale_format="e8m0", scale_layout="mx")`` returns) by a weight
quantized the same way, on the tensor cores (``cutie_gemm_mxfp8``,
hand-written tcgen05 kernel), fp32 accumulation, bf16 out:
``D = dequant(a) @ dequant(b).T``. The reference has no GEMM on this path
(src/cutie/rms_norm/bench.py stops before it); this is the consumer its
quantizer feeds.
"""

from __future__ import annotations

import torch

from . import _lib
from .layouts import mx_swizzled_size
from .ops import E8M0_DTYPES, FP8_DTYPE


def _operand(name: str, t: torch.Tensor, K: int) -> int:
    if not isinstance(t, torch.Tensor) or t.dim() != 2 or not t.is_cuda:
        raise ValueError(f"{name} must be a 2-D CUDA tensor")
    if t.dtype not in (FP8_DTYPE, torch.uint8):
        raise ValueError(f"{name} must be float8_e4m3fn, got {t.dtype}")
    if t.shape[1] != K or (t.shape[0] > 1 and t.stride(1) != 1):
        raise ValueError(f"{name} must be [rows, {K}] and contiguous along K")
    return max(t.stride(0), K) if t.shape[0] > 1 else K


def mxfp8_gemm(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_scale: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [M, N] = (a * 2^(a_scale-127)) @ (b * 2^(b_scale-127)).T, on the current stream.

    a: e4m3 [M, K]; b: e4m3 [N, K]; a_scale / b_scale: e8m0 scales of 1x32
    groups in the swizzled layout ([rows padded to 128] x [K/32 padded to 4]
    bytes). N and K must be multiples of 128.
    """
    M, K = a.shape
    N = b.shape[0]
    lda, ldb = _operand("a", a, K), _operand("b", b, K)
    for name, s, rows in (("a_scale", a_scale, M), ("b_scale", b_scale, N)):
        if s.dtype not in E8M0_DTYPES or not s.is_contiguous() or s.device != a.device:
            raise ValueError(f"{name} must be contiguous e8m0 (or uint8) bytes on {a.device}")
        if s.numel() < mx_swizzled_size(rows, -(-K // 32)):
            raise ValueError(f"{name} holds {s.numel()} bytes, the swizzled layout needs "
                             f"{mx_swizzled_size(rows, -(-K // 32))}")
    if b.device != a.device:
        raise ValueError("a and b must be on the same device")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    elif out.shape != (M, N) or out.dtype != torch.bfloat16 or (N > 1 and out.stride(1) != 1):
        raise ValueError(f"out must be a bf16 [{M}, {N}] tensor contiguous along N")
    ldd = max(out.stride(0), N) if M > 1 else N
    lib = _lib.load()
    with torch.cuda.device(a.device):
        status = lib.cutie_gemm_mxfp8(
            a.data_ptr(), lda, a_scale.data_ptr(), b.data_ptr(), ldb, b_scale.data_ptr(),
            out.data_ptr(), ldd, M, N, K, torch.cuda.current_stream(a.device).cuda_stream)
    _lib.check(status)
    return out


# Rows up to which the fused kernel is the default (measured on a B200 at
# K = N = 5120 against the two-kernel path: with eager launches 1.32-1.41x at
# M = 1-16 and 1.05x at 32; in device time, launches replayed from a CUDA
# graph, 0.93-0.98x at M = 1-16 and 0.71x at 32).
FUSED_MAX_ROWS = 16


def rms_norm_mxfp8_gemm(x: torch.Tensor, weight: torch.Tensor, eps: float, b: torch.Tensor,
                        b_scale: torch.Tensor, out: torch.Tensor | None = None,
                        q: torch.Tensor | None = None,
                        q_scale: torch.Tensor | None = None,
                        fused: bool | None = None) -> torch.Tensor:
    """bf16 [M, N] = mxfp8_gemm(*rms_norm_fp8(x, weight, eps, group 32, e8m0, mx), b, b_scale).

    fused=True (the default up to FUSED_MAX_ROWS rows): one kernel
    (``cutie_rms_norm_mxfp8_gemm``): the RMSNorm and the 1x32 UE8M0
    quantization of x run inside the GEMM as the producer of its A tiles, so
    the FP8 activation is never written to HBM. fused=False (the default
    above it): ``rms_norm_fp8`` then ``mxfp8_gemm``, two kernels, the
    activation through HBM. x: bf16 [M, K] (rows contiguous); weight: bf16
    [K]; b / b_scale: the e4m3 weight [N, K] and its swizzled e8m0 scales, as
    for ``mxfp8_gemm``. ``q`` (e4m3 [M, K]) and ``q_scale`` (swizzled e8m0,
    ``empty_scale(M, K, 32, "e8m0", "mx")``), if given, also receive the
    quantized activation, what ``rms_norm_fp8`` returns for the same x. Runs
    on the current stream.
    """
    if fused is None:
        fused = x.dim() == 2 and x.shape[0] <= FUSED_MAX_ROWS
    if not fused:
        from .fused import empty_scale
        from .ops import launch_rms_norm_fp8

        if (q is None) != (q_scale is None):
            raise ValueError("q and q_scale must be given together")
        M, K = x.shape
        if q is None:
            q = torch.empty(M, K, dtype=FP8_DTYPE, device=x.device)
            q_scale = empty_scale(M, K, 32, "e8m0", "mx", x.device)
        launch_rms_norm_fp8(x, weight, eps, q=q, scale=q_scale, group_size=32,
                            scale_format="e8m0", scale_layout="mx")
        return mxfp8_gemm(q, q_scale, b, b_scale, out=out)
    if not isinstance(x, torch.Tensor) or x.dim() != 2 or not x.is_cuda or x.dtype != torch.bfloat16:
        raise ValueError("x must be a 2-D bf16 CUDA tensor")
    M, K = x.shape
    if M > 0 and K > 1 and x.stride(1) != 1:
        raise ValueError("x must be contiguous along K")
    ldx = max(x.stride(0), K) if M > 1 else K
    if weight.shape != (K,) or weight.dtype != torch.bfloat16 or weight.device != x.device \
            or not weight.is_contiguous():
        raise ValueError(f"weight must be a contiguous bf16 [{K}] tensor on {x.device}")
    N = b.shape[0]
    ldb = _operand("b", b, K)
    if b_scale.dtype not in E8M0_DTYPES or not b_scale.is_contiguous() or b_scale.device != x.device:
        raise ValueError(f"b_scale must be contiguous e8m0 (or uint8) bytes on {x.device}")
    if b_scale.numel() < mx_swizzled_size(N, -(-K // 32)):
        raise ValueError(f"b_scale holds {b_scale.numel()} bytes, the swizzled layout needs "
                         f"{mx_swizzled_size(N, -(-K // 32))}")
    if b.device != x.device:
        raise ValueError("x and b must be on the same device")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    elif out.shape != (M, N) or out.dtype != torch.bfloat16 or (N > 1 and out.stride(1) != 1):
        raise ValueError(f"out must be a bf16 [{M}, {N}] tensor contiguous along N")
    ldd = max(out.stride(0), N) if M > 1 else N
    if (q is None) != (q_scale is None):
        raise ValueError("q and q_scale must be given together")
    ldq = 0
    if q is not None:
        ldq = _operand("q", q, K)
        if q.shape[0] != M:
            raise ValueError(f"q must be [{M}, {K}]")
        if q_scale.dtype not in E8M0_DTYPES or not q_scale.is_contiguous() \
                or q_scale.device != x.device:
            raise ValueError(f"q_scale must be contiguous e8m0 (or uint8) bytes on {x.device}")
        if q_scale.numel() < mx_swizzled_size(M, -(-K // 32)):
            raise ValueError(f"q_scale holds {q_scale.numel()} bytes, the swizzled layout needs "
                             f"{mx_swizzled_size(M, -(-K // 32))}")
    lib = _lib.load()
    with torch.cuda.device(x.device):
        status = lib.cutie_rms_norm_mxfp8_gemm(
            x.data_ptr(), ldx, weight.data_ptr(), float(eps), b.data_ptr(), ldb,
            b_scale.data_ptr(), out.data_ptr(), ldd, M, N, K,
            None if q is None else q.data_ptr(), ldq,
            None if q_scale is None else q_scale.data_ptr(),
            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(status)
    return out
