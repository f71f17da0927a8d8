"""Drop-in for src/cutie/rms_norm/rms_norm.py.

``RMSNorm`` keeps the reference class's constructor knobs and its
destination-passing ``__call__(x, residual, weight, eps, out, scale,
residual_out, normalized_out, stream)`` (rms_norm.py:36-113), but launches the
hand-written sm_100a kernel through the C ABI instead of a CuTe DSL JIT.
``rms_norm`` / ``rms_norm_on_stream`` replace the torch.compile baseline
(rms_norm.py:11-33); ``out`` is honoured here (the reference ignores it).
The reference's ``rms_norm`` is itself a torch.compile region; here it is
backed by two torch.library ops with fake implementations,
``thingy_b200::rms_norm`` (functional) and ``thingy_b200::rms_norm_out``
(writes ``out``), so ``torch.compile(fullgraph=True)`` traces a call to
``rms_norm`` as one opaque op. Eager calls skip the op dispatcher and launch
through the binding directly.
"""

from __future__ import annotations

import torch

from .ops import launch_rms_norm, launch_rms_norm_fp8

_LOAD_PATHS = ("shared", "direct")
_REDUCTIONS = ("warp0", "all")


def _threads_hint(threads_per_row: int | None, H: int) -> int:
    """The requested threads per row when this kernel can honour it, else 0 (auto)."""
    if not threads_per_row:
        return 0
    chunks = -(-H // 32)  # 64-byte chunks of a bf16 row
    per_thread = max(1, -(-chunks // threads_per_row))
    ok = per_thread == 1 or (per_thread == 2 and threads_per_row <= 512)
    return threads_per_row if ok else 0


class RMSNorm:
    """Fused residual add -> RMSNorm -> 1x128 FP8 quantization (bf16 in).

    elements_per_thread, threads_per_row, load_path and reduction are the
    reference's compile-time knobs (rms_norm.py:37-48) and are validated the
    way its bench validates them (bench.py:166-188). This kernel always moves
    16-byte vectors and keeps the row in registers, so load_path and reduction
    do not change the result or the code path; threads_per_row is used as the
    CTA size whenever it covers the row with one 64-byte chunk per thread (or
    two, up to 512 threads).

    Keyword-only extensions select per-token (group_size=None), 1x32/1x64
    groups, power-of-two or e8m0 scales and column-major or swizzled layouts.
    """

    def __init__(
        self,
        elements_per_thread: int = 8,
        threads_per_row: int | None = None,
        load_path: str = "shared",
        reduction: str = "all",
        *,
        group_size: int | None = 128,
        scale_format: str = "fp32",
        scale_layout: str = "row",
    ):
        if elements_per_thread not in (4, 8):
            raise ValueError("elements_per_thread must be 4 or 8")
        if threads_per_row is not None and (
            not 32 <= threads_per_row <= 1024 or threads_per_row % 32
        ):
            raise ValueError("threads_per_row must be a multiple of 32 between 32 and 1024")
        if load_path not in _LOAD_PATHS:
            raise ValueError(f"load_path must be one of {_LOAD_PATHS}")
        if reduction not in _REDUCTIONS:
            raise ValueError(f"reduction must be one of {_REDUCTIONS}")
        self.elements_per_thread = elements_per_thread
        self.threads_per_row = threads_per_row
        self.load_path = load_path
        self.reduction = reduction
        self.group_size = group_size
        self.scale_format = scale_format
        self.scale_layout = scale_layout

    def __call__(
        self,
        x: torch.Tensor,
        residual: torch.Tensor | None,
        weight: torch.Tensor,
        eps: float,
        out: torch.Tensor,
        scale: torch.Tensor,
        residual_out: torch.Tensor | None,
        normalized_out: torch.Tensor | None,
        stream=None,
    ) -> None:
        """Write q (out), scale, residual_out and normalized_out; returns nothing."""
        launch_rms_norm_fp8(
            x, weight, eps, residual=residual, q=out, scale=scale, residual_out=residual_out,
            normalized_out=normalized_out, group_size=self.group_size,
            scale_format=self.scale_format, scale_layout=self.scale_layout,
            threads_per_row=_threads_hint(self.threads_per_row, x.shape[-1]), stream=stream,
        )


def _rms_norm_into(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> None:
    H = x.shape[-1]
    x2 = x if x.dim() == 2 else x.reshape(-1, H)
    out2 = out if out.dim() == 2 else out.view(-1, H)
    launch_rms_norm(x2, weight, eps, out2)


@torch.library.custom_op("thingy_b200::rms_norm", mutates_args=())
def rms_norm_op(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    _rms_norm_into(x, weight, eps, out)
    return out


@rms_norm_op.register_fake
def _rms_norm_op_fake(x, weight, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("thingy_b200::rms_norm_out", mutates_args=("out",))
def rms_norm_out_op(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> None:
    _rms_norm_into(x, weight, eps, out)


@rms_norm_out_op.register_fake
def _rms_norm_out_op_fake(x, weight, eps, out):
    return None


def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-5,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Standalone RMSNorm on the current stream.

    fp32 x: ``x / sqrt(mean(x^2) + eps) * weight`` in fp32 (rms_norm.py:11-20).
    bf16 x: ``bf16(x * rsqrt(mean(x^2) + eps)) * weight`` with fp32 statistics
    (the Prime-RL form at bench.py:58-65 that the fused path generalises).
    Inside a torch.compile region the call is the op ``thingy_b200::rms_norm``
    (or ``thingy_b200::rms_norm_out`` when ``out`` is given).
    """
    if torch.compiler.is_compiling():
        if out is None:
            return torch.ops.thingy_b200.rms_norm(x, weight, float(eps))
        torch.ops.thingy_b200.rms_norm_out(x, weight, float(eps), out)
        return out
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    _rms_norm_into(x, weight, eps, out)
    return out


def rms_norm_on_stream(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    out: torch.Tensor | None,
    *,
    stream: torch.cuda.Stream,
) -> torch.Tensor:
    """Launch the standalone RMSNorm on a specific CUDA stream (rms_norm.py:23-33)."""
    with torch.cuda.stream(stream):
        return rms_norm(x, weight, eps, out)
