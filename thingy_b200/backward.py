"""Backward of the fused path, and an autograd Function around both directions.

The reference (S1ro1/thingy) has no backward pass: its fused RMSNorm -> FP8
kernel and its PyTorch reference path are forward only
(src/cutie/rms_norm/bench.py). The gradients here are the ones torch
autograd computes for that PyTorch path (bench.py:58-65 and the residual add
of :97), op for op; csrc/backward.cu states them.

``rms_norm_fp8_backward`` is the functional form (destination passing when
outputs are given). ``ResidualRMSNormFP8`` runs the fused forward and this
backward under autograd: the FP8 codes and scales are not differentiable;
the gradient that reaches them is expected as the gradient of the bf16
normalized output (what a dgrad GEMM in FP8 training returns), and the
residual stream's gradient as that of residual_out.
"""

from __future__ import annotations

import torch

from .fused import empty_scale, rms_norm_fp8
from .ops import FP8_DTYPE, backward_workspace_bytes, launch_rms_norm_backward


def rms_norm_fp8_backward(
    d_normalized: torch.Tensor,
    r: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    d_residual_out: torch.Tensor | None = None,
    weight_grad: bool = True,
    quantize: bool = False,
    scale_format: str = "fp32",
    scale_layout: str = "row",
    dx: torch.Tensor | None = None,
    d_weight: torch.Tensor | None = None,
    q: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
):
    """Gradients of [residual add] -> RMSNorm.

    r is the forward's RMSNorm input (residual_out when there was a residual,
    else x). Returns (dx, d_weight, q, scale): dx is the gradient of x and of
    the residual; d_weight (bf16 [H]) is None unless ``weight_grad``;
    q / scale quantize dx in 1x128 groups when ``quantize`` (or when q and
    scale are given).
    """
    M, H = d_normalized.shape
    device = d_normalized.device
    if dx is None:
        dx = torch.empty(M, H, dtype=torch.bfloat16, device=device)
    if weight_grad:
        if d_weight is None:
            d_weight = torch.empty(H, dtype=torch.bfloat16, device=device)
        if workspace is None:
            workspace = torch.empty(backward_workspace_bytes(M, H, device), dtype=torch.uint8,
                                    device=device)
    else:
        d_weight = None
    if quantize or q is not None or scale is not None:
        if q is None:
            q = torch.empty(M, H, dtype=FP8_DTYPE, device=device)
        if scale is None:
            scale = empty_scale(M, H, 128, scale_format, scale_layout, device)
    launch_rms_norm_backward(
        d_normalized, r, weight, eps, dx=dx, d_residual_out=d_residual_out, d_weight=d_weight,
        workspace=workspace, q=q, scale=scale, scale_format=scale_format,
        scale_layout=scale_layout,
    )
    return dx, d_weight, q, scale


class ResidualRMSNormFP8(torch.autograd.Function):
    """(x, residual, weight) -> (q, scale, residual_out, normalized) with a backward.

    residual may be None. The forward is the fused kernel (1xG or per-token
    FP8 quantization as requested); the backward is csrc/backward.cu. q and
    scale carry no gradient.
    """

    @staticmethod
    def forward(ctx, x, residual, weight, eps=1e-6, group_size=128, scale_format="fp32",
                scale_layout="row"):
        q, scale, r, n = rms_norm_fp8(
            x, weight, eps, residual=residual, group_size=group_size, scale_format=scale_format,
            scale_layout=scale_layout, return_normalized=True,
        )
        ctx.save_for_backward(r if residual is not None else x, weight)
        ctx.eps = eps
        ctx.has_residual = residual is not None
        ctx.mark_non_differentiable(q, scale)
        if r is None:
            r = torch.empty(0, device=x.device, dtype=x.dtype)
            ctx.mark_non_differentiable(r)
        return q, scale, r, n

    @staticmethod
    def backward(ctx, dq, dscale, d_residual_out, d_normalized):
        r, weight = ctx.saved_tensors
        if d_normalized is None:
            d_normalized = torch.zeros_like(r)
        dro = d_residual_out if ctx.has_residual and d_residual_out is not None else None
        dx, dw, _, _ = rms_norm_fp8_backward(
            d_normalized.contiguous(), r, weight, ctx.eps,
            d_residual_out=None if dro is None else dro.contiguous(),
            weight_grad=ctx.needs_input_grad[2],
        )
        dres = dx if ctx.has_residual and ctx.needs_input_grad[1] else None
        return dx, dres, dw, None, None, None, None
