"""torch.library ops so torch.compile(fullgraph=True) regions can call the path.

``thingy_b200::per_token_fp8_quant`` has the schema of the reference's
``cutie::per_token_fp8_quant`` (src/cutie/rms_norm/bench.py:68-80):
bf16 [M, H] -> (e4m3 [M, H], fp32 [M, ceil(H / 128)]), with a fake (meta)
implementation for tracing. ``thingy_b200::residual_rms_norm_fp8`` is the
whole fused contract (bench.py:10-11): (q, scale, residual_out, normalized).

Importing this module also registers ``cutie::per_token_fp8_quant`` itself,
the name the reference's callers use (``torch.ops.cutie.per_token_fp8_quant``),
backed by this library, unless some module (the reference's own bench.py,
say) has already defined an op of that name: then that one is left in place
and ``REFERENCE_NAMESPACE_OP`` is False. The standalone RMSNorm ops
(``thingy_b200::rms_norm``, ``thingy_b200::rms_norm_out``) are registered by
``thingy_b200.rms_norm``.
"""

from __future__ import annotations

import torch

from .fp8_utils import per_token_cast_to_fp8
from .fused import residual_rms_norm_fp8

GROUP_SIZE = 128


@torch.library.custom_op("thingy_b200::per_token_fp8_quant", mutates_args=())
def quantize_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    return per_token_cast_to_fp8(x, use_ue8m0=False)


@quantize_fp8.register_fake
def _quantize_fp8_fake(x):
    return (
        torch.empty_like(x, dtype=torch.float8_e4m3fn),
        x.new_empty((x.shape[0], -(-x.shape[1] // GROUP_SIZE)), dtype=torch.float32),
    )


@torch.library.custom_op("thingy_b200::residual_rms_norm_fp8", mutates_args=())
def residual_rms_norm_fp8_op(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return residual_rms_norm_fp8(x, residual, weight, eps)


@residual_rms_norm_fp8_op.register_fake
def _residual_rms_norm_fp8_fake(x, residual, weight, eps):
    return (
        torch.empty_like(x, dtype=torch.float8_e4m3fn),
        x.new_empty((x.shape[0], -(-x.shape[1] // GROUP_SIZE)), dtype=torch.float32),
        torch.empty_like(x),
        torch.empty_like(x),
    )


def _reference_op_defined() -> bool:
    try:
        torch.ops.cutie.per_token_fp8_quant
    except (AttributeError, RuntimeError):
        return False
    return True


REFERENCE_NAMESPACE_OP = False
if not _reference_op_defined():

    @torch.library.custom_op("cutie::per_token_fp8_quant", mutates_args=())
    def cutie_per_token_fp8_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return per_token_cast_to_fp8(x, use_ue8m0=False)

    @cutie_per_token_fp8_quant.register_fake
    def _cutie_per_token_fp8_quant_fake(x):
        return _quantize_fp8_fake(x)

    REFERENCE_NAMESPACE_OP = True
