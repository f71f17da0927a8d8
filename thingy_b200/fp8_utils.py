"""Drop-in for the activation quantizer of src/cutie/vendor/prime_rl/fp8_utils.py.

``per_token_cast_to_fp8(x, use_ue8m0, gran_k=128)`` returns the same
``(out e4m3 [M, H], sf fp32 [M, ceil(H/gran_k)])`` as
``per_token_cast_to_fp8_triton`` (fp8_utils.py:63-89): per (row, gran_k
group) amax, ``s = max(amax/448, 1e-4)``, ``2^ceil(log2 s)`` when use_ue8m0,
``e4m3(x / s)``; a partial last group is reduced over its valid columns only.
It runs the hand-written sm_100a kernel; gran_k may also be 32 or 64.
"""

from __future__ import annotations

import torch

from .fused import empty_scale
from .ops import FP8_DTYPE, launch_rms_norm_fp8

GROUP_ALIGNMENT = 128


def ceil_div(x: int, y: int) -> int:
    return (x + y - 1) // y


def per_token_cast_to_fp8(
    x: torch.Tensor, use_ue8m0: bool, gran_k: int = GROUP_ALIGNMENT
) -> tuple[torch.Tensor, torch.Tensor]:
    assert x.dim() == 2
    assert gran_k in (32, 64, 128)
    rows, cols = x.shape
    out = torch.empty_like(x, dtype=FP8_DTYPE)
    sf = empty_scale(rows, cols, gran_k, "ue8m0" if use_ue8m0 else "fp32", "row", x.device)
    launch_rms_norm_fp8(
        x, None, 0.0, q=out, scale=sf, group_size=gran_k,
        scale_format="ue8m0" if use_ue8m0 else "fp32", scale_layout="row", normalize=False,
    )
    return out, sf


# The name the reference's callers import (fp8_utils.py:63).
per_token_cast_to_fp8_triton = per_token_cast_to_fp8
