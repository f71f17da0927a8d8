"""thingy_b200 — B200-native (sm_100a) residual-add + RMSNorm + FP8 quantization.

Drop-in host API for the reference's hot path (S1ro1/thingy, package
``cutie``):

    RMSNorm, rms_norm, rms_norm_on_stream   <- src/cutie/rms_norm/rms_norm.py
    residual_rms_norm_fp8                   <- residual_rms_norm_fp8_reference,
                                               src/cutie/rms_norm/bench.py:83-100
    per_token_cast_to_fp8(_triton)          <- src/cutie/vendor/prime_rl/fp8_utils.py:63-89
    rms_norm_fp8                            general form (per-token / 1xG / MXFP8,
                                               fp32 / pow2 / e8m0 scales, layouts)
    rms_norm_fp8_backward, ResidualRMSNormFP8
                                            backward (no counterpart in the reference):
                                               the gradients autograd gives its forward

Every op runs hand-written CUDA from ``lib/libcutie_b200.so`` through the C
ABI in ``include/cutie.h``; there is no CPU or PyTorch fallback.
"""

from .backward import ResidualRMSNormFP8, rms_norm_fp8_backward
from .fp8_utils import per_token_cast_to_fp8, per_token_cast_to_fp8_triton
from .fused import empty_scale, residual_rms_norm_fp8, rms_norm_fp8
from .layouts import mx_swizzle, mx_swizzle_offset, mx_swizzled_size, mx_unswizzle
from .rms_norm import RMSNorm, rms_norm, rms_norm_on_stream

__all__ = [
    "RMSNorm",
    "ResidualRMSNormFP8",
    "empty_scale",
    "mx_swizzle",
    "mx_swizzle_offset",
    "mx_swizzled_size",
    "mx_unswizzle",
    "per_token_cast_to_fp8",
    "per_token_cast_to_fp8_triton",
    "residual_rms_norm_fp8",
    "rms_norm",
    "rms_norm_fp8",
    "rms_norm_fp8_backward",
    "rms_norm_on_stream",
]
