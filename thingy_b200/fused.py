"""Functional (tensor-in / tensor-out) forms of the fused path.

``residual_rms_norm_fp8`` is the drop-in for the reference's
``residual_rms_norm_fp8_reference`` (src/cutie/rms_norm/bench.py:83-100):
same arguments, same 4-tuple ``(q, scale, residual_out, normalized)``, same
defaults (eps=1e-6, 1x128 groups, fp32 row-major scales). Unlike the
reference, which ignores its output arguments, output tensors passed in are
written and returned (destination passing); missing ones are allocated.

``rms_norm_fp8`` is the general entry: optional residual, per-token / 1xG
group / MXFP8 scaling, fp32 / power-of-two / e8m0 scales, row-major,
column-major or Blackwell-swizzled scale layouts.
"""

from __future__ import annotations

import torch

from .layouts import SCALE_FORMATS, SCALE_LAYOUTS, mx_swizzled_size, n_groups, packed_ld
from .ops import FP8_DTYPE, launch_rms_norm_fp8

E8M0_DTYPE = getattr(torch, "float8_e8m0fnu", torch.uint8)


def empty_scale(M: int, H: int, group_size: int | None, scale_format: str = "fp32",
                scale_layout: str = "row", device=None) -> torch.Tensor:
    """Allocate the scale tensor for one call.

    row: [M, G] row-major. col: a [M, G] view with strides (1, M) over a
    [G, M] buffer (``.t()`` gives the [G, M] tensor a blockwise FP8 GEMM
    reads). mx: flat e8m0 buffer of ceil(M/128)*128 * ceil(G/4)*4 bytes.
    packed (e8m0 only): an int32 [M, ceil(G/4)] view with strides (1, ld),
    ld = M rounded up to 4, four exponents a word (thingy_b200.layouts).
    """
    if scale_format not in SCALE_FORMATS:
        raise ValueError(f"scale_format must be one of {SCALE_FORMATS}")
    if scale_layout not in SCALE_LAYOUTS:
        raise ValueError(f"scale_layout must be one of {SCALE_LAYOUTS}")
    G = n_groups(H, group_size)
    if scale_layout == "packed":
        if scale_format != "e8m0":
            raise ValueError("the packed scale layout needs scale_format='e8m0'")
        W = (G + 3) // 4
        # the unwritten pad bytes of the last word start at zero
        alloc = torch.zeros if G % 4 else torch.empty
        return alloc((W, packed_ld(M)), dtype=torch.int32, device=device).t()[:M]
    dtype = E8M0_DTYPE if scale_format == "e8m0" else torch.float32
    if scale_layout == "mx":
        return torch.empty(mx_swizzled_size(M, G), dtype=dtype, device=device)
    if scale_layout == "col":
        return torch.empty((G, M), dtype=dtype, device=device).t()
    return torch.empty((M, G), dtype=dtype, device=device)


def _as_2d(t: torch.Tensor | None, H: int) -> torch.Tensor | None:
    if t is None:
        return None
    return t if t.dim() == 2 else t.reshape(-1, H)


def rms_norm_fp8(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    residual: torch.Tensor | None = None,
    group_size: int | None = 128,
    scale_format: str = "fp32",
    scale_layout: str = "row",
    out: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    normalized_out: torch.Tensor | None = None,
    return_residual: bool = True,
    return_normalized: bool = False,
    threads_per_row: int = 0,
    stream=None,
):
    """[residual add] -> RMSNorm -> FP8 e4m3. Returns (q, scale, residual_out, normalized).

    x (and residual) are bf16 [..., H]; leading dimensions are flattened.
    residual_out is returned when a residual is given and return_residual is
    true (or residual_out is passed); normalized when return_normalized is
    true (or normalized_out is passed); otherwise those slots are None.
    """
    H = x.shape[-1]
    lead = x.shape[:-1]
    x2 = _as_2d(x, H)
    M = x2.shape[0]
    res2 = _as_2d(residual, H)
    if out is None:
        out = torch.empty_like(x2, dtype=FP8_DTYPE)
    if scale is None:
        scale = empty_scale(M, H, group_size, scale_format, scale_layout, x.device)
    if res2 is not None and residual_out is None and return_residual:
        residual_out = torch.empty_like(x2)
    if normalized_out is None and return_normalized:
        normalized_out = torch.empty_like(x2)
    launch_rms_norm_fp8(
        x2, weight, eps, residual=res2, q=_as_2d(out, H), scale=scale,
        residual_out=_as_2d(residual_out, H), normalized_out=_as_2d(normalized_out, H),
        group_size=group_size, scale_format=scale_format, scale_layout=scale_layout,
        threads_per_row=threads_per_row, stream=stream,
    )
    shape = (*lead, H)
    return (
        out.reshape(shape),
        scale,
        None if residual_out is None else residual_out.reshape(shape),
        None if normalized_out is None else normalized_out.reshape(shape),
    )


def residual_rms_norm_fp8(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    out: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    normalized_out: torch.Tensor | None = None,
):
    """Drop-in for residual_rms_norm_fp8_reference (bench.py:83-100).

    residual_out = x + residual (bf16); normalized = RMSNorm(residual_out)
    (fp32 statistics, bf16 cast before the weight multiply); (q, scale) = the
    1x128 FP8 quantization of normalized with fp32 scales [M, H/128].
    Returns (q, scale, residual_out, normalized); the inputs are not mutated.
    """
    if residual is None:
        raise ValueError("residual is required (use rms_norm_fp8 for the residual-free form)")
    return rms_norm_fp8(
        x, weight, eps, residual=residual, group_size=128, scale_format="fp32",
        scale_layout="row", out=out, scale=scale, residual_out=residual_out,
        normalized_out=normalized_out, return_residual=True, return_normalized=True,
    )
