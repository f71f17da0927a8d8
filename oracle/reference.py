"""CPU oracle of the fused RMSNorm -> FP8 path.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this module, and only as the checker or the timed CPU baseline; the
product path (thingy_b200) never calls it.

It restates the reference's own PyTorch path with the same torch CPU ops:
  rms_norm_reference     src/cutie/rms_norm/bench.py:58-65
  residual add           src/cutie/rms_norm/bench.py:97
  group quantization     src/cutie/vendor/prime_rl/fp8_utils.py:38-60
                         (the Triton kernel's tensor math: masked load with
                         other=0.0 :45-49, amax :50, clamp :51, UE8M0 :52-53,
                         divide :54, e4m3 cast :57)
  fp32 rms_norm          src/cutie/rms_norm/rms_norm.py:11-20 (eager form)
  backward               torch autograd of the forward above (the reference
                         has no backward pass)
generalised to one scale per row (group = H), 1x32 / 1x64 groups and e8m0
bytes, which the reference does not implement (its quantizer asserts
gran_k == 128, fp8_utils.py:67).

Pinning: tests/golden/ holds vectors produced by importing the reference's
own functions (bench.py's rms_norm_reference and residual path, and the
vendored Triton kernel run by Triton's CPU interpreter); tests check this
oracle against them. The interpreter mis-rounds e4m3 when rounding carries
into the next binade; those elements are recorded and checked separately.
"""

from __future__ import annotations

import numpy as np
import torch

E4M3_MAX = 448.0
MIN_SCALE = 1e-4


def residual_add(x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """bench.py:97 — bf16 + bf16 (fp32 sum rounded to bf16)."""
    return x + residual


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """bench.py:58-65 — fp32 statistics, cast to x.dtype before the weight multiply."""
    x_f32 = x.float()
    variance = x_f32.square().mean(dim=-1, keepdim=True)
    normalized = x_f32 * torch.rsqrt(variance + eps)
    return normalized.to(x.dtype) * weight


def rms_norm_f32(
    x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5, ieee_sqrt: bool = True
) -> torch.Tensor:
    """rms_norm.py:11-20 — the standalone fp32 RMSNorm.

    The reference runs this under torch.compile on the GPU, where the square
    root is the IEEE (correctly rounded) one. Eager torch on the CPU is not
    always: on AVX-512 builds its float32 sqrt was observed 1 ulp off
    (sqrt(1.360060215) -> 1.1662161 instead of 1.1662163). ieee_sqrt=True
    (default) takes the square root in float64 and rounds it to float32,
    which is the correctly rounded float32 square root (the double rounding
    is innocuous for sqrt); ieee_sqrt=False is the literal eager expression.
    """
    variance = x.pow(2).mean(dim=-1, keepdim=True) + eps
    root = torch.sqrt(variance.double()).float() if ieee_sqrt else torch.sqrt(variance)
    x = x / root
    return x * weight


def pow2_ceil(scale: torch.Tensor) -> torch.Tensor:
    """fp8_utils.py:52-53 — 2^ceil(log2 s), computed exactly from the bits.

    For positive normal fp32 s this equals exp2(ceil(log2(s))) whenever log2
    is exact on powers of two and distinguishes non-powers; the bit form has
    no such caveat. tests/test_oracle.py checks both agree on the inputs used.
    """
    bits = scale.contiguous().view(torch.int32)
    exp = bits & 0x7F800000
    bumped = torch.where((bits & 0x007FFFFF) != 0, exp + 0x00800000, exp)
    return bumped.view(torch.float32)


def quantize(
    n: torch.Tensor, group_size: int | None = 128, scale_format: str = "fp32"
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-(row, group) FP8 e4m3 quantization of n [M, H].

    group_size None means one group per row. Returns (q as uint8 codes [M, H],
    scale [M, G]): fp32 for "fp32" / "ue8m0", uint8 biased exponents for
    "e8m0". A partial last group is padded with zeros, as the Triton kernel's
    masked load (other=0.0) does.
    """
    M, H = n.shape
    gs = H if not group_size else group_size
    G = -(-H // gs)
    xf = n.float()
    if G * gs != H:
        xf = torch.nn.functional.pad(xf, (0, G * gs - H))
    xg = xf.view(M, G, gs)
    amax = xg.abs().amax(dim=-1)
    scale = torch.clamp(amax / E4M3_MAX, min=MIN_SCALE)
    if scale_format in ("ue8m0", "e8m0"):
        scale = pow2_ceil(scale)
    y = xg / scale[..., None]
    q = y.to(torch.float8_e4m3fn).view(torch.uint8).view(M, G * gs)[:, :H].contiguous()
    if scale_format == "e8m0":
        scale = ((scale.view(torch.int32) >> 23) & 0xFF).to(torch.uint8)
    return q, scale


def rms_norm_fp8(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    residual: torch.Tensor | None = None,
    group_size: int | None = 128,
    scale_format: str = "fp32",
):
    """[residual add] -> rms_norm_reference -> quantize (bench.py:83-100 generalised).

    Returns (q uint8 [M, H], scale [M, G], residual_out or None, normalized).
    """
    r = residual_add(x, residual) if residual is not None else x
    n = rms_norm_reference(r, weight, eps)
    q, s = quantize(n, group_size, scale_format)
    return q, s, (r if residual is not None else None), n


class _IeeeRsqrt(torch.autograd.Function):
    """RN(1 / RN(sqrt(v))) with a correctly rounded square root, and rsqrt's
    autograd rule (-0.5 * grad * result^3).

    Eager torch on some CPUs (AVX-512 builds) returns a float32 sqrt 1 ulp off
    for some inputs; the reference computes on the GPU, whose sqrt is IEEE.
    The float64 sqrt rounded to float32, and the float64 quotient rounded to
    float32, are the correctly rounded float32 results (double rounding is
    innocuous for sqrt and division at these precisions).
    """

    @staticmethod
    def forward(ctx, v):
        root = torch.sqrt(v.double()).float()
        y = (1.0 / root.double()).float()
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, grad):
        (y,) = ctx.saved_tensors
        return -0.5 * grad * y.pow(3)


def rms_norm_fp8_backward(
    x: torch.Tensor,
    weight: torch.Tensor,
    d_normalized: torch.Tensor,
    eps: float = 1e-6,
    residual: torch.Tensor | None = None,
    d_residual_out: torch.Tensor | None = None,
    group_size: int | None = None,
    scale_format: str = "fp32",
    ieee_rsqrt: bool = True,
):
    """Gradients of rms_norm_fp8's differentiable outputs, by torch autograd.

    The reference has no backward pass; its forward (bench.py:58-65 and the
    residual add of bench.py:97, restated above with the same torch ops) is
    differentiated by autograd on the CPU. The FP8 codes and scales are not
    differentiable: the gradient that reaches them arrives as
    ``d_normalized`` (the bf16 gradient of the normalized output), and
    ``d_residual_out`` is the gradient of residual_out (the residual stream).

    Returns (dx, d_weight, q, scale): dx is the gradient of x (and of
    residual, which receives the same tensor); q / scale quantize dx like
    ``quantize`` (None when scale_format is None). ieee_rsqrt (default)
    takes inv_rms with an IEEE square root (see _IeeeRsqrt); False is the
    literal eager rms_norm_reference.
    """
    xg = x.detach().clone().requires_grad_(True)
    wg = weight.detach().clone().requires_grad_(True)
    if residual is not None:
        rg = residual.detach().clone().requires_grad_(True)
        r = residual_add(xg, rg)
    else:
        r = xg
    if ieee_rsqrt:  # rms_norm_reference's ops with the IEEE rsqrt of the GPU
        r_f32 = r.float()
        inv = _IeeeRsqrt.apply(r_f32.square().mean(dim=-1, keepdim=True) + eps)
        n = (r_f32 * inv).to(r.dtype) * wg
    else:
        n = rms_norm_reference(r, wg, eps)
    outs, grads = [n], [d_normalized]
    if residual is not None and d_residual_out is not None:
        outs.append(r)
        grads.append(d_residual_out)
    torch.autograd.backward(outs, grads)
    dx = xg.grad
    q = s = None
    if scale_format is not None:
        q, s = quantize(dx, group_size, scale_format)
    return dx, wg.grad, q, s


def ue8m0_pack(scales: np.ndarray) -> np.ndarray:
    """[M, G] e8m0 bytes -> [ceil(G/4), ld] int32 words, ld = M rounded up to 4.

    Word (j, m) holds the exponents of groups 4j..4j+3 of row m, group 4j in
    the least significant byte; missing groups and pad rows are 0. Written
    independently of thingy_b200.layouts (which the kernel mirrors).
    """
    M, G = scales.shape
    W, ld = -(-G // 4), -(-M // 4) * 4
    out = np.zeros((W, ld), dtype=np.int64)
    for g in range(G):
        out[g // 4, :M] |= scales[:, g].astype(np.int64) << (8 * (g % 4))
    return out.astype(np.uint32).view(np.int32)


def mx_swizzle(scales: np.ndarray) -> np.ndarray:
    """[M, G] e8m0 bytes -> flat Blackwell block-scaled layout (zero padded).

    Restated from the public cuBLAS / PTX description of the 1D block
    scaling-factor layout: 128x4 tiles, 512 bytes each, tile-row-major;
    inside a tile row r, column c at (r % 32) * 16 + (r // 32) * 4 + c.
    Written independently of thingy_b200.layouts (which the kernel mirrors).
    """
    M, G = scales.shape
    rows = -(-M // 128) * 128
    cols = -(-G // 4) * 4
    padded = np.zeros((rows, cols), dtype=np.uint8)
    padded[:M, :G] = scales
    # tile view [row_tile, 128, col_tile, 4] -> [row_tile, col_tile, 4 (r//32), 32 (r%32), 4 (c)]
    t = padded.reshape(rows // 128, 4, 32, cols // 4, 4)  # r = 32*a + b
    t = t.transpose(0, 3, 2, 1, 4)  # [rt, ct, b (r%32), a (r//32), c]
    return np.ascontiguousarray(t).reshape(-1)


def layout_scales(scale: torch.Tensor, layout: str) -> np.ndarray:
    """The device buffer contents for a [M, G] scale matrix in ``layout``."""
    s = scale.numpy()
    if layout == "row":
        return s
    if layout == "col":
        return np.ascontiguousarray(s.T)
    if layout == "mx":
        return mx_swizzle(s)
    if layout == "packed":
        return ue8m0_pack(s)
    raise ValueError(layout)
