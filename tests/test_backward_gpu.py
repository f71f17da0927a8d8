"""GPU parity of the backward kernel (csrc/backward.cu) against the CPU oracle.

The oracle is torch autograd of the reference's forward
(oracle.reference.rms_norm_fp8_backward, pinned to the reference's own
autograd in test_backward_oracle.py). Tolerance contract:

* dx: bit-exact on >= 99% of elements, and everywhere within the fp32
  rounding error of its two terms (dt * inv and dsq * 2r, which can cancel)
  plus the two bf16 roundings, measured against a float64 evaluation (the
  row sums sum(r^2) and sum(dt * r) are added in another order; the CPU
  oracle meets the same bound); fully bit-exact on inputs whose sums are
  exact in any order (values k/16);
* d_weight: within the error of an fp32 sum over the rows (accumulated in
  another order) plus one bf16 rounding; bit-identical from run to run;
* the FP8 codes and scales of dx: bit-exact against quantizing the GPU's
  own dx with the oracle.
"""

import numpy as np
import pytest
import torch

from oracle import reference as ora
from parity import bf16_bits, bf16_ulp_diff, q_codes

import thingy_b200 as tb
from thingy_b200.ops import backward_workspace_bytes

pytestmark = pytest.mark.gpu


def _inputs(M, H, residual, seed, exact=False):
    g = torch.Generator().manual_seed(seed)
    if exact:
        # k/16 values and power-of-two weights: dt = dn * w is exact, and both
        # row sums (of multiples of 2^-9 below 2^15) are exact in any order
        rnd = lambda: torch.randint(-16, 17, (M, H), generator=g).float() / 16
        x, res, dn, dro = rnd(), rnd(), rnd(), rnd()
        w = torch.exp2(torch.randint(-1, 2, (H,), generator=g).float())
    else:
        x = torch.randn(M, H, generator=g)
        res = 2.0 * torch.randn(M, H, generator=g)
        dn = torch.randn(M, H, generator=g)
        dro = torch.randn(M, H, generator=g)
        w = 1.0 + 0.1 * torch.randn(H, generator=g)
    bf = lambda t: t.to(torch.bfloat16)
    d = {"x": bf(x), "weight": bf(w), "d_normalized": bf(dn), "eps": 1e-6}
    if residual:
        d["residual"] = bf(res)
        d["d_residual_out"] = bf(dro)
    return d


def _gpu_backward(d, quantize=False, scale_format="fp32", scale_layout="row"):
    dev = torch.device("cuda")
    r = d["x"] + d["residual"] if "residual" in d else d["x"]
    dro = d.get("d_residual_out")
    dx, dw, q, s = tb.rms_norm_fp8_backward(
        d["d_normalized"].to(dev), r.to(dev), d["weight"].to(dev), d["eps"],
        d_residual_out=None if dro is None else dro.to(dev), weight_grad=True,
        quantize=quantize, scale_format=scale_format, scale_layout=scale_layout)
    torch.cuda.synchronize()
    return dx.cpu(), dw.cpu(), q, s


def _scale_buffer(s, layout, fmt):
    """The device buffer of a scale tensor, as oracle.layout_scales lays it out."""
    t = s.detach().cpu()
    if layout == "packed":  # [M, W] int32 view -> [W, M] words
        return t.t().contiguous().numpy()
    if fmt == "e8m0":
        t = t.view(torch.uint8)
    if layout == "col":
        return t.t().contiguous().numpy()
    return t.numpy().reshape(-1) if layout == "mx" else t.numpy()


def _oracle(d):
    dx, dw, _, _ = ora.rms_norm_fp8_backward(
        d["x"], d["weight"], d["d_normalized"], d["eps"], residual=d.get("residual"),
        d_residual_out=d.get("d_residual_out"), scale_format=None)
    return dx, dw


def _check_dx(dx, d):
    """dx (bf16) against a float64 evaluation, within fp32 + bf16 rounding."""
    r = d["x"] + d["residual"] if "residual" in d else d["x"]
    rf = r.double()
    H = rf.shape[-1]
    inv = 1.0 / torch.sqrt(rf.square().mean(-1, keepdim=True) + d["eps"])
    dt = (d["d_normalized"] * d["weight"]).double()
    b = (dt * rf).sum(-1, keepdim=True)
    g1 = dt * inv
    g2 = ((-0.5 * b) * inv ** 3 / H) * (2 * rf)
    exact = g1 + g2
    tol = (g1.abs() + g2.abs()) * 2.0 ** -20 + exact.abs() * 2.0 ** -8
    if "d_residual_out" in d:
        exact = exact + d["d_residual_out"].double()
        tol = tol + exact.abs() * 2.0 ** -8
    err = (dx.double() - exact).abs()
    assert bool((err <= tol + 1e-30).all()), float((err - tol).max())


def _check_dw(dw_gpu, d):
    """|dw - sum| within an fp32-accumulation bound plus a bf16 rounding."""
    r = d["x"] + d["residual"] if "residual" in d else d["x"]
    rf = r.float()
    inv = torch.rsqrt(rf.square().mean(-1, keepdim=True) + d["eps"])
    p = (d["d_normalized"] * (rf * inv).to(torch.bfloat16)).double()
    exact = p.sum(0)
    M = p.shape[0]
    bound = exact.abs() * 2.0 ** -8 + p.abs().sum(0) * (M + 8) * 2.0 ** -22
    err = (dw_gpu.double() - exact).abs()
    assert bool((err <= bound).all()), float((err - bound).max())


# up to 8192: the ring kernel, two CTAs an SM; 12288 and 16384: the ring
# kernel, one 384- / 512-thread CTA an SM; 20480 and 32768: the direct kernel
SHAPES = [(64, 1024), (300, 7168), (129, 8192), (33, 200), (7, 4096), (1, 5120), (260, 3000),
          (300, 12288), (150, 16384), (40, 20480), (17, 32768)]


@pytest.mark.parametrize("M,H", SHAPES)
@pytest.mark.parametrize("residual", [False, True])
def test_backward_random(M, H, residual):
    d = _inputs(M, H, residual, seed=M * 31 + H)
    dx, dw, _, _ = _gpu_backward(d)
    dx_ref, _ = _oracle(d)
    ulps = bf16_ulp_diff(bf16_bits(dx), bf16_bits(dx_ref))
    assert (ulps == 0).mean() >= 0.99
    _check_dx(dx, d)
    _check_dx(dx_ref, d)
    _check_dw(dw, d)


@pytest.mark.parametrize("M,H", [(64, 1024), (100, 7168), (9, 200), (40, 8192), (200, 16384),
                                 (30, 32768)])
@pytest.mark.parametrize("residual", [False, True])
def test_backward_exact_sums_bitexact(M, H, residual):
    d = _inputs(M, H, residual, seed=M + H, exact=True)
    dx, dw, _, _ = _gpu_backward(d)
    dx_ref, _ = _oracle(d)
    assert torch.equal(dx, dx_ref)
    _check_dw(dw, d)


@pytest.mark.parametrize("fmt,layout", [("fp32", "row"), ("fp32", "col"), ("ue8m0", "row"),
                                        ("e8m0", "row"), ("e8m0", "mx"), ("e8m0", "packed")])
@pytest.mark.parametrize("M,H", [(256, 7168), (70, 1000), (160, 16384), (20, 24576)])
def test_backward_fp8_quant_of_dx(fmt, layout, M, H):
    d = _inputs(M, H, True, seed=7 * M + H)
    dx, _, q, s = _gpu_backward(d, quantize=True, scale_format=fmt, scale_layout=layout)
    q_ref, s_ref = ora.quantize(dx, 128, fmt)
    assert np.array_equal(q_codes(q), q_ref.numpy())
    want = ora.layout_scales(s_ref, layout)
    if layout == "packed":
        want = want[:, :M]  # the words of the M rows (the pad rows are not written)
    assert np.array_equal(_scale_buffer(s, layout, fmt), want)


def test_weight_grad_is_deterministic():
    d = _inputs(2048, 4096, True, seed=5)
    _, dw1, _, _ = _gpu_backward(d)
    _, dw2, _, _ = _gpu_backward(d)
    assert torch.equal(dw1, dw2)


def test_autograd_function():
    d = _inputs(96, 2048, True, seed=11)
    dev = torch.device("cuda")
    x = d["x"].to(dev).requires_grad_(True)
    res = d["residual"].to(dev).requires_grad_(True)
    w = d["weight"].to(dev).requires_grad_(True)
    q, s, r, n = tb.ResidualRMSNormFP8.apply(x, res, w, d["eps"], 128, "fp32", "row")
    torch.autograd.backward([n, r], [d["d_normalized"].to(dev), d["d_residual_out"].to(dev)])
    dx_ref, _ = _oracle(d)
    ulps = bf16_ulp_diff(bf16_bits(x.grad.cpu()), bf16_bits(dx_ref))
    assert (ulps == 0).mean() >= 0.99
    _check_dx(x.grad.cpu(), d)
    assert torch.equal(x.grad, res.grad)
    _check_dw(w.grad.cpu(), d)


def test_empty_batch_and_errors():
    dev = torch.device("cuda")
    H = 1024
    z = torch.empty(0, H, dtype=torch.bfloat16, device=dev)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    dx, dw, _, _ = tb.rms_norm_fp8_backward(z, z, w, 1e-6)
    torch.cuda.synchronize()
    assert dx.shape == (0, H) and torch.count_nonzero(dw) == 0
    x = torch.zeros(4, 40000, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        tb.rms_norm_fp8_backward(x, x, torch.ones(40000, dtype=torch.bfloat16, device=dev))
    x = torch.zeros(4, H, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(16, dtype=torch.uint8, device=dev)
    assert backward_workspace_bytes(4, H) > 16
    with pytest.raises(ValueError):
        tb.rms_norm_fp8_backward(x, x, w, workspace=ws)
