"""The backward oracle against gradients of the reference's own forward.

tests/golden/backward_vectors.npz holds torch-autograd gradients of the
reference's rms_norm_reference and residual add (bench.py:58-65, :97),
produced by tests/golden/make_backward_golden.py from the reference's code.
oracle.reference.rms_norm_fp8_backward restates that forward and must give
the same gradients bit for bit. Also checked here, on the CPU: the
closed-form gradient the CUDA kernel computes (csrc/backward.cu) equals
autograd's bit for bit on these inputs.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference as ora

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "backward_vectors.npz")
CASES = sorted({k.split("__")[0] for k in GOLD.files})


def _bf16(a):
    return torch.from_numpy(np.asarray(a).astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _load(tag):
    get = lambda k: GOLD[f"{tag}__{k}"]
    d = {k: _bf16(get(k)) for k in ("x", "weight", "d_normalized", "dx", "d_weight")}
    d["eps"] = float(get("eps"))
    if f"{tag}__residual" in GOLD.files:
        d["residual"] = _bf16(get("residual"))
        d["d_residual_out"] = _bf16(get("d_residual_out"))
    return d


def closed_form(x, w, dn, eps, residual=None, dro=None):
    """The kernel's formula (csrc/backward.cu), in torch fp32 ops on the CPU."""
    r = x + residual if residual is not None else x
    rf = r.float()
    H = rf.shape[-1]
    inv = torch.rsqrt(rf.square().mean(-1, keepdim=True) + eps)
    dt = (dn * w).float()
    b = (dt * rf).sum(-1, keepdim=True)
    dsq = ((-0.5 * b) * (inv * inv * inv)) / H
    dx = (dt * inv + dsq * (2 * rf)).to(torch.bfloat16)
    if dro is not None:
        dx = dx + dro
    t = (rf * inv).to(torch.bfloat16)
    dw = (dn * t).float().sum(0).to(torch.bfloat16)
    return dx, dw


@pytest.mark.parametrize("tag", CASES)
@pytest.mark.parametrize("ieee_rsqrt", [False, True])
def test_oracle_backward_matches_reference_autograd(tag, ieee_rsqrt):
    """Both forms of the oracle: the literal eager forward, and the one with an
    IEEE rsqrt (equal here wherever the CPU's rsqrt is correctly rounded)."""
    d = _load(tag)
    eager_rsqrt_ok = True
    if ieee_rsqrt:
        r = d["x"] + d["residual"] if "residual" in d else d["x"]
        v = r.float().square().mean(-1, keepdim=True) + d["eps"]
        ieee = (1.0 / torch.sqrt(v.double()).float().double()).float()
        eager_rsqrt_ok = torch.equal(torch.rsqrt(v), ieee)
    dx, dw, _, _ = ora.rms_norm_fp8_backward(
        d["x"], d["weight"], d["d_normalized"], d["eps"], residual=d.get("residual"),
        d_residual_out=d.get("d_residual_out"), scale_format=None, ieee_rsqrt=ieee_rsqrt)
    if not eager_rsqrt_ok:
        pytest.skip("this CPU's eager rsqrt is not correctly rounded on these rows")
    assert torch.equal(dx, d["dx"])
    assert torch.equal(dw, d["d_weight"])


@pytest.mark.parametrize("tag", CASES)
def test_closed_form_is_autograd(tag):
    d = _load(tag)
    dx, dw = closed_form(d["x"], d["weight"], d["d_normalized"], d["eps"], d.get("residual"),
                         d.get("d_residual_out"))
    assert torch.equal(dx, d["dx"])
    assert torch.equal(dw, d["d_weight"])
