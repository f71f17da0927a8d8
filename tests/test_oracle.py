"""The CPU oracle against the reference's own outputs (tests/golden/).

The vectors were produced by the reference's functions themselves
(tests/golden/make_golden.py). residual_out, normalized and scales must match
bit for bit. FP8 codes must match bit for bit except where Triton's CPU
interpreter (which ran the reference's quantizer) mis-rounds, in three ways:
(a) when round to nearest carries into the next binade it returns the code
one binade below (half the value); (b) on an exact tie it rounds away from
zero instead of to the even code; (c) subnormal results are mis-rounded. On
the GPU the same kernel's cast is cvt.rn (ties to even), which the oracle
follows. Each mismatch is checked to be one of these cases, and at each one
the oracle's code must equal the OCP-spec encoding from oracle/e4m3.py.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import e4m3
from oracle import reference as ora

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_vectors.npz"


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def check_codes(q_oracle: np.ndarray, q_golden: np.ndarray, y: np.ndarray) -> int:
    """Equal codes except the interpreter's two rounding defects; returns their count."""
    diff = q_oracle != q_golden
    if not diff.any():
        return 0
    co, cg, yd = q_oracle[diff], q_golden[diff], y[diff].astype(np.float64)
    vo, vg = e4m3.decode(co), e4m3.decode(cg)
    # (a) binade carry: the correct code is a power of two reached by rounding up,
    #     the interpreter's is half of it
    carry = ((co & 0x07) == 0) & (vo == 2.0 * vg) & (np.abs(yd) < np.abs(vo))
    # (b) exact tie: y is the midpoint of two neighbouring codes; the oracle took
    #     the even one, the interpreter the odd one farther from zero
    tie = (
        (np.abs(yd) == (np.abs(vo) + np.abs(vg)) / 2)
        & ((co & 1) == 0)
        & ((cg & 0x7F) == (co & 0x7F) + 1)
        & ((co & 0x80) == (cg & 0x80))
    )
    # (c) subnormal outputs (|y| below the smallest normal, 2^-6) are mis-rounded
    subnormal = np.abs(yd) < 2.0**-6
    # wherever the interpreter deviates, the oracle must give the OCP-spec code
    np.testing.assert_array_equal(co, e4m3.encode_rne(yd))
    bad = ~(carry | tie | subnormal)
    assert not bad.any(), (
        f"{int(bad.sum())} code mismatches are neither interpreter defect: "
        f"y={yd[bad][:5]}, oracle={co[bad][:5]}, golden={cg[bad][:5]}"
    )
    return int(diff.sum())


def quant_inputs_y(n: torch.Tensor, scale: torch.Tensor, gs: int) -> np.ndarray:
    M, H = n.shape
    G = scale.shape[1]
    nf = torch.nn.functional.pad(n.float(), (0, G * gs - H)).view(M, G, gs)
    return (nf / scale[..., None]).view(M, G * gs)[:, :H].numpy()


def test_fused_residual_contract(golden):
    g = golden
    x, res, w = bf16(g["fused_res__x"]), bf16(g["fused_res__residual"]), bf16(g["fused_res__weight"])
    q, s, r, n = ora.rms_norm_fp8(x, w, float(g["fused_res__eps"]), residual=res)
    np.testing.assert_array_equal(bits16(r), g["fused_res__residual_out"])
    np.testing.assert_array_equal(bits16(n), g["fused_res__normalized"])
    np.testing.assert_array_equal(s.numpy(), g["fused_res__scale"])
    check_codes(q.numpy(), g["fused_res__q"], quant_inputs_y(n, s, 128))


def test_outlier_channels(golden):
    g = golden
    x, w = bf16(g["outliers__x"]), bf16(g["outliers__weight"])
    q, s, _, n = ora.rms_norm_fp8(x, w, float(g["outliers__eps"]))
    np.testing.assert_array_equal(bits16(n), g["outliers__normalized"])
    np.testing.assert_array_equal(s.numpy(), g["outliers__scale"])
    check_codes(q.numpy(), g["outliers__q"], quant_inputs_y(n, s, 128))


@pytest.mark.parametrize("tag,fmt", [("ragged_fp32", "fp32"), ("ragged_ue8m0", "ue8m0")])
def test_ragged_quantizer(golden, tag, fmt):
    x = bf16(golden[f"{tag}__x"])
    q, s = ora.quantize(x, 128, fmt)
    assert s.shape == (x.shape[0], 2)
    np.testing.assert_array_equal(s.numpy(), golden[f"{tag}__scale"])
    check_codes(q.numpy(), golden[f"{tag}__q"], quant_inputs_y(x, s, 128))


def test_pow2_scales(golden):
    g = golden
    n = bf16(g["ue8m0__normalized"])
    x, w = bf16(g["ue8m0__x"]), bf16(g["ue8m0__weight"])
    np.testing.assert_array_equal(bits16(ora.rms_norm_reference(x, w, 1e-6)), g["ue8m0__normalized"])
    q, s = ora.quantize(n, 128, "ue8m0")
    np.testing.assert_array_equal(s.numpy(), g["ue8m0__scale"])
    # power-of-two scales make n / s exact, so the codes carry no division rounding
    check_codes(q.numpy(), g["ue8m0__q"], quant_inputs_y(n, s, 128))


def test_edge_rows(golden):
    g = golden
    x, w = bf16(g["edge__x"]), bf16(g["edge__weight"])
    q, s, _, n = ora.rms_norm_fp8(x, w, float(g["edge__eps"]))
    np.testing.assert_array_equal(bits16(n), g["edge__normalized"])
    np.testing.assert_array_equal(s.numpy(), g["edge__scale"])
    assert s[0, 0].item() == np.float32(1e-4)  # all-zero row clamps to the minimum scale
    check_codes(q.numpy(), g["edge__q"], quant_inputs_y(n, s, 128))


def test_fp32_rms_norm(golden):
    g = golden
    x = torch.from_numpy(g["f32__x"])
    w = torch.from_numpy(g["f32__weight"])
    eps = float(g["f32__eps"])
    # the literal eager expression reproduces the reference's function exactly
    y = ora.rms_norm_f32(x, w, eps, ieee_sqrt=False)
    np.testing.assert_array_equal(y.numpy(), g["f32__out"])
    # the IEEE form differs only in rows whose eager sqrt is not correctly rounded
    y_ieee = ora.rms_norm_f32(x, w, eps)
    variance = x.pow(2).mean(dim=-1, keepdim=True) + eps
    sqrt_off = (torch.sqrt(variance) != torch.sqrt(variance.double()).float()).flatten()
    rows_differ = (y_ieee != y).any(-1)
    assert bool((rows_differ <= sqrt_off).all())


def test_torch_cpu_sqrt_is_not_always_ieee():
    """Why the fp32 oracle takes its square root in float64 (see rms_norm_f32)."""
    v = torch.tensor([1.360060214996338], dtype=torch.float32)
    assert torch.sqrt(v.double()).float().item() == np.float32(1.1662163)  # the IEEE root
    # eager torch may or may not agree depending on the CPU build; the oracle
    # must not depend on it: it divides by the correctly rounded root
    g = torch.Generator().manual_seed(9)
    x = torch.randn(64, 256, generator=g)
    w = torch.randn(256, generator=g)
    var = x.pow(2).mean(dim=-1, keepdim=True) + 1e-5
    assert torch.equal(ora.rms_norm_f32(x, w, 1e-5), x / torch.sqrt(var.double()).float() * w)


def test_pow2_ceil_matches_log2_form():
    """The bit-exact pow2 rule equals fp8_utils.py:53's exp2(ceil(log2 s)) on real scales."""
    gen = torch.Generator().manual_seed(3)
    amax = torch.randn(200000, generator=gen).abs().to(torch.bfloat16).float() * 20
    s = torch.clamp(amax / 448.0, min=1e-4)
    np.testing.assert_array_equal(ora.pow2_ceil(s).numpy(), torch.exp2(torch.ceil(torch.log2(s))).numpy())
    # every bf16 amax value, including exact powers of two and the clamp region
    allbf = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()
    s = torch.clamp(allbf / 448.0, min=1e-4)
    np.testing.assert_array_equal(ora.pow2_ceil(s).numpy(), torch.exp2(torch.ceil(torch.log2(s))).numpy())


def test_e8m0_bytes_are_pow2_exponents():
    gen = torch.Generator().manual_seed(4)
    n = torch.randn(8, 256, generator=gen).to(torch.bfloat16)
    _, s_pow2 = ora.quantize(n, 32, "ue8m0")
    q1, s_e8 = ora.quantize(n, 32, "e8m0")
    q2, _ = ora.quantize(n, 32, "ue8m0")
    np.testing.assert_array_equal(q1.numpy(), q2.numpy())
    np.testing.assert_array_equal(np.exp2(s_e8.numpy().astype(np.float64) - 127), s_pow2.numpy())


def test_per_token_is_one_group_per_row():
    gen = torch.Generator().manual_seed(5)
    n = torch.randn(4, 384, generator=gen).to(torch.bfloat16)
    q_tok, s_tok = ora.quantize(n, None, "fp32")
    q_grp, s_grp = ora.quantize(n, 384, "fp32")
    assert s_tok.shape == (4, 1)
    np.testing.assert_array_equal(q_tok.numpy(), q_grp.numpy())
    np.testing.assert_array_equal(s_tok.numpy(), s_grp.numpy())
