"""Comparison helpers shared by the GPU parity tests (GPU output vs CPU oracle)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import reference as ora
from thingy_b200.layouts import mx_unswizzle, n_groups, unpack_ue8m0


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bf16_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two bit patterns (monotone ordering)."""

    def ordered(u):
        u = u.astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u)

    return np.abs(ordered(a) - ordered(b))


def e4m3_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in e4m3 codes (monotone ordering; +0 and -0 coincide)."""

    def ordered(c):
        c = c.astype(np.int32)
        return np.where(c & 0x80, -(c & 0x7F), c)

    return np.abs(ordered(a) - ordered(b))


def q_codes(q: torch.Tensor) -> np.ndarray:
    return q.detach().cpu().contiguous().view(torch.uint8).numpy()


def scale_matrix(s: torch.Tensor, M: int, H: int, group_size, fmt: str, layout: str) -> np.ndarray:
    """The GPU's scales as an [M, G] array (uint8 exponents for e8m0)."""
    G = n_groups(H, group_size)
    s = s.detach().cpu()
    if layout == "packed":  # int32 [M, W] view over [W, ld] words
        return unpack_ue8m0(s.reshape(M, -1).t().contiguous().numpy(), M, G)
    if fmt == "e8m0":
        s = s.view(torch.uint8)
    if layout == "mx":
        return mx_unswizzle(s.numpy(), M, G)
    if s.dim() == 1:
        return s.numpy().reshape(M, G)
    return s.contiguous().numpy().reshape(M, G)


def gpu_run(inp: dict, group_size, fmt: str, layout: str, *, normalized=True, threads=0,
            device="cuda"):
    import thingy_b200 as tb

    x = inp["x"].to(device)
    w = inp["weight"].to(device)
    res = inp.get("residual")
    res = None if res is None else res.to(device)
    q, s, r, n = tb.rms_norm_fp8(
        x, w, inp["eps"], residual=res, group_size=group_size, scale_format=fmt,
        scale_layout=layout, return_normalized=normalized, threads_per_row=threads,
    )
    torch.cuda.synchronize()
    return q, s, r, n


def check_parity(inp: dict, group_size, fmt: str, layout: str, *, exact: bool = False,
                 threads: int = 0, budget: float = 1e-3) -> dict:
    """Run GPU and oracle on the same inputs; assert the tolerance contract.

    residual_out: bit-exact. normalized: at most 2 bf16 ulps on <= budget of
    elements (fp32 sum order is the only difference: inv_rms moves by an fp32
    ulp, bf16(r * inv) by at most one bf16 ulp, and the bf16 weight product can
    turn that into two when it drops into the binade below). Quantization of the
    GPU's own normalized output: bit-exact (scales and codes). End to end:
    scales bit-exact wherever the group's normalized values agree, codes within
    1 e4m3 ulp on <= budget of elements. exact=True: everything bit-exact.

    Scales against the north-star tolerance (fp32 scales within 1e-6
    relative): ``scale_outside_1e6_frac`` is the fraction of (row, group)
    scales that differ from the oracle's by more than 1e-6 relative; it must
    stay within the same budget as the codes. Such a scale can only come from
    a group whose amax moved by a bf16 ulp (the fp32 sum order moved inv_rms),
    so each deviation of an fp32 scale is also bounded by two bf16 ulps of the
    amax (2^-6); a power-of-two scale that moves doubles or halves.
    """
    M, H = inp["x"].shape
    q, s, r, n = gpu_run(inp, group_size, fmt, layout, threads=threads)
    q_ref, s_ref, r_ref, n_ref = ora.rms_norm_fp8(
        inp["x"], inp["weight"], inp["eps"], residual=inp.get("residual"),
        group_size=group_size, scale_format=fmt,
    )
    stats = {}
    if r_ref is not None:
        np.testing.assert_array_equal(bf16_bits(r), bf16_bits(r_ref))
    nd = bf16_ulp_diff(bf16_bits(n), bf16_bits(n_ref))
    stats["normalized_diff_frac"] = float((nd != 0).mean()) if nd.size else 0.0
    if exact:
        assert nd.max(initial=0) == 0, "normalized differs on exact-sum inputs"
    else:
        assert nd.max(initial=0) <= 2
        assert stats["normalized_diff_frac"] <= budget
    # quantization stage, fed the GPU's own normalized values: bit-exact
    qc = q_codes(q)
    sm = scale_matrix(s, M, H, group_size, fmt, layout)
    q_own, s_own = ora.quantize(n.cpu(), group_size, fmt)
    np.testing.assert_array_equal(sm, s_own.numpy())
    np.testing.assert_array_equal(qc, q_own.numpy())
    if layout == "mx":  # the whole buffer, zero padding included
        np.testing.assert_array_equal(
            s.detach().cpu().view(torch.uint8).numpy(), ora.layout_scales(s_own, "mx")
        )
    if layout == "packed" and M > 0:  # whole words of the M rows, zero pad bytes included
        np.testing.assert_array_equal(
            s.detach().cpu().reshape(M, -1).t().numpy(), ora.layout_scales(s_own, "packed")[:, :M]
        )
    # end to end against the oracle
    gs = H if not group_size else group_size
    G = n_groups(H, group_size)
    pad = G * gs - H
    group_same = (np.pad(nd, ((0, 0), (0, pad))).reshape(M, G, gs) == 0).all(-1)
    sr = s_ref.numpy()
    np.testing.assert_array_equal(sm[group_same], sr[group_same])
    sv, rv = scale_values(sm, fmt), scale_values(sr, fmt)
    rel = np.abs(sv - rv) / rv
    stats["scale_outside_1e6_frac"] = float((rel > 1e-6).mean()) if rel.size else 0.0
    stats["scale_max_rel_diff"] = float(rel.max(initial=0.0))
    qd = e4m3_ulp_diff(qc, q_ref.numpy())
    stats["q_diff_frac"] = float((qd != 0).mean()) if qd.size else 0.0
    if exact:
        np.testing.assert_array_equal(sm, sr)
        assert qd.max(initial=0) == 0, "codes differ on exact-sum inputs"
    else:
        if fmt == "fp32":  # (a power-of-two scale moves by a factor of 2 when it moves)
            assert stats["scale_max_rel_diff"] <= 2.0**-6, "scale moved by more than two bf16 ulps"
        assert stats["scale_outside_1e6_frac"] <= budget, (
            f"{stats['scale_outside_1e6_frac']:.2e} of scales outside 1e-6 relative")
        assert qd.max(initial=0) <= 1
        assert stats["q_diff_frac"] <= budget
    return stats


def scale_values(s: np.ndarray, fmt: str) -> np.ndarray:
    """Scales as float64 values (e8m0 exponent bytes decoded to 2^(e - 127))."""
    if fmt == "e8m0":
        return np.ldexp(1.0, s.astype(np.int64) - 127)
    return s.astype(np.float64)


def exact_sum_inputs(M: int, H: int, *, residual: bool, seed: int = 0) -> dict:
    """Inputs whose fp32 sum of squares is exact in any order.

    x (and residual) are k/16 with small integers k, so every square is a
    multiple of 2^-8 and every partial sum over H <= 8192 elements stays below
    2^15: 23 significant bits, exact in fp32. Any summation order gives the
    oracle's bits, so every output can be compared bit for bit.
    """
    g = torch.Generator().manual_seed(seed)
    lim = 16 if residual else 32
    x = (torch.randint(-lim, lim + 1, (M, H), generator=g).float() / 16).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    out = {"x": x, "weight": w, "eps": 1e-6}
    if residual:
        out["residual"] = (torch.randint(-16, 17, (M, H), generator=g).float() / 16).to(torch.bfloat16)
    return out


def random_inputs(M: int, H: int, *, residual: bool, seed: int = 0, eps: float = 1e-6) -> dict:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    out = {"x": x, "weight": w, "eps": eps}
    if residual:
        out["residual"] = (2.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16)
    return out
