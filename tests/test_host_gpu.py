"""The host-buffer path (thingy_b200.host.rms_norm_fp8_host) against the oracle.

This is the path the benchmark's end-to-end number runs through: pinned host
x (and residual) in, q, scales (and residual_out) back in host memory, the
batch streamed in row chunks over three CUDA streams, the scales of the whole
batch written into one device buffer through per-chunk views of it (row
slices of the row-major, column-major and packed layouts; 128-row slabs of
the swizzled MX layout) and copied back once.

Every case uses exact-sum inputs, so each output must equal the CPU oracle's
bit for bit, and covers the chunk edges where a per-chunk view would go
wrong: a batch shorter than one chunk, a whole number of chunks, and a
ragged last chunk (37 rows) — for the MX layout also its zero padding rows.
"""

import numpy as np
import pytest
import torch

from oracle import reference as ora
from parity import bf16_bits, e4m3_ulp_diff, exact_sum_inputs, q_codes, scale_matrix

import thingy_b200 as tb
from thingy_b200.host import rms_norm_fp8_host
from thingy_b200.layouts import n_groups

pytestmark = pytest.mark.gpu

CHUNK = 256
MODES = [
    # (group_size, scale_format, scale_layout)
    (128, "fp32", "row"),
    (128, "fp32", "col"),
    (32, "e8m0", "mx"),
    (128, "e8m0", "packed"),
    (None, "fp32", "row"),
    (None, "fp32", "col"),
]


def _pinned_scale(M, H, group_size, fmt, layout):
    s = tb.empty_scale(M, H, group_size, fmt, layout, "cpu")
    if s.is_contiguous():
        return s.pin_memory()
    return s.t().contiguous().pin_memory().t()  # column-major / packed: [M, G] views


def _check(inp, group_size, fmt, layout, q, s, ro):
    M, H = inp["x"].shape
    q_ref, s_ref, r_ref, _ = ora.rms_norm_fp8(inp["x"], inp["weight"], inp["eps"],
                                              residual=inp.get("residual"),
                                              group_size=group_size, scale_format=fmt)
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())
    np.testing.assert_array_equal(scale_matrix(s, M, H, group_size, fmt, layout), s_ref.numpy())
    if layout == "mx":  # the whole swizzled buffer, zero padding rows and groups included
        np.testing.assert_array_equal(s.view(torch.uint8).numpy(), ora.layout_scales(s_ref, "mx"))
    if r_ref is not None:
        np.testing.assert_array_equal(bf16_bits(ro), bf16_bits(r_ref))


@pytest.mark.parametrize("group_size,fmt,layout", MODES)
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("M", [37, 3 * CHUNK, 2 * CHUNK + 37])
def test_host_path_matches_oracle(group_size, fmt, layout, residual, M):
    H = 2048
    inp = exact_sum_inputs(M, H, residual=residual, seed=M * 5 + H + (group_size or 0))
    w = inp["weight"].cuda()
    xh = inp["x"].pin_memory()
    rh = inp["residual"].pin_memory() if residual else None
    qh = torch.empty(M, H, dtype=torch.float8_e4m3fn).pin_memory()
    sh = _pinned_scale(M, H, group_size, fmt, layout)
    roh = torch.empty(M, H, dtype=torch.bfloat16).pin_memory() if residual else None
    rms_norm_fp8_host(xh, w, inp["eps"], residual=rh, out=qh, scale=sh, residual_out=roh,
                      group_size=group_size, scale_format=fmt, scale_layout=layout,
                      chunk_rows=CHUNK)
    torch.cuda.synchronize()
    _check(inp, group_size, fmt, layout, qh, sh, roh)


@pytest.mark.parametrize("group_size,fmt,layout", [(128, "fp32", "col"), (32, "e8m0", "mx")])
def test_host_pipeline_reuse(group_size, fmt, layout):
    """The returned pipeline reused for a second batch (new inputs, same shape)
    and a third of another length: its buffers and cached scale slab must not
    carry anything over."""
    H = 2048
    pipe = None
    for M, seed in ((2 * CHUNK + 37, 1), (2 * CHUNK + 37, 2), (CHUNK + 5, 3)):
        inp = exact_sum_inputs(M, H, residual=True, seed=seed)
        xh, rh = inp["x"].pin_memory(), inp["residual"].pin_memory()
        qh = torch.empty(M, H, dtype=torch.float8_e4m3fn).pin_memory()
        sh = _pinned_scale(M, H, group_size, fmt, layout)
        roh = torch.empty(M, H, dtype=torch.bfloat16).pin_memory()
        pipe = rms_norm_fp8_host(xh, inp["weight"].cuda(), inp["eps"], residual=rh, out=qh,
                                 scale=sh, residual_out=roh, group_size=group_size,
                                 scale_format=fmt, scale_layout=layout, pipeline=pipe,
                                 chunk_rows=CHUNK)
        torch.cuda.synchronize()
        _check(inp, group_size, fmt, layout, qh, sh, roh)


def test_host_path_random_inputs_within_the_tolerance_contract():
    """Random inputs at the DeepSeek-V3 width, more rows than the row-staged
    kernel's threshold: the host path's 2048-row chunks run other kernels
    than one device launch of the whole batch (another summation order), so
    each is held to the oracle under the parity contract: codes within one
    e4m3 ulp on <= 0.1% of elements, scales outside 1e-6 relative on <= 0.1%
    of groups, each within two bf16 ulps of the amax."""
    M, H = 2 * 2048 + 37, 7168
    g = torch.Generator().manual_seed(9)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    wt = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(x, wt, 1e-6, group_size=128)
    w = wt.cuda()
    q_d, s_d, _, _ = tb.rms_norm_fp8(x.cuda(), w, 1e-6, group_size=128, scale_layout="col")
    qh = torch.empty(M, H, dtype=torch.float8_e4m3fn).pin_memory()
    sh = _pinned_scale(M, H, 128, "fp32", "col")
    rms_norm_fp8_host(x.pin_memory(), w, 1e-6, out=qh, scale=sh, group_size=128,
                      scale_layout="col")
    torch.cuda.synchronize()
    for q, s in ((qh, sh), (q_d.cpu(), s_d.cpu())):
        qd = e4m3_ulp_diff(q_codes(q), q_ref.numpy())
        assert qd.max() <= 1 and (qd != 0).mean() <= 1e-3
        rel = (s.double() - s_ref.double()).abs() / s_ref.double()
        assert float((rel > 1e-6).double().mean()) <= 1e-3 and float(rel.max()) <= 2.0 ** -6
    assert n_groups(H, 128) == sh.shape[1]
