"""Bounded device waits that run out: device error 1, then a clean GPU.

Every wait the kernels make for their own bulk copies and row exchanges is
bounded (about 2 s of SM cycles by default), so a copy that never lands
cannot hang a kernel. cutie_set_wait_limit(-1) makes every wait that would
have to block give up at once. The copies themselves are valid and still
land: the kernel stops early, records code 1 in the device error word, lets
the copies it issued land, and returns. Each test then checks that word,
clears it, and runs the same launch again with the default limit on the same
stream, which must give the oracle's (or the earlier run's) bits exactly:
the failure left nothing behind on the GPU.
"""

import numpy as np
import pytest
import torch

from parity import check_parity, exact_sum_inputs

import thingy_b200 as tb
from thingy_b200 import _lib

pytestmark = pytest.mark.gpu


def _run_with_limit(fn, cycles):
    prev = _lib.set_wait_limit(cycles)
    try:
        fn()
    finally:
        _lib.set_wait_limit(prev)
    torch.cuda.synchronize()


@pytest.mark.parametrize(
    "kernel,M,H,group_size,fmt,layout,residual,threads",
    [
        ("pipelined", 4096, 7168, 128, "fp32", "col", False, 0),
        ("pipelined, residual, MXFP8", 2048, 5120, 32, "e8m0", "mx", True, 0),
        ("single-pass, per-token", 4096, 4096, None, "fp32", "row", True, 0),
        ("warp-per-row", 2048, 7168, 128, "fp32", "row", True, 32),
    ],
)
def test_forward_wait_runs_out_then_clean_launch(kernel, M, H, group_size, fmt, layout, residual,
                                                 threads):
    assert _lib.device_error(clear=True) == 0
    inp = exact_sum_inputs(M, H, residual=residual, seed=M + H)
    x, w = inp["x"].cuda(), inp["weight"].cuda()
    res = inp["residual"].cuda() if residual else None

    def launch():
        tb.rms_norm_fp8(x, w, inp["eps"], residual=res, group_size=group_size,
                        scale_format=fmt, scale_layout=layout, threads_per_row=threads)

    _run_with_limit(launch, -1)
    assert _lib.device_error(clear=True) == 1, f"{kernel}: no wait ran out"
    assert _lib.device_error(clear=False) == 0
    # the same launch with the default limit: bit-exact against the oracle
    check_parity(inp, group_size, fmt, layout, exact=True, threads=threads)
    assert _lib.device_error(clear=True) == 0


def test_backward_wait_runs_out_then_clean_launch():
    assert _lib.device_error(clear=True) == 0
    M, H = 4096, 7168
    g = torch.Generator().manual_seed(5)
    r = (2 * torch.randn(M, H, generator=g)).to(torch.bfloat16).cuda()
    dn = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    dro = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()

    def run():
        return tb.rms_norm_fp8_backward(dn, r, w, 1e-6, d_residual_out=dro, quantize=True,
                                        scale_layout="col")

    ref = run()
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    _run_with_limit(run, -1)
    assert _lib.device_error(clear=True) == 1, "no wait of the backward ran out"
    got = run()
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    for a, b in zip(ref, got):
        if a is None:
            assert b is None
            continue
        assert torch.equal(a.view(torch.uint8) if a.dtype == torch.float8_e4m3fn else a,
                           b.view(torch.uint8) if b.dtype == torch.float8_e4m3fn else b)


@pytest.mark.parametrize("M,N,K", [(8, 5120, 5120), (200, 512, 2048)])
def test_fused_gemm_wait_runs_out_then_clean_launch(M, N, K):
    """The fused RMSNorm -> MXFP8 -> GEMM kernel (thread-block clusters over K):
    with every wait giving up at once, each CTA still meets its cluster barriers,
    lets its own copies land and records code 1; the next launch is unaffected."""
    from thingy_b200.gemm import rms_norm_mxfp8_gemm
    from thingy_b200.ops import launch_rms_norm_fp8

    assert _lib.device_error(clear=True) == 0
    inp = exact_sum_inputs(M, K, residual=False, seed=M + K)
    x, w = inp["x"].cuda(), inp["weight"].cuda()
    g = torch.Generator().manual_seed(9)
    W = (0.05 * torch.randn(N, K, generator=g)).to(torch.bfloat16).cuda()
    qb = torch.empty(N, K, dtype=torch.float8_e4m3fn, device="cuda")
    sb = tb.empty_scale(N, K, 32, "e8m0", "mx", "cuda")
    launch_rms_norm_fp8(W, None, 0.0, q=qb, scale=sb, group_size=32, scale_format="e8m0",
                        scale_layout="mx", normalize=False)
    ref = rms_norm_mxfp8_gemm(x, w, 1e-6, qb, sb, fused=True)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    _run_with_limit(lambda: rms_norm_mxfp8_gemm(x, w, 1e-6, qb, sb, fused=True), -1)
    assert _lib.device_error(clear=True) == 1, "no wait of the fused GEMM ran out"
    got = rms_norm_mxfp8_gemm(x, w, 1e-6, qb, sb, fused=True)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert torch.equal(ref, got)
