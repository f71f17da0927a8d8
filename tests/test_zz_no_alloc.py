"""The allocation-free backward entry point agrees with the regular one.

cutie_rms_norm_backward_noalloc serves callers that cannot allocate device
memory: code running where a cudaMalloc is not allowed or not wanted (for
example inside an allocator's own callbacks, in a plug-in whose host
framework owns all device memory, or where a memory pool must not grow). It
is the backward of the fused path with the per-CTA partial sums of d_weight
kept in the library's own fixed device array instead of a caller-provided
workspace.

This test calls it through the C ABI twice in a row (the second call runs
on the array as the first call left it) and compares each result with
cutie_rms_norm_backward given a workspace: dx and its FP8 codes and scales
bit for bit (they do not depend on how d_weight is summed), d_weight within
the bound the backward's own tests use (the allocation-free call runs fewer
CTAs, so its partial sums are grouped differently). It lives in a file that
pytest collects last, and passes alone in a fresh process as well as after
every other test.
"""

import ctypes

import pytest
import torch

from thingy_b200 import _lib
from thingy_b200.ops import backward_workspace_bytes

pytestmark = pytest.mark.gpu

M, H = 4096, 7168


def _p(t):
    return None if t is None else t.data_ptr()


def _inputs(seed):
    g = torch.Generator().manual_seed(seed)
    r = (torch.randn(M, H, generator=g) * 2).to(torch.bfloat16)
    dn = torch.randn(M, H, generator=g).to(torch.bfloat16)
    dro = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    return {k: v.cuda() for k, v in dict(r=r, dn=dn, dro=dro, w=w).items()}


def _outputs():
    dev = torch.device("cuda")
    return dict(dx=torch.empty(M, H, dtype=torch.bfloat16, device=dev),
                dw=torch.empty(H, dtype=torch.bfloat16, device=dev),
                q=torch.empty(M, H, dtype=torch.uint8, device=dev),
                s=torch.empty(H // 128, M, dtype=torch.float32, device=dev))


def _call(lib, d, o, noalloc, ws=None):
    stream = torch.cuda.current_stream().cuda_stream
    common_head = (_p(d["dn"]), H, _p(d["r"]), H, _p(d["w"]), _p(d["dro"]), H, 1e-6, M, H,
                   _p(o["dx"]), H, _p(o["dw"]))
    common_tail = (_lib.QUANT_GROUP, 128, _lib.SCALE_FP32, _lib.LAYOUT_COL_MAJOR, M,
                   _p(o["q"]), H, _p(o["s"]), stream)
    if noalloc:
        status = lib.cutie_rms_norm_backward_noalloc(*common_head, *common_tail)
    else:
        status = lib.cutie_rms_norm_backward(*common_head, _p(ws), ws.numel(), *common_tail)
    _lib.check(status)


def _dw_close(a, b, d):
    """Both d_weight results within the fp32-sum + bf16 bound of each other."""
    rf = d["r"].float()
    inv = torch.rsqrt(rf.square().mean(-1, keepdim=True) + 1e-6)
    p = (d["dn"] * (rf * inv).to(torch.bfloat16)).double()
    bound = 2 * (p.sum(0).abs() * 2.0 ** -8 + p.abs().sum(0) * (M + 8) * 2.0 ** -22)
    assert bool(((a.double() - b.double()).abs() <= bound).all())


def test_noalloc_backward_matches_workspace_backward_twice():
    lib = _lib.load()
    ws = torch.empty(backward_workspace_bytes(M, H), dtype=torch.uint8, device="cuda")
    for seed in (0, 1):  # two calls in a row on the shared array
        d = _inputs(seed)
        ref, got = _outputs(), _outputs()
        _call(lib, d, ref, noalloc=False, ws=ws)
        _call(lib, d, got, noalloc=True)
        torch.cuda.synchronize()
        assert torch.equal(got["dx"], ref["dx"])
        assert torch.equal(got["q"], ref["q"])
        assert torch.equal(got["s"], ref["s"])
        _dw_close(got["dw"].cpu(), ref["dw"].cpu(), {k: v.cpu() for k, v in d.items()})
