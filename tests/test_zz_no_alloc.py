"""The allocation-free backward entry point agrees with the regular one.

cutie_rms_norm_backward_noalloc serves callers that cannot allocate device
memory: code running where a cudaMalloc is not allowed or not wanted (for
example inside an allocator's own callbacks, in a plug-in whose host
framework owns all device memory, or where a memory pool must not grow). It
is the backward of the fused path with the per-CTA partial sums of d_weight
kept in the library's own fixed device array instead of a caller-provided
workspace.

These tests call it through the C ABI, twice in a row on one input set (the
second call runs on the array as the first call left it), over row widths
served by both backward kernels (H = 7168: the bulk-copy ring kernel, capped
at 146 CTAs; H = 32768: the direct kernel, capped at 32), with and without a
residual gradient and FP8 quantization, with no d_weight, and with no rows,
and compare each result with cutie_rms_norm_backward given a workspace: dx and its FP8 codes and scales
bit for bit (they do not depend on how d_weight is summed), d_weight within
the bound the backward's own tests use (the allocation-free call runs fewer
CTAs, so its partial sums are grouped differently). It lives in a file that
pytest collects last, and passes alone in a fresh process as well as after
every other test.
"""

import pytest
import torch

from thingy_b200 import _lib
from thingy_b200.ops import backward_workspace_bytes

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else t.data_ptr()


def _inputs(M, H, seed, residual):
    g = torch.Generator().manual_seed(seed)
    r = (torch.randn(M, H, generator=g) * 2).to(torch.bfloat16)
    dn = torch.randn(M, H, generator=g).to(torch.bfloat16)
    dro = torch.randn(M, H, generator=g).to(torch.bfloat16) if residual else None
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    d = dict(r=r, dn=dn, dro=dro, w=w)
    return {k: (None if v is None else v.cuda()) for k, v in d.items()}


def _outputs(M, H, quant, dw):
    dev = torch.device("cuda")
    return dict(dx=torch.full((M, H), float("nan"), dtype=torch.bfloat16, device=dev),
                dw=torch.full((H,), float("nan"), dtype=torch.bfloat16, device=dev) if dw else None,
                q=torch.empty(M, H, dtype=torch.uint8, device=dev) if quant else None,
                s=torch.empty(H // 128, M, dtype=torch.float32, device=dev) if quant else None)


def _call(lib, M, H, d, o, noalloc, ws=None):
    stream = torch.cuda.current_stream().cuda_stream
    quant = o["q"] is not None
    common_head = (_p(d["dn"]), H, _p(d["r"]), H, _p(d["w"]), _p(d["dro"]), H, 1e-6, M, H,
                   _p(o["dx"]), H, _p(o["dw"]))
    common_tail = (_lib.QUANT_GROUP if quant else _lib.QUANT_NONE, 128, _lib.SCALE_FP32,
                   _lib.LAYOUT_COL_MAJOR, M, _p(o["q"]), H, _p(o["s"]), stream)
    if noalloc:
        status = lib.cutie_rms_norm_backward_noalloc(*common_head, *common_tail)
    else:
        status = lib.cutie_rms_norm_backward(*common_head, _p(ws),
                                             0 if ws is None else ws.numel(), *common_tail)
    _lib.check(status)


def _dw_close(a, b, d, M):
    """Both d_weight results within the fp32-sum + bf16 bound of each other."""
    rf = d["r"].float()
    inv = torch.rsqrt(rf.square().mean(-1, keepdim=True) + 1e-6)
    p = (d["dn"] * (rf * inv).to(torch.bfloat16)).double()
    bound = 2 * (p.sum(0).abs() * 2.0 ** -8 + p.abs().sum(0) * (M + 8) * 2.0 ** -22)
    assert bool(((a.double() - b.double()).abs() <= bound).all())


CASES = [
    # (M, H, residual gradient, FP8 copy of dx, d_weight)
    (4096, 7168, True, True, True),
    (512, 32768, True, True, True),
    (1000, 7168, False, False, True),
    (3000, 7168, True, True, False),
    (0, 7168, True, True, True),
]


@pytest.mark.parametrize("M,H,residual,quant,dw", CASES)
def test_noalloc_backward_matches_workspace_backward_twice(M, H, residual, quant, dw):
    lib = _lib.load()
    ws = (torch.empty(max(1, backward_workspace_bytes(M, H)), dtype=torch.uint8, device="cuda")
          if dw else None)
    for seed in (0, 1):  # two calls in a row on the shared array
        d = _inputs(M, H, seed, residual)
        ref, got = _outputs(M, H, quant, dw), _outputs(M, H, quant, dw)
        _call(lib, M, H, d, ref, noalloc=False, ws=ws)
        _call(lib, M, H, d, got, noalloc=True)
        torch.cuda.synchronize()
        assert torch.equal(got["dx"], ref["dx"])
        if quant:
            assert torch.equal(got["q"], ref["q"])
            assert torch.equal(got["s"], ref["s"])
        if dw:
            assert not torch.isnan(got["dw"].float()).any()
            if M == 0:  # no rows: the gradient of the weight is zero
                assert torch.equal(got["dw"], torch.zeros_like(got["dw"]))
                assert torch.equal(ref["dw"], got["dw"])
            else:
                _dw_close(got["dw"].cpu(), ref["dw"].cpu(),
                          {k: (None if v is None else v.cpu()) for k, v in d.items()}, M)
