"""The hand-written MXFP8 block-scaled GEMM (cutie_gemm_mxfp8) consuming this
path's output, against an fp32 GEMM of the dequantized operands and against
cuBLAS's MXFP8 GEMM on the same codes and scales.

A = the e4m3 codes of rms_norm_fp8(x, group_size=32, e8m0, swizzled) — the
path's own output, scales as written, M not a multiple of 128 included —
and B = a weight quantized by the same kernel (quantization only). D must
match sum_k dequant(A) dequant(B) within the rounding of fp32 accumulation
and the final bf16 cast, element by element.
"""

import pytest
import torch
import torch.nn.functional as F

import thingy_b200 as tb
from thingy_b200.gemm import mxfp8_gemm
from thingy_b200.layouts import mx_unswizzle, n_groups
from thingy_b200.ops import launch_rms_norm_fp8

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    x[:, torch.randperm(K, generator=g)[: max(1, K // 1000)]] *= 50.0
    w_norm = (1.0 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    qa, sa, _, _ = tb.rms_norm_fp8(x.to(torch.bfloat16).to(dev), w_norm.to(dev), 1e-6,
                                   group_size=32, scale_format="e8m0", scale_layout="mx")
    W = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    qb = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=dev)
    sb = tb.empty_scale(N, K, 32, "e8m0", "mx", dev)
    launch_rms_norm_fp8(W, None, 0.0, q=qb, scale=sb, group_size=32, scale_format="e8m0",
                        scale_layout="mx", normalize=False)
    return qa, sa, qb, sb


def _dequant(codes, scales, rows, K):
    e = torch.from_numpy(mx_unswizzle(scales.cpu().view(torch.uint8).numpy(), rows,
                                      n_groups(K, 32)))
    s = torch.exp2(e.double() - 127.0)
    return codes.cpu().double() * s.repeat_interleave(32, dim=1)[:, :K]


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 256, 512), (1000, 384, 7168),
                                   (77, 128, 2048), (2048, 1024, 4096),
                                   # enough tiles for 128 x 256 tiles
                                   (4800, 8192, 512), (4097, 9216, 384),
                                   # decode batches (<= 32 rows: swapped operands, K
                                   # split over 3 to 8 ranks, some K ranges uneven),
                                   # then the first M of the tiled kernel
                                   (1, 5120, 5120), (8, 1024, 2048), (32, 384, 7168),
                                   (17, 256, 512), (4, 128, 1024), (5, 5120, 7168),
                                   (2, 256, 384), (33, 256, 1024),
                                   # up to 128 rows when N leaves SMs idle: 128-row batch
                                   # boxes, 2-4 ranks
                                   (64, 5120, 5120), (100, 1024, 2048), (128, 384, 7168),
                                   (127, 7168, 1024)])
def test_mxfp8_gemm_matches_dequantized_product(M, N, K):
    qa, sa, qb, sb = _operands(M, N, K, seed=M + N + K)
    d = mxfp8_gemm(qa, sa, qb, sb)
    torch.cuda.synchronize()
    A, B = _dequant(qa, sa, M, K), _dequant(qb, sb, N, K)
    ref = A @ B.t()
    mag = A.abs() @ B.abs().t()
    # bf16 rounding of the result (half an ulp, 2^-9 relative) plus fp32
    # accumulation over K terms in any order
    bound = ref.abs() * 2.0 ** -8 + mag * (K * 2.0 ** -23) + 1e-30
    err = (d.cpu().double() - ref).abs()
    assert bool((err <= bound).all()), f"max excess {(err - bound).max().item():.3e}"


@pytest.mark.parametrize("M,N,K", [(256, 256, 1024), (1000, 512, 7168), (4736, 8192, 1024),
                                   (8, 5120, 5120), (32, 1024, 4096), (128, 5120, 5120)])
def test_mxfp8_gemm_matches_cublas(M, N, K):
    qa, sa, qb, sb = _operands(M, N, K, seed=7 * M + K)
    d = mxfp8_gemm(qa, sa, qb, sb)
    ref = F.scaled_mm(qa, qb.t(), sa, F.ScalingType.BlockWise1x32, sb, F.ScalingType.BlockWise1x32,
                      swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                      output_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    # both round an fp32 sum of exact products to bf16, in different orders (the
    # decode kernel splits K over ranks): a bf16 ulp of each rounding plus each
    # one's fp32 accumulation error, which cancellation can make large against
    # the result
    A, B = _dequant(qa, sa, M, K), _dequant(qb, sb, N, K)
    mag = (A.abs() @ B.abs().t()).float()
    diff = (d.float() - ref.float()).abs().cpu()
    ulp = torch.maximum(ref.float().abs(), d.float().abs()).cpu() * 2.0 ** -7
    assert bool((diff <= 2 * ulp + mag * (K * 2.0 ** -22) + 1e-30).all())


def test_mxfp8_gemm_empty_and_errors():
    qa, sa, qb, sb = _operands(128, 128, 256, seed=1)
    out = mxfp8_gemm(qa[:0], sa, qb, sb)
    assert out.shape == (0, 128)
    with pytest.raises(ValueError, match="multiples of 128"):
        mxfp8_gemm(qa, sa, qb[:64], sb)
    from thingy_b200 import _lib

    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("M,N,K", [(8, 5120, 5120), (32, 1024, 7168), (100, 5120, 5120)])
def test_mxfp8_gemm_decode_split_is_deterministic(M, N, K):
    """The split-K ranks are added in rank order: repeated calls agree bit for bit."""
    qa, sa, qb, sb = _operands(M, N, K, seed=3 * M + N)
    first = mxfp8_gemm(qa, sa, qb, sb)
    for _ in range(5):
        assert torch.equal(mxfp8_gemm(qa, sa, qb, sb), first)
