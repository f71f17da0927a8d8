"""The codes and scales go straight into Blackwell's block-scaled FP8 GEMM.

The path writes its scales in the layouts the downstream GEMM reads, so the
output of one call is the A operand of the next GEMM with no copy or
transpose. These tests feed them to block-scaled GEMMs on sm_100 and compare
the product with an fp32 GEMM of the same operands dequantized on the CPU:

* MXFP8: 1x32 groups with e8m0 scales in the 128x4 swizzled layout, against
  a weight quantized by the same kernel (quantization without the norm),
  through torch's scaled_mm (cuBLAS);
* 1x128 activation groups with M-major fp32 scales ([M, K/128] with strides
  (1, M), the DeepSeek-V3 recipe) against 128x128 weight blocks, through
  flashinfer's groupwise GEMM when it is available (torch's scaled_mm takes
  this recipe on sm_90 only).

The GEMM is a library call used as a consumer, not part of this path; what
is checked is that the layouts agree, so the tolerance is the GEMM's own
(bf16 output, fp32 accumulation in another order).
"""

import pytest
import torch
import torch.nn.functional as F

import thingy_b200 as tb
from thingy_b200.layouts import mx_unswizzle, n_groups
from thingy_b200.ops import launch_rms_norm_fp8

pytestmark = pytest.mark.gpu

E8M0 = torch.float8_e8m0fnu


def _inputs(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    cols = torch.randperm(K, generator=g)[: max(1, K // 1000)]
    x[:, cols] *= 50.0
    w_norm = (1.0 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    return x.to(torch.bfloat16), w_norm


def _quantize_128x128(W):
    """Weight [N, K] -> e4m3 codes and fp32 scales per 128x128 block (amax / 448)."""
    N, K = W.shape
    Wb = W.float().reshape(N // 128, 128, K // 128, 128)
    s = (Wb.abs().amax(dim=(1, 3)) / 448.0).clamp_min(1e-4)  # [N/128, K/128]
    q = (Wb / s[:, None, :, None]).reshape(N, K).to(torch.float8_e4m3fn)
    return q, s


def _rel_err(out, ref):
    return ((out.float() - ref).norm() / ref.norm()).item()


def _groupwise_gemm_1x128():
    """A Blackwell GEMM taking 1x128 activation scales, or None.

    torch's scaled_mm (cuBLAS) takes the DeepSeek-style recipe on sm_90 only;
    flashinfer's groupwise FP8 GEMM (trtllm backend, prebuilt kernels) takes
    it on sm_100 when the package and its kernels are present.
    """
    try:
        from flashinfer.gemm import gemm_fp8_nt_groupwise
    except Exception:
        return None
    return gemm_fp8_nt_groupwise


@pytest.mark.parametrize("M,K,N", [(256, 7168, 512), (384, 4096, 256)])
def test_blockwise_1x128_scales_feed_the_gemm(M, K, N):
    gemm = _groupwise_gemm_1x128()
    if gemm is None:
        pytest.skip("no block-scaled GEMM with 1x128 activation scales for sm_100 here")
    dev = torch.device("cuda")
    x, w_norm = _inputs(M, K, seed=M + K)
    q, sa, _, _ = tb.rms_norm_fp8(x.to(dev), w_norm.to(dev), 1e-6, group_size=128,
                                  scale_format="fp32", scale_layout="col")
    assert sa.shape == (M, K // 128) and sa.stride() == (1, M)  # M-major, as the GEMM reads it

    g = torch.Generator().manual_seed(N)
    W = torch.randn(N, K, generator=g) * 0.05
    Wq, sw = _quantize_128x128(W)
    sb = sw.to(dev).t()  # [K/128, N/128], strides (1, K/128): contiguous along K
    try:
        out = gemm(q, Wq.to(dev), sa, sb, scale_major_mode=None, backend="trtllm")
    except Exception as e:  # the library could not build or load its kernel here
        pytest.skip(f"groupwise FP8 GEMM unavailable: {type(e).__name__}: {str(e)[:160]}")
    torch.cuda.synchronize()

    deq_a = q.cpu().float() * sa.cpu().repeat_interleave(128, dim=1)
    deq_w = Wq.float() * sw.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)
    ref = deq_a @ deq_w.t()
    assert _rel_err(out.cpu(), ref) < 1e-2
    # and the quantized product stays close to the unquantized one
    n_ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(
        torch.bfloat16).float() * w_norm.float()
    assert _rel_err(out.cpu(), n_ref @ W.t()) < 0.08


@pytest.mark.parametrize("M,K,N", [(128, 5120, 256), (200, 4096, 384)])
def test_mxfp8_swizzled_scales_feed_the_gemm(M, K, N):
    dev = torch.device("cuda")
    x, w_norm = _inputs(M, K, seed=3 * M + K)
    q, sa, _, _ = tb.rms_norm_fp8(x.to(dev), w_norm.to(dev), 1e-6, group_size=32,
                                  scale_format="e8m0", scale_layout="mx")
    g = torch.Generator().manual_seed(N + 1)
    W = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    Wq = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=dev)
    sw = tb.empty_scale(N, K, 32, "e8m0", "mx", dev)
    launch_rms_norm_fp8(W.to(dev), None, 0.0, q=Wq, scale=sw, group_size=32, scale_format="e8m0",
                        scale_layout="mx", normalize=False)
    assert sa.dtype == E8M0 and sw.dtype == E8M0

    out = F.scaled_mm(q, Wq.t(), sa, F.ScalingType.BlockWise1x32, sw, F.ScalingType.BlockWise1x32,
                      swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                      output_dtype=torch.bfloat16)
    torch.cuda.synchronize()

    G = n_groups(K, 32)

    def dequant(codes, scales, rows):
        e = torch.from_numpy(mx_unswizzle(scales.cpu().view(torch.uint8).numpy(), rows, G))
        s = torch.exp2(e.float() - 127.0)
        return codes.cpu().float() * s.repeat_interleave(32, dim=1)[:, :K]

    ref = dequant(q, sa, M) @ dequant(Wq, sw, N).t()
    assert _rel_err(out.cpu(), ref) < 1e-2
