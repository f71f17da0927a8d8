"""RMSNorm -> MXFP8 -> GEMM in one kernel (cutie_rms_norm_mxfp8_gemm).

The fused kernel must compute the composition of the path's own two steps:
A = the 1x32 e8m0 quantization of rms_norm_reference(x) (the oracle,
bench.py:58-65 + fp8_utils.py:50-57 with gran_k 32), then the block-scaled
GEMM of A with the weight B. The kernel splits K over the CTAs of a cluster
and adds their fp32 partial tiles in a fixed order, so D is the exact sum of
the products rounded by fp32 additions in another grouping than the
standalone GEMM's: D is held to the fp32-accumulation + bf16 bound around an
fp64 product of the dequantized operands, and must be bit-identical from run
to run. Checked:

* exact-sum inputs (x = k/16: the sum of squares is exact in any order, so
  inv_rms cannot depend on how the kernel splits rows or columns): the A it
  writes out equals the oracle's codes and swizzled scales bit for bit, and
  D is within the bound of the product of the oracle's A and B;
* random inputs (Student-t and normal, BASELINE config 4's shapes among
  them): A within the tolerance contract of the other forward tests (codes at
  most 1 e4m3 ulp apart on <= 0.1% of elements, e8m0 scales equal on >=
  99.9% of groups, swizzle padding zero), D within the bound of the product
  of that A and B, and within the same bound of what cutie_gemm_mxfp8
  computes from that A;
* D without the A outputs, and a second run, bit-identical to the first.

Shapes cover one and several 128-row blocks, rows past M inside a block,
decode batches (M = 1, 8, 32, 128 at K = N = 5120), a single K block, and
grids from one tile (8-way split) to more tiles than SMs (no split).
"""

import numpy as np
import pytest
import torch

from oracle import reference as ora
from parity import e4m3_ulp_diff

import thingy_b200 as tb
from thingy_b200 import _lib
from thingy_b200.gemm import mxfp8_gemm, rms_norm_mxfp8_gemm
from thingy_b200.layouts import mx_unswizzle, n_groups
from thingy_b200.ops import launch_rms_norm_fp8

pytestmark = pytest.mark.gpu


def _weight_operand(N, K, seed):
    """An e4m3 weight [N, K] with swizzled e8m0 scales, quantized by the path."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    qb = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=dev)
    sb = tb.empty_scale(N, K, 32, "e8m0", "mx", dev)
    launch_rms_norm_fp8(W, None, 0.0, q=qb, scale=sb, group_size=32, scale_format="e8m0",
                        scale_layout="mx", normalize=False)
    return qb, sb


def _inputs(M, K, seed, kind):
    g = torch.Generator().manual_seed(seed)
    if kind == "exact":
        x = torch.randint(-32, 33, (M, K), generator=g).float() / 16
    elif kind == "student_t":
        torch.manual_seed(seed)
        x = torch.distributions.StudentT(4.0).sample((M, K))
    else:
        x = torch.randn(M, K, generator=g)
    w = (1.0 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    return x.to(torch.bfloat16), w


def _fused(x, w, eps, qb, sb, with_a=True):
    M, K = x.shape
    dev = torch.device("cuda")
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev) if with_a else None
    s = tb.empty_scale(M, K, 32, "e8m0", "mx", dev) if with_a else None
    if with_a:
        s.view(torch.uint8).fill_(0xAB)  # every byte, padding included, must be written
    d = torch.full((M, qb.shape[0]), float("nan"), dtype=torch.bfloat16, device=dev)
    rms_norm_mxfp8_gemm(x.cuda(), w.cuda(), eps, qb, sb, out=d, q=q, q_scale=s, fused=True)
    torch.cuda.synchronize()
    return d, q, s


SHAPES = [
    # (M, N, K); K split = min(8, K / 128, 148 // tiles)
    (1, 128, 128),
    (77, 256, 2048),
    (200, 512, 1024),
    (128, 1024, 7168),
    (300, 2048, 4096),
    (8, 5120, 5120),
    (1000, 384, 1536),
    (2100, 1280, 512),
    (20, 2048, 3072),
    (1, 16384, 16384),
    # at most 16 rows with every K block of a CTA resident (A made in place of
    # x, one release for the MMAs), and 16 rows that are not resident
    (13, 1024, 2048),
    (16, 5120, 5120),
    (16, 128, 16384),
]


def _dequant(codes, scales, rows, K):
    e = torch.from_numpy(mx_unswizzle(scales.cpu().view(torch.uint8).numpy(), rows,
                                      n_groups(K, 32)))
    return codes.cpu().double() * torch.exp2(e.double() - 127.0).repeat_interleave(32, 1)[:, :K]


def _assert_product(d, A, B, K):
    """d within fp32 accumulation (any grouping) + bf16 rounding of A @ B.T."""
    ref = A @ B.t()
    bound = ref.abs() * 2.0 ** -8 + (A.abs() @ B.abs().t()) * ((K + 16) * 2.0 ** -23) + 1e-30
    err = (d.cpu().double() - ref).abs()
    assert bool((err <= bound).all()), f"max excess {(err - bound).max().item():.3e}"


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_exact_sum_inputs_bit_exact(M, N, K):
    x, w = _inputs(M, K, seed=M + N + K, kind="exact")
    qb, sb = _weight_operand(N, K, seed=N + K)
    d, q, s = _fused(x, w, 1e-6, qb, sb)
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(x, w, 1e-6, group_size=32, scale_format="e8m0")
    np.testing.assert_array_equal(q.cpu().view(torch.uint8).numpy(), q_ref.numpy())
    np.testing.assert_array_equal(s.cpu().view(torch.uint8).numpy(),
                                  ora.layout_scales(s_ref, "mx"))
    A = _dequant(q, s, M, K)
    _assert_product(d, A, _dequant(qb, sb, N, K), K)
    d2, _, _ = _fused(x, w, 1e-6, qb, sb)
    assert torch.equal(d2, d)  # run to run
    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("M,N,K,kind", [
    (1, 5120, 5120, "student_t"), (8, 5120, 5120, "student_t"), (32, 5120, 5120, "student_t"),
    (128, 5120, 5120, "student_t"), (777, 1024, 7168, "normal"), (256, 640, 2048, "normal"),
    (16, 5120, 5120, "student_t"), (3, 2048, 7168, "normal"),
])
def test_random_inputs_within_contract(M, N, K, kind):
    x, w = _inputs(M, K, seed=7 * M + K, kind=kind)
    qb, sb = _weight_operand(N, K, seed=K)
    d, q, s = _fused(x, w, 1e-6, qb, sb)
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(x, w, 1e-6, group_size=32, scale_format="e8m0")
    codes = q.cpu().view(torch.uint8).numpy()
    qd = e4m3_ulp_diff(codes, q_ref.numpy())
    assert qd.max(initial=0) <= 1
    assert (qd != 0).mean() <= 1e-3
    sm = mx_unswizzle(s.cpu().view(torch.uint8).numpy(), M, n_groups(K, 32))
    assert (sm != s_ref.numpy()).mean() <= 1e-3
    # the swizzle padding (rows past M) is zero
    full = s.cpu().view(torch.uint8).numpy()
    np.testing.assert_array_equal(full, ora.layout_scales(torch.from_numpy(sm), "mx"))
    # D is the GEMM of exactly that A (fp32 sums in some grouping)
    A, B = _dequant(q, s, M, K), _dequant(qb, sb, N, K)
    _assert_product(d, A, B, K)
    d_ref = mxfp8_gemm(q, s, qb, sb)
    torch.cuda.synchronize()
    _assert_product(d_ref, A, B, K)
    # and the same bits when A is not written out
    d2, _, _ = _fused(x, w, 1e-6, qb, sb, with_a=False)
    assert torch.equal(d2, d)
    assert _lib.device_error(clear=True) == 0


def test_argument_errors():
    qb, sb = _weight_operand(128, 256, seed=1)
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="multiples of 128"):
        rms_norm_mxfp8_gemm(x[:, :192].contiguous(), w[:192].contiguous(), 1e-6, qb[:, :192],
                            sb, fused=True)
    with pytest.raises(ValueError, match="together"):
        rms_norm_mxfp8_gemm(x, w, 1e-6, qb, sb, q=torch.empty(4, 256, dtype=torch.uint8,
                                                               device="cuda"), fused=True)
    out = rms_norm_mxfp8_gemm(x[:0], w, 1e-6, qb, sb, fused=True)
    assert out.shape == (0, 128)
    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("M", [8, 200])
def test_two_kernel_path_agrees(M):
    """fused=False (the default above FUSED_MAX_ROWS) gives the same A and a D within the bound."""
    N, K = 512, 2048
    x, w = _inputs(M, K, seed=M, kind="normal")
    qb, sb = _weight_operand(N, K, seed=3)
    d, q, s = _fused(x, w, 1e-6, qb, sb)
    q2 = torch.empty_like(q)
    s2 = tb.empty_scale(M, K, 32, "e8m0", "mx", "cuda")
    d2 = rms_norm_mxfp8_gemm(x.cuda(), w.cuda(), 1e-6, qb, sb, q=q2, q_scale=s2, fused=False)
    torch.cuda.synchronize()
    codes = e4m3_ulp_diff(q.cpu().view(torch.uint8).numpy(), q2.cpu().view(torch.uint8).numpy())
    assert codes.max(initial=0) <= 1 and (codes != 0).mean() <= 1e-3
    A2, B = _dequant(q2, s2, M, K), _dequant(qb, sb, N, K)
    _assert_product(d2, A2, B, K)
