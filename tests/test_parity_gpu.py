"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle.

Tolerance contract (see parity.check_parity): residual_out bit-exact; codes
and scales bit-exact given the same normalized values; end to end at most
1 e4m3 ulp on <= 0.1% of codes where only the fp32 summation order differs;
fully bit-exact on inputs whose sum of squares is exact in any order.
"""

import numpy as np
import pytest
import torch

from oracle import reference as ora
from parity import (
    bf16_bits,
    bf16_ulp_diff,
    check_parity,
    e4m3_ulp_diff,
    exact_sum_inputs,
    q_codes,
    random_inputs,
    scale_matrix,
)

import thingy_b200 as tb
from thingy_b200.workloads import DECODE_ROWS, WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

MODES = [
    # (group_size, scale_format, scale_layout)
    (None, "fp32", "row"),
    (None, "fp32", "col"),
    (None, "ue8m0", "row"),
    (128, "fp32", "row"),
    (128, "fp32", "col"),
    (128, "ue8m0", "row"),
    (128, "e8m0", "row"),
    (64, "fp32", "row"),
    (32, "e8m0", "mx"),
    (32, "e8m0", "row"),
    (32, "fp32", "col"),
    (128, "e8m0", "packed"),
    (32, "e8m0", "packed"),
]


@pytest.mark.parametrize("group_size,fmt,layout", MODES)
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("M,H", [(1, 1024), (37, 7168), (130, 8192), (64, 4096), (9, 5120)])
def test_exact_sum_bitexact(group_size, fmt, layout, residual, M, H):
    inp = exact_sum_inputs(M, H, residual=residual, seed=M + H)
    check_parity(inp, group_size, fmt, layout, exact=True)


@pytest.mark.parametrize("group_size,fmt,layout", MODES)
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("M,H", [(1000, 7168), (5000, 1024), (700, 8192), (2000, 5120), (1999, 4096)])
def test_bulk_path_bitexact(group_size, fmt, layout, residual, M, H):
    """Batches of >= 4 rows per SM go through the bulk-copy ring (many rows per
    CTA, every stage reused several times, swizzle padding rows at the end)."""
    inp = exact_sum_inputs(M, H, residual=residual, seed=M * 7 + H)
    check_parity(inp, group_size, fmt, layout, exact=True)


ROWSTAGE_MODES = [
    (None, "fp32", "row"), (None, "ue8m0", "col"), (128, "fp32", "col"), (128, "ue8m0", "row"),
    (128, "e8m0", "row"), (128, "e8m0", "packed"), (128, "e8m0", "mx"),
]


@pytest.mark.parametrize("group_size,fmt,layout", ROWSTAGE_MODES)
@pytest.mark.parametrize("M,H", [(4096, 1000), (4100, 8184), (4500, 7168), (4097, 2056),
                                 (4099, 5120)])
def test_row_staged_bitexact(group_size, fmt, layout, M, H):
    """Residual-free batches of >= 4096 rows up to 8192 columns go to the
    row-staged kernel (one warp a row, the row held in registers) for 1x128
    groups and per-token scales, every scale destination: row widths from
    one 2 KB block to eight, whole and ragged last blocks, rows not a
    multiple of the warps."""
    inp = exact_sum_inputs(M, H, residual=False, seed=M * 11 + H)
    check_parity(inp, group_size, fmt, layout, exact=True)


@pytest.mark.parametrize("M,H", [(4096, 4096), (4111, 1032), (5000, 8192)])
def test_row_staged_plain_rmsnorm(M, H):
    """The row-staged kernel's no-quantization mode (bf16 RMSNorm output)."""
    inp = exact_sum_inputs(M, H, residual=False, seed=M + 3 * H)
    y = tb.rms_norm(inp["x"].cuda(), inp["weight"].cuda(), 1e-6)
    ref = ora.rms_norm_reference(inp["x"], inp["weight"], 1e-6)
    np.testing.assert_array_equal(bf16_bits(y), bf16_bits(ref))


@pytest.mark.parametrize("group_size,fmt,layout", MODES)
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("M,H", [(3, 7168), (41, 8192), (70, 1000), (9, 200), (5, 16384),
                                 (4, 24576)])
def test_warp_per_row_bitexact(group_size, fmt, layout, residual, M, H):
    """The two-pass warp-per-row kernel (threads_per_row=32): full rows, ragged
    rows (H % 32 != 0, partial chunks) and rows of more than 32 chunks per lane."""
    inp = (exact_sum_inputs(M, H, residual=residual, seed=M * 3 + H) if H <= 8192 else
           random_inputs(M, H, residual=residual, seed=M * 3 + H))
    check_parity(inp, group_size, fmt, layout, exact=H <= 8192, threads=32)


@pytest.mark.parametrize("group_size,fmt,layout", MODES)
@pytest.mark.parametrize("residual", [False, True])
def test_random_parity(group_size, fmt, layout, residual):
    inp = random_inputs(512, 7168, residual=residual, seed=7)
    check_parity(inp, group_size, fmt, layout)


@pytest.mark.parametrize("M,H", [(64, 4096), (300, 7168), (40, 1000)])
def test_residual_add_extremes(M, H):
    """bf16 + bf16 residual sums at the edges of the format: ties at bf16
    precision, exponent gaps of 16+ bits, subnormal operands and sums, exact
    cancellation. The kernels add bf16 pairs in one rounding; the reference
    adds in fp32 and rounds to bf16; the two agree on every bf16 pair."""
    g = torch.Generator().manual_seed(M + H)
    sign = lambda *shape: torch.where(torch.rand(*shape, generator=g) < 0.5, -1.0, 1.0)
    x = torch.randn(M, H, generator=g)
    r = torch.randn(M, H, generator=g) * 2.0
    c = torch.randint(0, 5, (M, H), generator=g)
    one = sign(M, H) * 2.0 ** torch.randint(-10, 10, (M, H), generator=g).float()
    ties = one * (1.0 + 2.0 ** -8 * torch.randint(1, 4, (M, H), generator=g).float())
    x = torch.where(c == 0, one, x)
    r = torch.where(c == 0, ties - one, r)  # x + r lands on or near a bf16 tie
    tiny = sign(M, H) * 2.0 ** -133 * torch.randint(1, 127, (M, H), generator=g).float()
    x = torch.where(c == 1, x * 2.0 ** 20, x)
    r = torch.where(c == 1, tiny, r)  # exponent gap of 16+ bits
    x = torch.where(c == 2, tiny, x)
    r = torch.where(c == 2, -tiny * 0.5, r)  # subnormal operands and sums
    r = torch.where(c == 3, -x, r)  # exact cancellation
    inp = {
        "x": x.to(torch.bfloat16),
        "residual": r.to(torch.bfloat16),
        "weight": (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16),
        "eps": 1e-6,
    }
    assert (inp["residual"].float().abs() < 2.0 ** -126).any(), "no subnormal operands"
    for gs, fmt, layout in [(128, "fp32", "col"), (32, "e8m0", "mx"), (None, "fp32", "row")]:
        check_parity(inp, gs, fmt, layout)


@pytest.mark.parametrize("H", [8, 16, 24, 200, 1000, 2048, 3072, 6144, 12288, 16384, 32768])
def test_widths(H):
    """Every vectors-per-thread instantiation and ragged last groups."""
    inp = exact_sum_inputs(33, H, residual=True, seed=H) if H <= 8192 else random_inputs(
        33, H, residual=True, seed=H)
    for gs, fmt, layout in [(None, "fp32", "row"), (128, "fp32", "col"), (32, "e8m0", "mx")]:
        check_parity(inp, gs, fmt, layout, exact=H <= 8192)


@pytest.mark.parametrize("threads", [32, 64, 128, 224, 256, 512, 1024])
def test_threads_per_row(threads):
    """32 selects the warp-per-row kernel; larger CTAs the single-pass kernel."""
    inp = exact_sum_inputs(300, 7168, residual=True, seed=11)
    chunks = 7168 // 32  # 64-byte chunks per row
    per_thread = -(-chunks // threads)
    if threads > 32 and (per_thread > 2 or (per_thread == 2 and threads > 512)):
        with pytest.raises(ValueError):
            check_parity(inp, 128, "fp32", "row", exact=True, threads=threads)
        return
    check_parity(inp, 128, "fp32", "row", exact=True, threads=threads)


def test_golden_vectors_on_gpu():
    """The reference's own golden inputs through the GPU path (oracle-pinned outputs)."""
    from pathlib import Path

    g = dict(np.load(Path(__file__).resolve().parent / "golden" / "reference_vectors.npz"))

    def bf(a):
        return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)

    inp = {"x": bf(g["fused_res__x"]), "residual": bf(g["fused_res__residual"]),
           "weight": bf(g["fused_res__weight"]), "eps": float(g["fused_res__eps"])}
    q, s, r, n = tb.residual_rms_norm_fp8(
        inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda(), inp["eps"])
    np.testing.assert_array_equal(bf16_bits(r), g["fused_res__residual_out"])
    nd = bf16_ulp_diff(bf16_bits(n), g["fused_res__normalized"])
    assert nd.max() <= 2 and (nd != 0).mean() <= 1e-3
    if nd.max() == 0:
        np.testing.assert_array_equal(s.cpu().numpy(), g["fused_res__scale"])
    check_parity(inp, 128, "fp32", "row")


@pytest.mark.parametrize("name", ["token_4096x4096", "g128_16384x7168", "residual_token_32768x8192"])
def test_workload_full_size(name):
    w = WORKLOADS[name]
    inp = make_inputs(w, device="cpu", seed=0)
    stats = check_parity(inp, w.group_size, w.scale_format, w.scale_layout)
    print(name, stats)


@pytest.mark.parametrize("M", DECODE_ROWS)
def test_decode_mxfp8(M):
    w = WORKLOADS["mx32_decode_5120"]
    inp = make_inputs(w, M, device="cpu", seed=M)
    stats = check_parity(inp, 32, "e8m0", "mx")
    print(f"mx32_decode_5120 M={M}", stats)


def test_sharded_workload_rows_independent():
    """Config 5 at full size: row shards computed separately equal the slices of one launch."""
    w = WORKLOADS["g128_sharded_262144x8192"]
    inp = make_inputs(w, device="cuda", seed=0)
    x, wt = inp["x"], inp["weight"]
    M, H = x.shape
    q, s, _, _ = tb.rms_norm_fp8(x, wt, w.eps, group_size=128, scale_layout="col")
    from thingy_b200.shard import all_shards

    for sh in all_shards(M, 8):
        qs, ss, _, _ = tb.rms_norm_fp8(x[sh.start:sh.stop], wt, w.eps, group_size=128,
                                       scale_layout="col")
        assert torch.equal(qs.view(torch.uint8), q[sh.start:sh.stop].view(torch.uint8))
        assert torch.equal(ss, s[sh.start:sh.stop])
    # sampled rows against the oracle
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:256].sort().values
    sub = {"x": x[rows.cuda()].cpu(), "weight": wt.cpu(), "eps": w.eps}
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(sub["x"], sub["weight"], w.eps, group_size=128)
    qd = e4m3_ulp_diff(q_codes(q[rows.cuda()]), q_ref.numpy())
    assert qd.max() <= 1 and (qd != 0).mean() <= 1e-3
    sv, rv = s[rows.cuda()].cpu().double().numpy(), s_ref.double().numpy()
    rel = np.abs(sv - rv) / rv
    outside = float((rel > 1e-6).mean())
    print("g128_sharded_262144x8192 sampled rows", {"q_diff_frac": float((qd != 0).mean()),
          "scale_outside_1e6_frac": outside, "scale_max_rel_diff": float(rel.max())})
    assert outside <= 1e-3 and rel.max() <= 2.0**-6
    # dequantisation bound on the whole tensor: |q*s| <= 448*s and s >= 1e-4
    assert bool((s >= 1e-4).all())
    torch.cuda.synchronize()


def test_quantizer_exhaustive_amax():
    """Every positive finite bf16 value as a group amax: scales and codes bit-exact."""
    amax = torch.arange(1, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    n = amax.numel()
    G = 32
    rows = -(-n // 128)
    g = torch.Generator().manual_seed(1)
    frac = torch.rand(rows * 128, G, generator=g) * 2 - 1
    am = torch.cat([amax, torch.ones(rows * 128 - n, dtype=torch.bfloat16)]).float()
    x = (frac * am[:, None]).to(torch.bfloat16)
    x[:, 0] = am.to(torch.bfloat16)
    x = x.view(rows, 128 * G)
    for fmt in ("fp32", "ue8m0"):
        q, s = tb.per_token_cast_to_fp8(x.cuda(), use_ue8m0=(fmt == "ue8m0"), gran_k=G)
        q_ref, s_ref = ora.quantize(x, G, fmt)
        np.testing.assert_array_equal(s.cpu().numpy(), s_ref.numpy())
        np.testing.assert_array_equal(q_codes(q), q_ref.numpy())


@pytest.mark.parametrize("use_ue8m0", [False, True])
@pytest.mark.parametrize("M,H", [(8, 200), (5, 128), (64, 7168), (3, 4104)])
def test_per_token_cast_to_fp8(use_ue8m0, M, H):
    g = torch.Generator().manual_seed(H)
    x = (3 * torch.randn(M, H, generator=g)).to(torch.bfloat16)
    q, s = tb.per_token_cast_to_fp8_triton(x.cuda(), use_ue8m0)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (M, -(-H // 128))
    q_ref, s_ref = ora.quantize(x, 128, "ue8m0" if use_ue8m0 else "fp32")
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref.numpy())
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())


@pytest.mark.parametrize("M,H", [(1, 4096), (513, 1024), (64, 7168), (16, 16384)])
def test_rms_norm_fp32(M, H):
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, H, generator=g)
    w = torch.randn(H, generator=g)
    y = tb.rms_norm(x.cuda(), w.cuda(), 1e-5).cpu()
    ref = ora.rms_norm_f32(x, w, 1e-5)
    torch.testing.assert_close(y, ref, rtol=2e-6, atol=1e-30)
    # exact-sum fp32 inputs (k/16): bit-exact
    xe = (torch.randint(-32, 33, (M, H), generator=g).float() / 16)
    ye = tb.rms_norm(xe.cuda(), w.cuda(), 1e-5).cpu()
    assert torch.equal(ye, ora.rms_norm_f32(xe, w, 1e-5))


def test_rms_norm_bf16_matches_prime_rl_form():
    inp = exact_sum_inputs(77, 4096, residual=False, seed=3)
    y = tb.rms_norm(inp["x"].cuda(), inp["weight"].cuda(), 1e-6)
    ref = ora.rms_norm_reference(inp["x"], inp["weight"], 1e-6)
    np.testing.assert_array_equal(bf16_bits(y), bf16_bits(ref))


def test_rmsnorm_class_destination_passing_and_nan_prefill():
    """The reference's call form; NaN-prefilled outputs are fully overwritten."""
    inp = random_inputs(96, 3072, residual=True, seed=5)
    x, res, w = inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda()
    M, H = x.shape
    out = torch.full((M, H), float("nan"), device="cuda").to(torch.float8_e4m3fn)
    scale = torch.full((M, H // 128), float("nan"), device="cuda")
    residual_out = torch.full_like(x, float("nan"))
    normalized_out = torch.full_like(x, float("nan"))
    norm = tb.RMSNorm(elements_per_thread=8, threads_per_row=128, load_path="shared", reduction="all")
    ret = norm(x, res, w, 1e-6, out, scale, residual_out, normalized_out)
    torch.cuda.synchronize()
    assert ret is None
    for t in (out.float(), scale, residual_out.float(), normalized_out.float()):
        assert not torch.isnan(t).any()
    q2, s2, r2, n2 = tb.residual_rms_norm_fp8(x, res, w, 1e-6)
    assert torch.equal(out.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(scale, s2) and torch.equal(residual_out, r2) and torch.equal(normalized_out, n2)


def test_strided_rows_and_padding_untouched():
    """Leading dimensions larger than H; bytes between rows are never written."""
    inp = exact_sum_inputs(50, 1024, residual=True, seed=9)
    big_x = torch.zeros(50, 1536, dtype=torch.bfloat16, device="cuda")
    big_r = torch.zeros(50, 1280, dtype=torch.bfloat16, device="cuda")
    big_x[:, :1024] = inp["x"].cuda()
    big_r[:, :1024] = inp["residual"].cuda()
    qbuf = torch.full((50, 1104), 0x5A, dtype=torch.uint8, device="cuda")
    rbuf = torch.full((50, 1040), 7.0, dtype=torch.bfloat16, device="cuda")
    sbuf = torch.full((8, 64), -1.0, device="cuda")  # column-major, ld 64 >= M
    tb.rms_norm_fp8(big_x[:, :1024], inp["weight"].cuda(), 1e-6, residual=big_r[:, :1024],
                    out=qbuf[:, :1024], scale=sbuf[:, :50].t(), residual_out=rbuf[:, :1024],
                    scale_layout="col")
    torch.cuda.synchronize()
    q_ref, s_ref, r_ref, _ = ora.rms_norm_fp8(inp["x"], inp["weight"], 1e-6,
                                              residual=inp["residual"])
    np.testing.assert_array_equal(qbuf[:, :1024].cpu().numpy(), q_ref.numpy())
    np.testing.assert_array_equal(sbuf[:, :50].cpu().numpy(), s_ref.numpy().T)
    np.testing.assert_array_equal(bf16_bits(rbuf[:, :1024]), bf16_bits(r_ref))
    assert bool((qbuf[:, 1024:] == 0x5A).all())
    assert bool((rbuf[:, 1024:] == 7.0).all())
    assert bool((sbuf[:, 50:] == -1.0).all())


@pytest.mark.parametrize("M", [64, 4096])
def test_in_place_residual_update(M):
    """residual_out may alias residual (the residual stream updated in place),
    also for batches large enough to prefer the two-pass kernel (which the
    library then avoids, since it re-reads its inputs)."""
    inp = exact_sum_inputs(M, 2048, residual=True, seed=13)
    x, res, w = inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda()
    q, s, _, _ = tb.rms_norm_fp8(x, w, 1e-6, residual=res, residual_out=res)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(res), bf16_bits(inp["x"] + inp["residual"]))
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(inp["x"], inp["weight"], 1e-6, residual=inp["residual"])
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())
    with pytest.raises(ValueError):  # the two-pass kernel refuses aliasing outright
        tb.rms_norm_fp8(x, w, 1e-6, residual=res, residual_out=res, threads_per_row=32)


def test_empty_batch_and_mx_padding():
    x = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
    q, s, _, _ = tb.rms_norm_fp8(x, w, group_size=32, scale_format="e8m0", scale_layout="mx")
    assert q.shape == (0, 1024) and s.numel() == 0
    # M=3 with a 36-group row: padded to 128 x 36, every padding byte zero
    inp = exact_sum_inputs(3, 1152, residual=False, seed=2)
    q, s, _, _ = tb.rms_norm_fp8(inp["x"].cuda(), inp["weight"].cuda(), 1e-6, group_size=32,
                                 scale_format="e8m0", scale_layout="mx")
    buf = s.cpu().view(torch.uint8).numpy()
    assert buf.size == 128 * 36
    sm = scale_matrix(s, 3, 1152, 32, "e8m0", "mx")
    assert buf.sum() == sm.astype(np.int64).sum()  # everything else is zero


def test_argument_errors():
    x = torch.zeros(4, 1024, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
    wide = torch.zeros(4, 1032, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        tb.rms_norm_fp8(wide[:, 4:1028], w, group_size=128)  # rows start 8 bytes off
    with pytest.raises(ValueError):
        tb.rms_norm_fp8(torch.zeros(4, 1020, dtype=torch.bfloat16, device="cuda"),
                        torch.ones(1020, dtype=torch.bfloat16, device="cuda"))  # H % 8
    with pytest.raises(ValueError):
        tb.rms_norm_fp8(x, w, group_size=48)
    with pytest.raises(ValueError):
        tb.rms_norm_fp8(x, w, scale_format="fp32", scale_layout="mx", group_size=32)
    with pytest.raises(ValueError):
        tb.rms_norm_fp8(x.float(), w)


def test_ops_in_compiled_regions_match_the_oracle():
    """Each torch.library op inside torch.compile(fullgraph=True), against the
    CPU oracle on exact-sum inputs (so every output is bit-exact): the
    standalone RMSNorm (bf16 and fp32, functional and with `out`), the
    reference's own op name cutie::per_token_fp8_quant, and the fused op."""
    import thingy_b200.custom_ops as co

    assert co.REFERENCE_NAMESPACE_OP
    inp = exact_sum_inputs(96, 7168, residual=True, seed=31)
    x, res, w = inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda()

    norm = torch.compile(tb.rms_norm, fullgraph=True, dynamic=False)
    y = norm(x, w, 1e-6)
    np.testing.assert_array_equal(bf16_bits(y), bf16_bits(ora.rms_norm_reference(
        inp["x"], inp["weight"], 1e-6)))
    g = torch.Generator().manual_seed(31)
    xf = torch.randint(-32, 33, (64, 3072), generator=g).float() / 16
    wf = torch.randn(3072, generator=g)
    out = torch.full((64, 3072), float("nan"), device="cuda")
    got = norm(xf.cuda(), wf.cuda(), 1e-5, out)
    assert got.data_ptr() == out.data_ptr()
    assert torch.equal(out.cpu(), ora.rms_norm_f32(xf, wf, 1e-5))

    @torch.compile(fullgraph=True, dynamic=False)
    def quant(t):
        return torch.ops.cutie.per_token_fp8_quant(t)

    q, s = quant(x)
    q_ref, s_ref = ora.quantize(inp["x"], 128, "fp32")
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref.numpy())

    @torch.compile(fullgraph=True, dynamic=False)
    def fused(x, res, w):
        return torch.ops.thingy_b200.residual_rms_norm_fp8(x, res, w, 1e-6)

    q, s, r, n = fused(x, res, w)
    q_ref, s_ref, r_ref, n_ref = ora.rms_norm_fp8(inp["x"], inp["weight"], 1e-6,
                                                  residual=inp["residual"])
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref.numpy())
    np.testing.assert_array_equal(bf16_bits(r), bf16_bits(r_ref))
    np.testing.assert_array_equal(bf16_bits(n), bf16_bits(n_ref))


def test_custom_op_in_compiled_region():
    import thingy_b200.custom_ops  # noqa: F401

    inp = random_inputs(32, 1024, residual=True, seed=21)
    x, res, w = inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda()

    @torch.compile(fullgraph=True, dynamic=False)
    def f(x, res, w):
        return torch.ops.thingy_b200.residual_rms_norm_fp8(x, res, w, 1e-6)

    q, s, r, n = f(x, res, w)
    q2, s2, r2, n2 = tb.residual_rms_norm_fp8(x, res, w, 1e-6)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s, s2)
    qq, ss = torch.ops.thingy_b200.per_token_fp8_quant(n)
    assert torch.equal(qq.view(torch.uint8), q2.view(torch.uint8))


def test_division_matches_ieee_on_gpu():
    """The one-correction division used for n / s against CUDA's own IEEE division.

    Every bf16 magnitude in the normal range, divided by fp32 scales of every
    kind (amax/448 from all bf16 amax values): the e4m3 codes (via the
    quantizer) equal those of torch's CUDA division x / s followed by the
    e4m3 cast, which uses IEEE division.
    """
    g = torch.Generator().manual_seed(17)
    amax = torch.arange(0x3C00, 0x4700, 7, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    G = 128
    rows = -(-amax.numel() // 16)
    am = torch.cat([amax, torch.ones(rows * 16 - amax.numel(), dtype=torch.bfloat16)]).float()
    vals = torch.randint(0x0080, 0x7F80, (rows * 16, G), generator=g, dtype=torch.int32)
    x = vals.to(torch.int16).view(torch.bfloat16).float()
    # fold values above the group amax back into [0, amax) exactly (float64 fmod;
    # float32 remainder overflows for huge / tiny pairs)
    folded = torch.fmod(x.abs().double(), am[:, None].double()).float()
    x = torch.where(x.abs() <= am[:, None], x, folded)
    x = (x * torch.where(torch.rand(x.shape, generator=g) < 0.5, -1.0, 1.0)).to(torch.bfloat16)
    x[:, 0] = am.to(torch.bfloat16)
    x = x.view(rows, 16 * G)
    q, s = tb.per_token_cast_to_fp8(x.cuda(), use_ue8m0=False)
    xs = x.cuda().float().view(rows, 16, G) / s.view(rows, 16, 1)
    q_ieee = xs.to(torch.float8_e4m3fn).view(rows, 16 * G)
    assert torch.equal(q.view(torch.uint8), q_ieee.view(torch.uint8))
    # tensor / tensor: torch's CUDA division by a CPU scalar multiplies by the
    # reciprocal, which is not the IEEE quotient
    s_ieee = torch.clamp(am.cuda() / torch.full_like(am, 448.0).cuda(), min=1e-4).view(rows, 16)
    assert torch.equal(s, s_ieee)


@pytest.mark.parametrize("M,H", [(16384, 7168), (64, 5120), (4096, 4096)])
def test_back_to_back_launches_see_previous_outputs(M, H):
    """Kernels start their prologue while the previous kernel drains
    (programmatic dependent launch); each must still read only complete
    outputs of the kernel before it. A chain where every launch consumes the
    previous launch's normalized output and residual sum, enqueued back to
    back on one stream, must equal the same chain run with a synchronize
    between the steps."""
    g = torch.Generator().manual_seed(M + H)
    dev = torch.device("cuda")
    x = torch.randn(M, H, generator=g).to(torch.bfloat16).to(dev)
    r = (2.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16).to(dev)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(dev)

    def chain(sync):
        cur_x, cur_r, outs = x, r, []
        for _ in range(6):
            q, s, ro, n = tb.rms_norm_fp8(cur_x, w, 1e-6, residual=cur_r, group_size=128,
                                          scale_format="fp32", scale_layout="col",
                                          return_normalized=True)
            outs.append((q, s))
            cur_x, cur_r = n, ro  # the next launch reads this launch's outputs
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs

    ref = chain(True)
    for _ in range(3):
        got = chain(False)
        for (q0, s0), (q1, s1) in zip(ref, got):
            assert torch.equal(q0.view(torch.uint8), q1.view(torch.uint8))
            assert torch.equal(s0, s1)


@pytest.mark.parametrize("raw_stream", [False, True])
def test_packed_scales_leading_dimension(raw_stream):
    """Packed UE8M0 scales with a padded word stride (ld = 80 > M = 70), through
    the torch binding and through the ctypes path (a raw stream handle): the
    words of the M rows match the oracle's packing, the pad words are untouched."""
    from thingy_b200.ops import launch_rms_norm_fp8

    M, H, ld = 70, 7168, 80
    W = 56 // 4
    inp = exact_sum_inputs(M, H, residual=True, seed=21)
    x, res, w = inp["x"].cuda(), inp["residual"].cuda(), inp["weight"].cuda()
    buf = torch.full((W, ld), -1, dtype=torch.int32, device="cuda")
    q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream if raw_stream else None
    launch_rms_norm_fp8(x, w, 1e-6, residual=res, q=q, scale=buf.t()[:M], group_size=128,
                        scale_format="e8m0", scale_layout="packed", stream=stream)
    torch.cuda.synchronize()
    q_ref, s_ref, _, _ = ora.rms_norm_fp8(inp["x"], inp["weight"], 1e-6,
                                          residual=inp["residual"], scale_format="e8m0")
    got = buf.cpu().numpy()
    np.testing.assert_array_equal(got[:, :M], ora.layout_scales(s_ref, "packed")[:, :M])
    assert (got[:, M:] == -1).all()
    np.testing.assert_array_equal(q_codes(q), q_ref.numpy())
