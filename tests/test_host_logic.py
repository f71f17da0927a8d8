"""Host-side logic that needs no GPU: layouts, workloads, sharding, API validation."""

import numpy as np
import pytest
import torch

from oracle import reference as ora
import thingy_b200 as tb
from thingy_b200 import layouts
from thingy_b200.rms_norm import _threads_hint
from thingy_b200.shard import all_shards, shard_rows
from thingy_b200.workloads import WORKLOADS, make_inputs


def test_swizzle_two_implementations_agree():
    rng = np.random.default_rng(0)
    for M, G in [(1, 160), (8, 160), (128, 160), (130, 36), (300, 3), (5, 1)]:
        a = rng.integers(0, 256, (M, G), dtype=np.uint8)
        got = layouts.mx_swizzle(a)
        np.testing.assert_array_equal(got, ora.mx_swizzle(a))
        np.testing.assert_array_equal(layouts.mx_unswizzle(got, M, G), a)
        assert got.size == layouts.mx_swizzled_size(M, G)


def test_swizzle_known_positions():
    # inside one 128x4 tile: rows 0,32,64,96 of column c share a 16-byte line
    off = layouts.mx_swizzle_offset
    assert off(0, 0, 4) == 0 and off(0, 3, 4) == 3
    assert off(32, 0, 4) == 4 and off(64, 0, 4) == 8 and off(96, 1, 4) == 13
    assert off(1, 0, 4) == 16 and off(31, 2, 4) == 31 * 16 + 2
    # next column tile, next row tile
    assert off(0, 4, 8) == 512 and off(128, 0, 8) == 2 * 512


def test_workload_bytes_match_the_traffic_model():
    assert WORKLOADS["token_4096x4096"].bytes_moved() == 50_356_224
    assert WORKLOADS["g128_16384x7168"].bytes_moved() == 356_005_888
    assert WORKLOADS["residual_token_32768x8192"].bytes_moved() == 1_879_195_648
    assert [WORKLOADS["mx32_decode_5120"].bytes_moved(m) for m in (1, 8, 32, 128)] == [
        25_760, 134_400, 506_880, 1_996_800]
    assert WORKLOADS["g128_sharded_262144x8192"].bytes_moved() == 6_509_576_192
    # backward: d_normalized, r, d_residual_out read, dx written (4 x 2MH), weight read
    # and d_weight written (2 x 2H), FP8 codes of dx (MH) and fp32 scales (4 M H/128)
    M, H = 16384, 7168
    assert WORKLOADS["bwd_residual_g128_16384x7168"].bytes_moved() == (
        8 * M * H + 4 * H + M * H + 4 * M * (H // 128)) == 1_060_663_296


def test_inputs_are_seeded_and_shaped():
    w = WORKLOADS["g128_16384x7168"]
    a = make_inputs(w, 64, seed=0)
    b = make_inputs(w, 64, seed=0)
    assert torch.equal(a["x"], b["x"]) and torch.equal(a["weight"], b["weight"])
    assert a["x"].dtype == torch.bfloat16 and a["x"].shape == (64, 7168)
    col_rms = a["x"].float().square().mean(0).sqrt()
    assert int((col_rms > 10).sum()) == 7  # round(0.001 * 7168) outlier channels x50
    r = make_inputs(WORKLOADS["residual_token_32768x8192"], 256, seed=0)
    assert 1.8 < r["residual"].float().std().item() < 2.2
    t = make_inputs(WORKLOADS["mx32_decode_5120"], 128, seed=0)["x"].float()
    kurt = ((t - t.mean()) ** 4).mean() / t.var() ** 2
    assert kurt > 4.0  # heavy tails of Student-t(4)


def test_shard_rows_cover_everything_once():
    for M in (0, 1, 7, 16384, 262144, 262147):
        for world in (1, 2, 3, 4, 8):
            shards = all_shards(M, world)
            assert shards[0].start == 0 and shards[-1].stop == M
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            sizes = [s.rows for s in shards]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_python_api_rejects_cpu_tensors_without_touching_the_library():
    x = torch.zeros(4, 1024, dtype=torch.bfloat16)
    w = torch.ones(1024, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        tb.rms_norm_fp8(x, w)
    with pytest.raises(ValueError, match="CUDA"):
        tb.rms_norm(x, w)


def test_rmsnorm_knobs_validated_like_the_reference():
    with pytest.raises(ValueError):
        tb.RMSNorm(elements_per_thread=2, threads_per_row=128)
    with pytest.raises(ValueError):
        tb.RMSNorm(elements_per_thread=8, threads_per_row=100)
    with pytest.raises(ValueError):
        tb.RMSNorm(8, 128, load_path="tma")
    with pytest.raises(ValueError):
        tb.RMSNorm(8, 128, reduction="tree")
    tb.RMSNorm(4, 256, "direct", "warp0")


def test_threads_hint():
    assert _threads_hint(None, 7168) == 0
    assert _threads_hint(128, 7168) == 128  # 7 vectors a thread
    assert _threads_hint(32, 7168) == 0     # 28 vectors a thread: library picks
    assert _threads_hint(1024, 65536) == 0  # 8 vectors with 1024 threads: too many registers


def test_empty_scale_shapes():
    s = tb.empty_scale(10, 7168, 128, "fp32", "col")
    assert s.shape == (10, 56) and s.stride() == (1, 10)
    s = tb.empty_scale(10, 5120, 32, "e8m0", "mx")
    assert s.numel() == 128 * 160 and s.element_size() == 1
    assert tb.empty_scale(10, 4096, None).shape == (10, 1)


def test_packed_ue8m0_layout_known_answer():
    """Four exponents a little-endian int32 word along the groups, words M-major."""
    from oracle import reference as ora

    s = np.array([[1, 2, 3, 4, 5], [6, 7, 8, 9, 10], [11, 12, 13, 14, 255]], dtype=np.uint8)
    words = layouts.pack_ue8m0(s)
    assert words.dtype == np.int32 and words.shape == (2, 4)  # ld = 3 rounded up to 4
    assert words.view(np.uint32)[0].tolist() == [0x04030201, 0x09080706, 0x0E0D0C0B, 0]
    assert words.view(np.uint32)[1].tolist() == [0x05, 0x0A, 0xFF, 0]
    np.testing.assert_array_equal(ora.ue8m0_pack(s), words)
    np.testing.assert_array_equal(layouts.unpack_ue8m0(words, 3, 5), s)
    rng = np.random.default_rng(1)
    for M, G in [(1, 1), (7, 56), (130, 7), (5, 4)]:
        a = rng.integers(0, 256, (M, G)).astype(np.uint8)
        np.testing.assert_array_equal(ora.ue8m0_pack(a), layouts.pack_ue8m0(a))
        np.testing.assert_array_equal(layouts.unpack_ue8m0(layouts.pack_ue8m0(a), M, G), a)


def test_packed_scale_allocation_and_validation():
    from thingy_b200.ops import _scale_args

    s = tb.empty_scale(10, 7168, 128, "e8m0", "packed")  # 56 groups: 14 words a row
    assert s.shape == (10, 14) and s.stride() == (1, 12) and s.dtype == torch.int32
    assert _scale_args(s, 10, 7168, 128, "e8m0", "packed", s.device) == 12
    assert _scale_args(s.t(), 10, 7168, 128, "e8m0", "packed", s.device) == 12
    z = tb.empty_scale(6, 200 * 8, 128, "e8m0", "packed")  # 13 groups: last word padded
    assert z.shape == (6, 4) and int(z.abs().sum()) == 0
    with pytest.raises(ValueError):
        tb.empty_scale(10, 7168, 128, "fp32", "packed")
    with pytest.raises(ValueError):  # packed words are int32
        _scale_args(torch.zeros(10, 14, dtype=torch.uint8), 10, 7168, 128, "e8m0", "packed",
                    torch.device("cpu"))
    with pytest.raises(ValueError):  # row-contiguous is not the packed layout
        _scale_args(torch.zeros(10, 14, dtype=torch.int32), 10, 7168, 128, "e8m0", "packed",
                    torch.device("cpu"))


def test_torch_library_ops_trace_with_fake_tensors():
    """The ops a torch.compile region sees have fake implementations with the
    real outputs' shapes and dtypes, including the reference's own op name
    cutie::per_token_fp8_quant (registered when no module has claimed it)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    import thingy_b200.custom_ops as co

    assert co.REFERENCE_NAMESPACE_OP
    with FakeTensorMode():
        x = torch.empty(37, 7168, dtype=torch.bfloat16)
        w = torch.empty(7168, dtype=torch.bfloat16)
        y = torch.ops.thingy_b200.rms_norm(x, w, 1e-6)
        assert (y.shape, y.dtype) == (x.shape, torch.bfloat16)
        xf = torch.empty(5, 3072)
        yf = torch.ops.thingy_b200.rms_norm(xf, torch.empty(3072), 1e-5)
        assert (yf.shape, yf.dtype) == (xf.shape, torch.float32)
        for op in (torch.ops.cutie.per_token_fp8_quant, torch.ops.thingy_b200.per_token_fp8_quant):
            q, s = op(torch.empty(9, 200, dtype=torch.bfloat16))
            assert (q.shape, q.dtype, s.shape, s.dtype) == (
                (9, 200), torch.float8_e4m3fn, (9, 2), torch.float32)
        q, s, r, n = torch.ops.thingy_b200.residual_rms_norm_fp8(x, x, w, 1e-6)
        assert q.dtype == torch.float8_e4m3fn and s.shape == (37, 56)
        assert r.shape == n.shape == x.shape
