"""Known-answer tests pinning torch's float8_e4m3fn cast (used by the oracle)
to the OCP OFP8 E4M3 definition, via the independent codec in oracle/e4m3.py."""

import numpy as np
import torch

from oracle import e4m3


def test_decode_table():
    v = e4m3.decode(np.arange(256, dtype=np.uint8))
    assert v[0x00] == 0.0 and np.signbit(v[0x80])
    assert v[0x01] == 2.0**-9  # smallest subnormal
    assert v[0x07] == 7 * 2.0**-9  # largest subnormal
    assert v[0x08] == 2.0**-6  # smallest normal
    assert v[0x38] == 1.0
    assert v[0x7E] == 448.0 and v[0xFE] == -448.0
    assert np.isnan(v[0x7F]) and np.isnan(v[0xFF])
    assert np.count_nonzero(np.isnan(v)) == 2
    # torch decodes every code identically
    t = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(np.isnan(t), np.isnan(v))
    ok = ~np.isnan(v)
    np.testing.assert_array_equal(t[ok], v[ok])


def _boundary_values() -> np.ndarray:
    vals = e4m3.decode(np.arange(127, dtype=np.uint8))
    mids = (vals[:-1] + vals[1:]) / 2
    pts = np.concatenate([vals, mids, [464.0, 448.0 + 1e-3, 2.0**-10, 3 * 2.0**-11]])
    f = pts.astype(np.float32)
    near = np.concatenate([f, np.nextafter(f, np.float32(0)), np.nextafter(f, np.float32(np.inf))])
    return np.concatenate([near, -near]).astype(np.float32)


def test_torch_cast_is_rne_at_every_boundary():
    x = _boundary_values()
    x = x[np.abs(x) <= 464.0]
    got = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    want = e4m3.encode_rne(x.astype(np.float64))
    np.testing.assert_array_equal(got, want)


def test_torch_cast_random():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(400000) * np.exp2(rng.integers(-12, 9, 400000))).astype(np.float32)
    x = x[np.abs(x) <= 448.0]
    got = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(got, e4m3.encode_rne(x.astype(np.float64)))


def test_ties_to_even():
    # 7.25 lies halfway between 7.0 (0.1001.110) and 7.5 (0.1001.111): even mantissa wins
    assert e4m3.encode_rne(np.array([7.25]))[0] == 0x4E
    assert torch.tensor([7.25]).to(torch.float8_e4m3fn).view(torch.uint8).item() == 0x4E
    # 464 ties between 448 and the (unrepresentable) 480 -> 448
    assert e4m3.encode_rne(np.array([464.0]))[0] == 0x7E
