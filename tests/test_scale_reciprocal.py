"""The scale reciprocal of the kernels is correctly rounded on its whole domain.

The kernels divide by a group scale s through Markstein's one-correction
division, which needs rc = RN(1/s). They compute rc with Markstein's
reciprocal iteration (csrc/fused_kernel.cuh, rcp_scale): y0 = rcp.approx(s),
which PTX documents as at most 1 ulp from 1/s, then e = RN(1 - s*y0) and
y1 = RN(y0 + e*y0), both single fused multiply-adds.

One iteration is not correctly rounded for every fp32 s. The scales here are
a finite set, though: s = max(RN(amax / 448), 1e-4) with amax a finite bf16
magnitude (fp8_utils.py:50-51 of the reference), 16969 distinct values. This
test runs the iteration in exact rational arithmetic from every start within
2 ulps of 1/s (twice the documented error of the approximation) and requires
RN(1/s) every time. It tests the method, restated here; the GPU parity tests
check the kernels' codes and scales end to end.
"""

from __future__ import annotations

import struct
from fractions import Fraction as F


def _bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def _from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def rn32(q: F) -> F:
    """Round a rational to the nearest fp32 value, ties to even (normal range)."""
    if q == 0:
        return F(0)
    sign = -1 if q < 0 else 1
    q = abs(q)
    e = q.numerator.bit_length() - q.denominator.bit_length()
    if F(2) ** e > q:
        e -= 1
    if F(2) ** (e + 1) <= q:
        e += 1
    assert -126 <= e <= 127, "outside the normal fp32 range"
    ulp = F(2) ** (e - 23)
    m = q / ulp
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return sign * fl * ulp


def scale_domain() -> list[float]:
    """Every fp32 scale max(RN(a / 448), 1e-4) for a positive finite bf16 a (and a = 0)."""
    floor = rn32(F(1, 10000))
    out = {float(floor)}
    for b in range(1, 0x7F80):
        a = F(_from_bits(b << 16))
        if a / 448 < floor:
            continue
        out.add(float(rn32(a / 448)))
    return sorted(out)


def markstein_reciprocal(s: F, y0: F) -> F:
    e = rn32(1 - s * y0)
    return rn32(y0 + e * y0)


def test_markstein_reciprocal_is_correctly_rounded_on_every_scale():
    scales = scale_domain()
    assert len(scales) == 16969
    for s in scales:
        want = rn32(1 / F(s))
        wb = _bits(float(want))
        for k in (-2, -1, 0, 1, 2):
            y0 = F(_from_bits(wb + k))
            assert markstein_reciprocal(F(s), y0) == want, (s, k)


def test_one_iteration_is_not_enough_for_arbitrary_fp32():
    """The check above is not vacuous: off the scale domain the same iteration,
    started one ulp away, misses RN(1/s) for some fp32 s (significands near
    all ones are the classic failures)."""
    misses = 0
    for b in range(_bits(1.0), _bits(2.0), 4099):
        s = F(_from_bits(b))
        want = rn32(1 / s)
        for k in (-1, 1):
            y0 = F(_from_bits(_bits(float(want)) + k))
            misses += markstein_reciprocal(s, y0) != want
    s = F(_from_bits(_bits(2.0) - 1))  # 1.11...1 * 2^0
    want = rn32(1 / s)
    misses += any(markstein_reciprocal(s, F(_from_bits(_bits(float(want)) + k))) != want
                  for k in (-1, 1))
    assert misses > 0
