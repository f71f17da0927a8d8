"""Independent FP8 E4M3 (OCP "E4M3FN") codec in numpy.  TEST INFRASTRUCTURE ONLY.

Written from the OCP 8-bit Floating Point Specification (OFP8, rev. 1.0):
1 sign bit, 4 exponent bits (bias 7), 3 mantissa bits; no infinities; the
only NaN encodings are S.1111.111; the largest finite magnitude is 448
(0.1111.110); subnormals are mant/8 * 2^-6. Conversion from wider formats is
round-to-nearest, ties to even. Used to pin torch's float8_e4m3fn cast (which
the oracle uses) to the specification.
"""

from __future__ import annotations

import numpy as np


def decode(codes: np.ndarray) -> np.ndarray:
    """uint8 codes -> float64 values (NaN for S.1111.111)."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    mag = np.where(e == 0, m / 8.0 * 2.0**-6, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return sign * mag


_POS_CODES = np.arange(0, 127, dtype=np.uint8)  # 0x00 .. 0x7E, all finite, increasing
_POS_VALUES = decode(_POS_CODES)


def encode_rne(values: np.ndarray) -> np.ndarray:
    """float64 values -> uint8 codes, round to nearest, ties to even.

    Magnitudes above the midpoint between 448 and the next step (464) are not
    representable and map to NaN (0x7F / 0xFF), as a non-saturating cast does.
    """
    v = np.asarray(values, dtype=np.float64)
    a = np.abs(v)
    hi = np.clip(np.searchsorted(_POS_VALUES, a, side="left"), 1, len(_POS_VALUES) - 1)
    lo = hi - 1
    d_lo = a - _POS_VALUES[lo]
    d_hi = _POS_VALUES[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (_POS_CODES[hi] % 2 == 0))
    code = np.where(pick_hi, _POS_CODES[hi], _POS_CODES[lo]).astype(np.int64)
    code = np.where(a <= _POS_VALUES[0], 0, code)
    code = np.where(a > 464.0, 0x7F, code)
    code = np.where(np.isnan(a), 0x7F, code)
    code = np.where(np.signbit(v), code | 0x80, code)
    return code.astype(np.uint8)
