"""Scale layouts of the FP8 path and their index maps.

``row``  scale[m, g] at m * ld + g (the reference's [M, ceil(H/128)] fp32
         scales, src/cutie/vendor/prime_rl/fp8_utils.py:70).
``col``  scale[m, g] at g * ld + m: the column-major [H/128, M] scales a
         DeepGEMM-style blockwise FP8 GEMM reads along M.
``mx``   Blackwell block-scaled GEMM layout for e8m0 scales (cuBLAS "1D block
         scaling factors layout", tcgen05 scale-factor layout): the [M, G]
         scale matrix is padded to [ceil(M/128)*128, ceil(G/4)*4] and cut into
         128x4 tiles of 512 bytes stored tile-row-major; inside a tile, row r
         and column c sit at (r % 32) * 16 + (r // 32) * 4 + c. Padding bytes
         are 0.
``packed`` e8m0 exponents packed four to a little-endian int32 word along the
         groups, words M-major: scale[m, g] is byte g % 4 of word
         (g // 4) * ld + m, ld >= M (default M rounded up to 4). This is the
         int32 [M, ceil(G/4)] tensor with strides (1, ld) that DeepGEMM-style
         SM100 FP8 GEMMs take as packed UE8M0 scales. Bytes of groups past the
         last one in the final word are not written by the kernels.
"""

from __future__ import annotations

import numpy as np

SCALE_LAYOUTS = ("row", "col", "mx", "packed")
SCALE_FORMATS = ("fp32", "ue8m0", "e8m0")


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def n_groups(H: int, group_size: int | None) -> int:
    """Scales per row: 1 for per-token (group_size None/0), else ceil(H/G)."""
    return 1 if not group_size else ceil_div(H, group_size)


def mx_padded_shape(M: int, groups: int) -> tuple[int, int]:
    return ceil_div(M, 128) * 128, ceil_div(groups, 4) * 4


def mx_swizzled_size(M: int, groups: int) -> int:
    rows, cols = mx_padded_shape(M, groups)
    return rows * cols


def mx_swizzle_offset(row, g, groups: int):
    """Byte offset of scale (row, g) in the swizzled buffer (numpy-vectorised)."""
    row = np.asarray(row, dtype=np.int64)
    g = np.asarray(g, dtype=np.int64)
    tiles_per_row = ceil_div(groups, 4)
    tile = (row // 128) * tiles_per_row + g // 4
    r = row % 128
    return tile * 512 + (r % 32) * 16 + (r // 32) * 4 + g % 4


def mx_swizzle(scales: np.ndarray) -> np.ndarray:
    """[M, G] byte matrix -> flat swizzled buffer (zero padding)."""
    M, G = scales.shape
    rows, cols = mx_padded_shape(M, G)
    padded = np.zeros((rows, cols), dtype=scales.dtype)
    padded[:M, :G] = scales
    out = np.zeros(rows * cols, dtype=scales.dtype)
    rr, gg = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    out[mx_swizzle_offset(rr, gg, G)] = padded
    return out


def mx_unswizzle(buf: np.ndarray, M: int, G: int) -> np.ndarray:
    """Flat swizzled buffer -> [M, G] byte matrix (padding dropped)."""
    rr, gg = np.meshgrid(np.arange(M), np.arange(G), indexing="ij")
    return np.asarray(buf).reshape(-1)[mx_swizzle_offset(rr, gg, G)]


def packed_ld(M: int) -> int:
    """Default word stride of the packed layout: M rounded up to 4 (16-byte columns)."""
    return ceil_div(M, 4) * 4


def pack_ue8m0(scales: np.ndarray, ld: int | None = None) -> np.ndarray:
    """[M, G] exponent bytes -> [ceil(G/4), ld] int32 words (zero padding)."""
    scales = np.asarray(scales, dtype=np.uint8)
    M, G = scales.shape
    ld = packed_ld(M) if ld is None else ld
    W = ceil_div(G, 4)
    b = np.zeros((W, ld, 4), dtype=np.uint8)
    padded = np.zeros((M, W * 4), dtype=np.uint8)
    padded[:, :G] = scales
    b[:, :M, :] = padded.reshape(M, W, 4).transpose(1, 0, 2)
    return b.reshape(W, ld * 4).view("<i4").reshape(W, ld)


def unpack_ue8m0(words: np.ndarray, M: int, G: int) -> np.ndarray:
    """[ceil(G/4), ld] int32 words (ld >= M) -> [M, G] exponent bytes."""
    words = np.ascontiguousarray(np.asarray(words, dtype="<i4"))
    W = ceil_div(G, 4)
    b = words.reshape(W, -1).view(np.uint8).reshape(W, -1, 4)[:, :M, :]
    return b.transpose(1, 0, 2).reshape(M, W * 4)[:, :G]
