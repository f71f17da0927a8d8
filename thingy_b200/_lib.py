"""ctypes binding of the C ABI in include/cutie.h.

The shared library is built in-tree (``python -m thingy_b200.build``) at
``thingy_b200/lib/libcutie_b200.so``. There is no fallback: if the library is
missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libcutie_b200.so"

# include/cutie.h enums
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_ALIGNMENT = -3
ERR_CUDA = -4

QUANT_NONE, QUANT_TOKEN, QUANT_GROUP = 0, 1, 2
SCALE_FP32, SCALE_FP32_POW2, SCALE_E8M0 = 0, 1, 2
LAYOUT_ROW_MAJOR, LAYOUT_COL_MAJOR, LAYOUT_MX_SWIZZLED, LAYOUT_COL_MAJOR_PACKED = 0, 1, 2, 3
DTYPE_BF16, DTYPE_F32 = 0, 1

ABI_VERSION = 1

EXPORTED_SYMBOLS = (
    "cutie_rms_norm_fp8",
    "cutie_per_token_cast_to_fp8",
    "cutie_rms_norm",
    "cutie_rms_norm_backward",
    "cutie_rms_norm_backward_workspace",
    "cutie_rms_norm_backward_noalloc",
    "cutie_gemm_mxfp8",
    "cutie_rms_norm_mxfp8_gemm",
    "cutie_device_error",
    "cutie_set_wait_limit",
    "cutie_last_error",
    "cutie_abi_version",
)

_i64 = ctypes.c_int64
_int = ctypes.c_int
_ptr = ctypes.c_void_p
_f32 = ctypes.c_float

_SIGNATURES = {
    "cutie_rms_norm_fp8": (
        _int,
        [_ptr, _i64, _ptr, _i64, _ptr, _f32, _i64, _i64, _int, _int, _int, _int, _i64,
         _ptr, _i64, _ptr, _ptr, _i64, _ptr, _i64, _int, _ptr],
    ),
    "cutie_per_token_cast_to_fp8": (
        _int,
        [_ptr, _i64, _i64, _i64, _int, _int, _int, _i64, _ptr, _i64, _ptr, _int, _ptr],
    ),
    "cutie_rms_norm": (
        _int,
        [_ptr, _i64, _ptr, _f32, _i64, _i64, _int, _ptr, _i64, _int, _ptr],
    ),
    "cutie_rms_norm_backward": (
        _int,
        [_ptr, _i64, _ptr, _i64, _ptr, _ptr, _i64, _f32, _i64, _i64, _ptr, _i64, _ptr,
         _ptr, ctypes.c_size_t, _int, _int, _int, _int, _i64, _ptr, _i64, _ptr, _ptr],
    ),
    "cutie_rms_norm_backward_workspace": (ctypes.c_size_t, [_i64, _i64]),
    "cutie_rms_norm_backward_noalloc": (
        _int,
        [_ptr, _i64, _ptr, _i64, _ptr, _ptr, _i64, _f32, _i64, _i64, _ptr, _i64, _ptr,
         _int, _int, _int, _int, _i64, _ptr, _i64, _ptr, _ptr],
    ),
    "cutie_gemm_mxfp8": (
        _int, [_ptr, _i64, _ptr, _ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr],
    ),
    "cutie_rms_norm_mxfp8_gemm": (
        _int,
        [_ptr, _i64, _ptr, _f32, _ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr, _i64,
         _ptr, _ptr],
    ),
    "cutie_device_error": (_int, [_int]),
    "cutie_set_wait_limit": (_i64, [_i64]),
    "cutie_last_error": (ctypes.c_char_p, []),
    "cutie_abi_version": (_int, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class CutieError(RuntimeError):
    """A CUDA-side failure reported by the library (status CUTIE_ERR_CUDA)."""


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise RuntimeError(
                f"thingy_b200 CUDA library not built: {_LIB_PATH} is missing "
                "(run `python -m thingy_b200.build`)"
            )
        lib = ctypes.CDLL(os.fspath(_LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.cutie_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"{_LIB_PATH} has ABI version {version}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def device_error(clear: bool = True) -> int:
    """The library's device-side error word on the current device (0 = none)."""
    status = load().cutie_device_error(1 if clear else 0)
    if status < 0:
        check(status)
    return status


def set_wait_limit(cycles: int) -> int:
    """Bound every wait of this thread's later launches by ``cycles`` SM cycles.

    0 restores the default (about 2 s); a negative value makes a wait that
    would block give up at once (failure-path testing). Returns the previous
    limit."""
    return int(load().cutie_set_wait_limit(int(cycles)))


def check(status: int) -> None:
    """Map a status code to the exception the reference raises for it."""
    if status == OK:
        return
    msg = load().cutie_last_error().decode(errors="replace")
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_ALIGNMENT):
        raise ValueError(msg)
    raise CutieError(msg or f"cutie status {status}")
