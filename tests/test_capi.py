"""The C ABI library loads, exports every declared symbol, and rejects bad
arguments with status codes before touching CUDA (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from thingy_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "cutie.h"


@pytest.fixture(scope="module")
def lib():
    if not _lib.library_path().exists():
        from thingy_b200.build import build

        build()
    return _lib.load()


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"CUTIE_API\s+(?:const\s+)?\w+\s*\*?\s*(cutie_\w+)\s*\(", text)


def test_header_declares_the_binding_table():
    assert sorted(declared_symbols()) == sorted(_lib.EXPORTED_SYMBOLS)


def test_header_enums_match_the_python_constants():
    """Every CUTIE_* enum value in the header equals the _lib constant of the
    same name (CUTIE_ prefix dropped), and every such constant is in the header."""
    text = HEADER.read_text()
    enums = {m[0]: int(m[1]) for m in re.findall(r"\b(CUTIE_[A-Z0-9_]+)\s*=\s*(-?\d+)\s*,", text)}
    assert len(enums) >= 17
    for name, value in enums.items():
        assert getattr(_lib, name[len("CUTIE_"):]) == value, name
    prefixes = ("OK", "ERR_", "QUANT_", "SCALE_", "LAYOUT_", "DTYPE_")
    for name in dir(_lib):
        if name.startswith(prefixes) and isinstance(getattr(_lib, name), int):
            assert "CUTIE_" + name in enums, name


def test_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.cutie_abi_version() == _lib.ABI_VERSION


def test_exports_nothing_else():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.library_path())],
                         capture_output=True, text=True, check=True).stdout
    names = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {n for n in names if n.startswith("cutie_")} == set(_lib.EXPORTED_SYMBOLS)


FAKE = ctypes.c_void_p(0x10000)  # never dereferenced: every call below fails validation


def fused(lib, **kw):
    args = dict(x=FAKE, ldx=1024, residual=None, ldr=0, weight=FAKE, eps=1e-6, M=4, H=1024,
                quant_mode=_lib.QUANT_GROUP, group_size=128, scale_fmt=0, scale_layout=0,
                ld_scale=0, q=FAKE, ldq=1024, scale=FAKE, residual_out=None, ldro=0,
                normalized_out=None, ldn=0, threads_per_row=0, stream=None)
    args.update(kw)
    return lib.cutie_rms_norm_fp8(*args.values())


@pytest.mark.parametrize(
    "kw,code,needle",
    [
        ({"M": -1}, _lib.ERR_INVALID_ARGUMENT, "M >= 0"),
        ({"H": 0}, _lib.ERR_INVALID_ARGUMENT, "H > 0"),
        ({"H": 1020, "ldx": 1020, "ldq": 1020}, _lib.ERR_UNSUPPORTED, "multiple of 8"),
        ({"quant_mode": 9}, _lib.ERR_INVALID_ARGUMENT, "quant_mode"),
        ({"group_size": 48}, _lib.ERR_UNSUPPORTED, "group_size"),
        ({"scale_fmt": 5}, _lib.ERR_INVALID_ARGUMENT, "scale_fmt"),
        ({"scale_layout": 5}, _lib.ERR_INVALID_ARGUMENT, "scale_layout"),
        ({"residual_out": FAKE, "ldro": 1024}, _lib.ERR_INVALID_ARGUMENT, "requires residual"),
        ({"quant_mode": 0}, _lib.ERR_INVALID_ARGUMENT, "no output"),
        ({"scale_layout": 2}, _lib.ERR_INVALID_ARGUMENT, "E8M0"),
        ({"eps": float("nan")}, _lib.ERR_INVALID_ARGUMENT, "eps"),
        ({"scale_layout": _lib.LAYOUT_COL_MAJOR_PACKED}, _lib.ERR_INVALID_ARGUMENT,
         "packed scale layout needs E8M0"),
        ({"scale_layout": _lib.LAYOUT_COL_MAJOR_PACKED, "scale_fmt": _lib.SCALE_E8M0,
          "ld_scale": 3}, _lib.ERR_INVALID_ARGUMENT, "words < M"),
        ({"scale_layout": 4}, _lib.ERR_INVALID_ARGUMENT, "scale_layout"),
    ],
)
def test_argument_errors(lib, kw, code, needle):
    assert fused(lib, **kw) == code
    assert needle in lib.cutie_last_error().decode()


def backward(lib, **kw):
    args = dict(dn=FAKE, ldd=1024, r=FAKE, ldr=1024, weight=FAKE, dro=None, lddr=0, eps=1e-6,
                M=4, H=1024, dx=FAKE, lddx=1024, d_weight=None, workspace=None,
                workspace_bytes=ctypes.c_size_t(0), quant_mode=_lib.QUANT_GROUP, group_size=128,
                scale_fmt=0, scale_layout=0, ld_scale=0, q=FAKE, ldq=1024, scale=FAKE,
                stream=None)
    args.update(kw)
    return lib.cutie_rms_norm_backward(*args.values())


@pytest.mark.parametrize(
    "kw,code,needle",
    [
        ({"H": 40000, "ldd": 40000, "ldr": 40000, "lddx": 40000, "ldq": 40000},
         _lib.ERR_UNSUPPORTED, "32768"),
        ({"group_size": 32}, _lib.ERR_UNSUPPORTED, "1x128 groups only"),
        ({"scale_layout": _lib.LAYOUT_COL_MAJOR_PACKED}, _lib.ERR_INVALID_ARGUMENT,
         "packed scale layout needs E8M0"),
        ({"scale_layout": _lib.LAYOUT_COL_MAJOR_PACKED, "scale_fmt": _lib.SCALE_E8M0,
          "ld_scale": 3}, _lib.ERR_INVALID_ARGUMENT, "words < M"),
        ({"scale_layout": 4}, _lib.ERR_INVALID_ARGUMENT, "scale_layout"),
    ],
)
def test_backward_argument_errors(lib, kw, code, needle):
    assert backward(lib, **kw) == code
    assert needle in lib.cutie_last_error().decode()


def backward_noalloc(lib, **kw):
    args = dict(dn=FAKE, ldd=1024, r=FAKE, ldr=1024, weight=FAKE, dro=None, lddr=0, eps=1e-6,
                M=4, H=1024, dx=FAKE, lddx=1024, d_weight=None, quant_mode=_lib.QUANT_GROUP,
                group_size=128, scale_fmt=0, scale_layout=0, ld_scale=0, q=FAKE, ldq=1024,
                scale=FAKE, stream=None)
    args.update(kw)
    return lib.cutie_rms_norm_backward_noalloc(*args.values())


MISALIGNED = ctypes.c_void_p(0x10008)  # 8-byte aligned only


@pytest.mark.parametrize(
    "kw,code,needle",
    [
        ({"H": 40000, "ldd": 40000, "ldr": 40000, "lddx": 40000, "ldq": 40000},
         _lib.ERR_UNSUPPORTED, "32768"),
        ({"H": 1020, "ldd": 1020, "ldr": 1020, "lddx": 1020, "ldq": 1020},
         _lib.ERR_UNSUPPORTED, "multiple of 8"),
        ({"r": MISALIGNED}, _lib.ERR_ALIGNMENT, "16-byte aligned"),
        ({"dn": MISALIGNED}, _lib.ERR_ALIGNMENT, "16-byte aligned"),
        ({"weight": MISALIGNED}, _lib.ERR_ALIGNMENT, "weight"),
        ({"weight": None}, _lib.ERR_INVALID_ARGUMENT, "weight is NULL"),
        ({"M": -1}, _lib.ERR_INVALID_ARGUMENT, "M >= 0"),
        ({"group_size": 32}, _lib.ERR_UNSUPPORTED, "1x128 groups only"),
        ({"scale_layout": 4}, _lib.ERR_INVALID_ARGUMENT, "scale_layout"),
        ({"eps": float("inf")}, _lib.ERR_INVALID_ARGUMENT, "eps"),
    ],
)
def test_backward_noalloc_argument_errors(lib, kw, code, needle):
    """The allocation-free backward validates like the workspace one, before any CUDA call."""
    assert backward_noalloc(lib, **kw) == code
    assert needle in lib.cutie_last_error().decode()


def test_backward_noalloc_nothing_to_do_is_a_no_op(lib):
    """M = 0 with no d_weight requested returns at once, touching no device state."""
    assert backward_noalloc(lib, M=0, dn=None, r=None, dx=None, q=None, scale=None) == _lib.OK
    assert lib.cutie_last_error() == b""


def test_empty_batch_is_a_no_op(lib):
    assert fused(lib, M=0, x=None, q=None, scale=None, weight=None) == _lib.OK
    assert lib.cutie_last_error() == b""


def test_quantizer_and_rms_norm_errors(lib):
    assert lib.cutie_per_token_cast_to_fp8(FAKE, 1024, 4, 1024, 48, 0, 0, 0, FAKE, 1024, FAKE,
                                           0, None) == _lib.ERR_UNSUPPORTED
    assert lib.cutie_rms_norm(FAKE, 1024, FAKE, 1e-5, 4, 1024, 7, FAKE, 1024, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.cutie_rms_norm(FAKE, 1024, FAKE, 1e-5, 4, 1022, _lib.DTYPE_F32, FAKE, 1024, 0,
                              None) == _lib.ERR_UNSUPPORTED


def test_python_maps_status_to_exceptions(lib):
    with pytest.raises(ValueError, match="multiple of 8"):
        _lib.check(fused(lib, H=1020, ldx=1020, ldq=1020))


def test_wait_limit_is_per_thread_and_restorable(lib):
    """cutie_set_wait_limit returns the previous limit, 0 restores the default
    (~2 s of SM cycles), and the setting belongs to the calling thread."""
    import threading

    default = 4_000_000_000
    assert lib.cutie_set_wait_limit(-1) == default
    assert lib.cutie_set_wait_limit(0) == -1
    assert lib.cutie_set_wait_limit(123) == default
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.cutie_set_wait_limit(0)))
    t.start()
    t.join()
    assert seen == [default]  # the other thread never saw 123
    assert lib.cutie_set_wait_limit(0) == 123
    assert _lib.set_wait_limit(0) == default


def gemm(lib, **kw):
    args = dict(a=FAKE, lda=1024, a_scale=FAKE, b=FAKE, ldb=1024, b_scale=FAKE, d=FAKE,
                ldd=256, M=4, N=256, K=1024, stream=None)
    args.update(kw)
    return lib.cutie_gemm_mxfp8(*args.values())


def fused_gemm(lib, **kw):
    args = dict(x=FAKE, ldx=1024, weight=FAKE, eps=1e-6, b=FAKE, ldb=1024, b_scale=FAKE, d=FAKE,
                ldd=256, M=4, N=256, K=1024, q=None, ldq=0, q_scale=None, stream=None)
    args.update(kw)
    return lib.cutie_rms_norm_mxfp8_gemm(*args.values())


@pytest.mark.parametrize(
    "kw,code,needle",
    [
        ({"N": 192, "ldd": 192}, _lib.ERR_UNSUPPORTED, "multiples of 128"),
        ({"K": 1000, "lda": 1000, "ldb": 1000}, _lib.ERR_UNSUPPORTED, "multiples of 128"),
        ({"M": -1}, _lib.ERR_INVALID_ARGUMENT, "M >= 0"),
        ({"a": MISALIGNED}, _lib.ERR_ALIGNMENT, "16-byte aligned"),
        ({"lda": 1000}, _lib.ERR_INVALID_ARGUMENT, "leading dimension"),
        ({"b_scale": None}, _lib.ERR_INVALID_ARGUMENT, "NULL"),
        ({"a_scale": MISALIGNED}, _lib.ERR_ALIGNMENT, "scale"),
    ],
)
def test_gemm_argument_errors(lib, kw, code, needle):
    """The MXFP8 GEMM validates its arguments before any CUDA call."""
    assert gemm(lib, **kw) == code
    assert needle in lib.cutie_last_error().decode()


@pytest.mark.parametrize(
    "kw,code,needle",
    [
        ({"N": 192, "ldd": 192}, _lib.ERR_UNSUPPORTED, "multiples of 128"),
        ({"K": 1000, "ldx": 1000, "ldb": 1000}, _lib.ERR_UNSUPPORTED, "multiples of 128"),
        ({"K": 131072, "ldx": 131072, "ldb": 131072}, _lib.ERR_UNSUPPORTED, "65536"),
        ({"M": -1}, _lib.ERR_INVALID_ARGUMENT, "M >= 0"),
        ({"eps": float("nan")}, _lib.ERR_INVALID_ARGUMENT, "eps"),
        ({"q": FAKE, "ldq": 1024}, _lib.ERR_INVALID_ARGUMENT, "together"),
        ({"x": MISALIGNED}, _lib.ERR_ALIGNMENT, "16-byte aligned"),
        ({"weight": MISALIGNED}, _lib.ERR_ALIGNMENT, "weight"),
        ({"weight": None}, _lib.ERR_INVALID_ARGUMENT, "weight is NULL"),
        ({"ldx": 1020}, _lib.ERR_INVALID_ARGUMENT, "leading dimension"),
        ({"q": FAKE, "ldq": 1024, "q_scale": MISALIGNED}, _lib.ERR_ALIGNMENT, "scale"),
    ],
)
def test_fused_gemm_argument_errors(lib, kw, code, needle):
    """The fused RMSNorm -> MXFP8 -> GEMM validates its arguments before any CUDA call."""
    assert fused_gemm(lib, **kw) == code
    assert needle in lib.cutie_last_error().decode()


def test_gemms_with_no_rows_are_no_ops(lib):
    assert gemm(lib, M=0, a=None, a_scale=None, b=None, b_scale=None, d=None) == _lib.OK
    assert fused_gemm(lib, M=0, x=None, weight=None, b=None, b_scale=None, d=None) == _lib.OK
    assert lib.cutie_last_error() == b""
