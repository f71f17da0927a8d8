"""Regenerate tests/golden/reference_vectors.npz from the reference's own code.

Run where a checkout of the reference exists, naming its root by argument
or by the REFERENCE_ROOT environment variable (there is no default); the GPU
box has no checkout, and nothing at test time reads the reference — only
the committed .npz.

  python tests/golden/make_golden.py <reference-root>
  REFERENCE_ROOT=<reference-root> python tests/golden/make_golden.py

What runs is the reference's own Python, unmodified:
  * src/cutie/rms_norm/bench.py: rms_norm_reference, residual_rms_norm_fp8_reference
    (its torch.library op calls the vendored Triton quantizer);
  * src/cutie/vendor/prime_rl/fp8_utils.py: per_token_cast_to_fp8_triton,
    executed by Triton's CPU interpreter (TRITON_INTERPRET=1);
  * src/cutie/rms_norm/rms_norm.py: rms_norm, called through its eager
    callable (the torch.compile wrapper is bypassed; its math is the same).
bench.py imports cutlass.testing only for its benchmark harness; that module
is absent from this image's cutlass-dsl, so a stub providing the two names it
imports is installed first. Triton's interpreter rounds float -> e4m3 wrongly
when rounding carries into the next binade (the code comes out one binade
low); the test that reads these vectors accounts for exactly that defect.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_vectors.npz"


def reference_root() -> Path:
    """The reference checkout: the first command-line argument, else REFERENCE_ROOT."""
    args = [a for a in sys.argv[1:] if not a.startswith("-")]
    root = args[0] if args else os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("name the reference checkout: make_golden.py <reference-root> "
                         "(or set REFERENCE_ROOT)")
    root = Path(root)
    if not (root / "src" / "cutie" / "rms_norm" / "bench.py").exists():
        raise SystemExit(f"{root} does not look like the reference checkout "
                         "(src/cutie/rms_norm/bench.py is missing)")
    return root


def _import_reference():
    REF = reference_root()
    stub = types.ModuleType("cutlass.testing")
    stub.JitArguments = object
    stub.benchmark = None
    sys.modules.setdefault("cutlass.testing", stub)
    sys.path.insert(0, str(REF / "src"))
    sys.path.insert(0, str(REF / "src" / "cutie" / "rms_norm"))
    import bench as ref_bench  # noqa: E402
    import rms_norm as ref_rms_norm  # noqa: E402
    from cutie.vendor.prime_rl import fp8_utils as ref_fp8  # noqa: E402

    return ref_bench, ref_rms_norm, ref_fp8


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy()
    return t.contiguous().numpy()


def main() -> None:
    ref_bench, ref_rms_norm, ref_fp8 = _import_reference()
    g = torch.Generator().manual_seed(1234)

    def weight(H):
        return (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)

    out: dict[str, np.ndarray] = {}

    # 1. The reference's fused contract: residual add + RMSNorm + 1x128 FP8.
    M, H = 16, 1024
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    res = (2.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16)
    w = weight(H)
    q, s, r, n = ref_bench.residual_rms_norm_fp8_reference(x, res, w, eps=1e-6)
    out.update({"fused_res__x": bits(x), "fused_res__residual": bits(res), "fused_res__weight": bits(w),
                "fused_res__eps": np.float64(1e-6), "fused_res__q": bits(q), "fused_res__scale": bits(s),
                "fused_res__residual_out": bits(r), "fused_res__normalized": bits(n)})

    # 2. No residual, DeepSeek-V3 width with outlier channels x50.
    M, H = 4, 7168
    x = torch.randn(M, H, generator=g)
    x[:, torch.randperm(H, generator=g)[:7]] *= 50.0
    x = x.to(torch.bfloat16)
    w = weight(H)
    n = ref_bench.rms_norm_reference(x, w, 1e-6)
    q, s = ref_bench.quantize_fp8(n)
    out.update({"outliers__x": bits(x), "outliers__weight": bits(w), "outliers__eps": np.float64(1e-6),
                "outliers__q": bits(q), "outliers__scale": bits(s), "outliers__normalized": bits(n)})

    # 3/4. Quantizer alone on a ragged width (partial last group), both scale rules.
    M, H = 8, 200
    x = (3.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16)
    for ue8m0 in (False, True):
        q, s = ref_fp8.per_token_cast_to_fp8_triton(x, use_ue8m0=ue8m0)
        tag = "ragged_ue8m0" if ue8m0 else "ragged_fp32"
        out.update({f"{tag}__x": bits(x), f"{tag}__q": bits(q), f"{tag}__scale": bits(s)})

    # 5. Power-of-two scales on normalized activations.
    M, H = 16, 1024
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w = weight(H)
    n = ref_bench.rms_norm_reference(x, w, 1e-6)
    q, s = ref_fp8.per_token_cast_to_fp8_triton(n, use_ue8m0=True)
    out.update({"ue8m0__x": bits(x), "ue8m0__weight": bits(w), "ue8m0__eps": np.float64(1e-6),
                "ue8m0__normalized": bits(n), "ue8m0__q": bits(q), "ue8m0__scale": bits(s)})

    # 6. Edge rows: zeros (scale clamps to 1e-4), a constant row, one huge
    #    value among small ones, tiny values, alternating signs.
    H = 256
    rows = [
        torch.zeros(H),
        torch.full((H,), 0.75),
        torch.cat([torch.tensor([3.0e4]), 1e-3 * torch.randn(H - 1, generator=g)]),
        1e-6 * torch.randn(H, generator=g),
        torch.tensor([(-1.0) ** i * (1 + i % 7) for i in range(H)]),
    ]
    x = torch.stack(rows).to(torch.bfloat16)
    w = weight(H)
    n = ref_bench.rms_norm_reference(x, w, 1e-6)
    q, s = ref_fp8.per_token_cast_to_fp8_triton(n, use_ue8m0=False)
    out.update({"edge__x": bits(x), "edge__weight": bits(w), "edge__eps": np.float64(1e-6),
                "edge__normalized": bits(n), "edge__q": bits(q), "edge__scale": bits(s)})

    # 7. Standalone fp32 RMSNorm (rms_norm.py:11-20), eps 1e-5.
    M, H = 8, 1024
    x = torch.randn(M, H, generator=g)
    w = torch.randn(H, generator=g)
    eager = ref_rms_norm.rms_norm._torchdynamo_orig_callable
    y = eager(x, w, 1e-5)
    out.update({"f32__x": bits(x), "f32__weight": bits(w), "f32__eps": np.float64(1e-5), "f32__out": bits(y)})

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
