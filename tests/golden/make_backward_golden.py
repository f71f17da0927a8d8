"""Regenerate tests/golden/backward_vectors.npz from the reference's own forward.

The reference has no backward pass; the gradients of its PyTorch forward are
what torch autograd computes for it. This script imports the reference's
unmodified bench.py (as make_golden.py does: same stub, and the checkout named
by the first argument or REFERENCE_ROOT), differentiates its rms_norm_reference
(src/cutie/rms_norm/bench.py:58-65) and its residual add (x + residual, as in
residual_rms_norm_fp8_reference, bench.py:97) with torch.autograd on the CPU,
and stores inputs and gradients. Nothing at test time reads the reference.

  python tests/golden/make_backward_golden.py <reference-root>
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
from make_golden import _import_reference, bits  # noqa: E402

OUT = Path(__file__).resolve().parent / "backward_vectors.npz"


def main() -> None:
    ref_bench, _, _ = _import_reference()
    g = torch.Generator().manual_seed(4321)
    out: dict[str, np.ndarray] = {}

    def case(tag, M, H, residual, eps, scale_outliers=False):
        x = torch.randn(M, H, generator=g)
        if scale_outliers:
            x[:, torch.randperm(H, generator=g)[: max(1, H // 1000)]] *= 50.0
        x = x.to(torch.bfloat16)
        w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
        dn = torch.randn(M, H, generator=g).to(torch.bfloat16)
        xg = x.clone().requires_grad_(True)
        wg = w.clone().requires_grad_(True)
        outs, grads = [], []
        if residual:
            res = (2.0 * torch.randn(M, H, generator=g)).to(torch.bfloat16)
            dro = torch.randn(M, H, generator=g).to(torch.bfloat16)
            rg = res.clone().requires_grad_(True)
            r = xg + rg  # the residual add of residual_rms_norm_fp8_reference
            outs, grads = [r], [dro]
            out.update({f"{tag}__residual": bits(res), f"{tag}__d_residual_out": bits(dro)})
        else:
            r = xg
        n = ref_bench.rms_norm_reference(r, wg, eps)
        torch.autograd.backward([n] + outs, [dn] + grads)
        out.update({f"{tag}__x": bits(x), f"{tag}__weight": bits(w), f"{tag}__eps": np.float64(eps),
                    f"{tag}__d_normalized": bits(dn), f"{tag}__dx": bits(xg.grad),
                    f"{tag}__d_weight": bits(wg.grad)})
        if residual:
            assert torch.equal(rg.grad, xg.grad)

    case("plain", 8, 1024, residual=False, eps=1e-6)
    case("residual", 8, 2048, residual=True, eps=1e-5)
    case("deepseek", 2, 7168, residual=True, eps=1e-6, scale_outliers=True)
    case("ragged", 6, 200, residual=False, eps=1e-6)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
