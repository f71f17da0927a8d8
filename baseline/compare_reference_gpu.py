"""The reference's own GPU kernels beside this repo's, same box, same shapes, same buffers.

Runs on a B200 with the reference installed into ``baseline/_ref`` (the
git-ignored install of S1ro1/thingy that travels with the tree: pip's
``--target`` install of the reference's sources; its own build backend,
uv_build, is not needed by anything here, so any PEP 517 backend that copies
``src/cutie`` and ``src/kittie`` unchanged will do). Three implementations of the
reference's fused contract (src/cutie/rms_norm/bench.py:10-15: residual add,
RMSNorm, 1x128 FP8 with fp32 row-major scales, writing q, scale,
residual_out and normalized) are timed on the same rotating workspaces:

  reference_cute      the reference's CuTe DSL kernel ``RMSNorm``
                      (src/cutie/rms_norm/rms_norm.py:36-311), unmodified,
                      compiled and launched exactly as its bench does
                      (bench.py:250-301: from_dlpack(assumed_align=32),
                      cute.compile with a fake stream, then the current
                      stream), at its default knobs (threads_per_row 128,
                      elements_per_thread 8, load_path "shared",
                      reduction "all");
  reference_unfused   ``rms_norm_fp8_unfused`` (bench.py:106-108): the
                      torch.compile region (Inductor) around the vendored
                      Triton quantizer, as the reference's bench times it;
  thingy_b200         this repository's kernel through its destination-passing
                      launcher with the same outputs requested.

Correctness first, as the reference's bench checks it (bench.py:302-332,
its own tolerances against rms_norm_fp8_unfused), for both fused kernels.
Nothing of this repository runs in the two reference legs. The reference's
bench imports ``cutlass.testing`` for its harness only (JitArguments,
benchmark); that module is absent from this image's cutlass-dsl, so a stub
holding keyword arguments stands in for JitArguments, and the timing below
replaces ``benchmark``: CUDA events around K launches on the current stream,
each launch on the next of several workspaces whose total exceeds the L2.

The reference pins nvidia-cutlass-dsl >= 4.6.1; this image has 4.5.0, whose
``cute.math`` lacks two names the kernel calls (rms_norm.py:277 and :291).
``dsl_compat()`` adds them, mapped onto 4.5.0's own operations with the
same results for the kernel's finite values: ``cute.math.abs`` is
``cute.math.absf`` (elementwise |x| of a float tensor) and
``cute.math.max(a, b)`` is ``cute.where(a > b, a, b)`` (elementwise maximum;
the kernel applies it to its fp32 scales and the 1e-4 clamp). The kernel's
own code is not touched.

GB/s uses the reference's byte model ``fused_memory_bytes`` (bench.py:
149-158: inputs read once, all four outputs written once). One JSON line per
shape:

  python baseline/compare_reference_gpu.py [--shapes 16384x7168,4096x7168]
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
REF = HERE / "_ref"
L2_BYTES = 126 * 1024 * 1024


def dsl_compat():
    """Two cutlass-dsl 4.6 names the reference's kernel uses, on 4.5.0's operations."""
    from cutlass import cute

    if not hasattr(cute.math, "abs"):
        cute.math.abs = cute.math.absf
    if not hasattr(cute.math, "max"):
        cute.math.max = lambda a, b: cute.where(a > b, a, b)


def import_reference():
    """The reference's bench module and RMSNorm class, from the baseline/_ref install."""
    if not (REF / "cutie" / "rms_norm" / "rms_norm.py").exists():
        raise SystemExit(f"the reference is not installed in {REF}")

    class JitArguments:  # the only harness name the timing below does not replace
        def __init__(self, *args, **kwargs):
            self.args = args
            self.kwargs = kwargs

    stub = types.ModuleType("cutlass.testing")
    stub.JitArguments = JitArguments
    stub.benchmark = None
    sys.modules.setdefault("cutlass.testing", stub)
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(REF / "cutie" / "rms_norm"))
    import bench as ref_bench  # noqa: E402  (the reference's bench.py)
    import rms_norm as ref_rms_norm  # noqa: E402

    return ref_bench, ref_rms_norm


def time_launches(fn, workspaces, warmup: int, iters: int) -> float:
    """Mean microseconds a launch, K launches back to back on the current stream."""
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        fn(workspaces[i % len(workspaces)])
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(iters):
        fn(workspaces[i % len(workspaces)])
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) * 1e3 / iters


def check_like_reference(outputs, reference, names=("out", "scale", "residual_out",
                                                     "normalized_out")) -> dict:
    """The reference bench's own check (bench.py:302-326): allclose per output."""
    tolerances = ((0.15, 2**-8), (0.02, 1e-7), (0, 0), (0.02, 1e-5))
    result = {}
    for name, actual, ref, (rtol, atol) in zip(names, outputs, reference, tolerances):
        result[name] = bool(torch.allclose(actual.float(), ref.float(), rtol=rtol, atol=atol))
    return result


def run_shape(ref_bench, ref_rms_norm, M: int, H: int, warmup: int, iters: int,
              eps: float = 1e-6) -> dict:
    from cutlass import cute
    import cuda.bindings.driver as cuda_driver
    from cutlass.cute.runtime import make_fake_stream

    sys.path.insert(0, str(REPO))
    from thingy_b200.ops import launch_rms_norm_fp8

    nbytes = ref_bench.fused_memory_bytes(M, H)
    n_ws = max(2, math.ceil(3 * L2_BYTES / nbytes))
    torch.manual_seed(0)
    # the reference's own workspace generator (bench.py:118-146), NaN-prefilled outputs
    ws = [ref_bench.workspace_generator(M, H, eps=eps) for _ in range(n_ws)]
    kw0 = ws[0].kwargs
    baseline = ref_bench.rms_norm_fp8_unfused(**{k: kw0[k] for k in ("x", "residual", "weight",
                                                                       "eps")})
    torch.cuda.synchronize()
    row = {"shape": f"{M}x{H}", "M": M, "H": H, "bytes": nbytes, "workspaces": n_ws,
           "iterations": iters, "gpu": torch.cuda.get_device_name()}

    # --- the reference's CuTe kernel, compiled and launched as bench.py does
    stream = cuda_driver.CUstream(torch.cuda.current_stream().cuda_stream)
    norm = ref_rms_norm.RMSNorm(elements_per_thread=8, threads_per_row=128,
                                load_path="shared", reduction="all")
    names = ("x", "residual", "weight", "out", "scale", "residual_out", "normalized_out")
    cute_ws = [ref_bench.workspace_to_cute(*(w.kwargs[n] for n in names)) for w in ws]
    c0 = cute_ws[0]
    try:
        compiled = cute.compile(norm, x=c0[0], residual=c0[1], weight=c0[2], eps=eps, out=c0[3],
                                scale=c0[4], residual_out=c0[5], normalized_out=c0[6],
                                stream=make_fake_stream())

        def cute_launch(c):
            compiled(x=c[0], residual=c[1], weight=c[2], eps=eps, out=c[3], scale=c[4],
                     residual_out=c[5], normalized_out=c[6], stream=stream)

        for n in ("out", "scale", "residual_out", "normalized_out"):
            kw0[n].fill_(float("nan"))
        cute_launch(c0)
        torch.cuda.synchronize()
        row["reference_cute_correct"] = check_like_reference(
            [kw0[n] for n in ("out", "scale", "residual_out", "normalized_out")], baseline)
        us = time_launches(cute_launch, cute_ws, warmup, iters)
        row["reference_cute_us"] = round(us, 3)
        row["reference_cute_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)
    except Exception as e:  # recorded, not hidden: a DSL version this image cannot run
        row["reference_cute_error"] = f"{type(e).__name__}: {e}"[:400]

    # --- the reference's unfused torch.compile + Triton path
    def unfused(w):
        kw = w.kwargs
        ref_bench.rms_norm_fp8_unfused(kw["x"], kw["residual"], kw["weight"], eps)

    us = time_launches(unfused, ws, warmup, iters)
    row["reference_unfused_us"] = round(us, 3)
    row["reference_unfused_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)

    # --- this repository's kernel on the identical contract and buffers
    def ours(w):
        kw = w.kwargs
        launch_rms_norm_fp8(kw["x"], kw["weight"], eps, residual=kw["residual"], q=kw["out"],
                            scale=kw["scale"], residual_out=kw["residual_out"],
                            normalized_out=kw["normalized_out"], group_size=128,
                            scale_format="fp32", scale_layout="row")

    for n in ("out", "scale", "residual_out", "normalized_out"):
        kw0[n].fill_(float("nan"))
    ours(ws[0])
    torch.cuda.synchronize()
    row["thingy_b200_correct"] = check_like_reference(
        [kw0[n] for n in ("out", "scale", "residual_out", "normalized_out")], baseline)
    us = time_launches(ours, ws, warmup, iters)
    row["thingy_b200_us"] = round(us, 3)
    row["thingy_b200_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)
    if "reference_cute_us" in row:
        row["speedup_vs_reference_cute"] = round(row["reference_cute_us"] / us, 3)
    row["speedup_vs_reference_unfused"] = round(row["reference_unfused_us"] / us, 3)
    del ws, cute_ws
    torch.cuda.empty_cache()
    return row


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--shapes", default="16384x7168,4096x7168,16384x4096,16384x3072")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--iters", type=int, default=200)
    args = ap.parse_args()
    ref_bench, ref_rms_norm = import_reference()
    dsl_compat()
    with torch.no_grad():
        for shape in args.shapes.split(","):
            M, H = (int(v) for v in shape.split("x"))
            print(json.dumps(run_shape(ref_bench, ref_rms_norm, M, H, args.warmup, args.iters)),
                  flush=True)


if __name__ == "__main__":
    main()
