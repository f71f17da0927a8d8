"""Build the sm_100a shared library ``thingy_b200/lib/libcutie_b200.so``.

One nvcc process per translation unit (they run in parallel), then one link.
The library is built in-tree so it travels with the source tree; nothing is
installed into site-packages. Run ``python -m thingy_b200.build`` (add
``--verbose-ptxas`` for per-kernel register / spill / shared-memory reports).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB_DIR = PKG / "lib"
LIB_NAME = "libcutie_b200.so"
BUILD_DIR = REPO / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build thingy_b200")
    return path


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def lib_path() -> Path:
    return LIB_DIR / LIB_NAME


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    """Compile every .cu under csrc/ for sm_100a and link the shared library."""
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objs = []
    todo = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            todo.append(cmd)
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), todo))
    failed = False
    for cmd, res in zip(todo, results):
        if res.returncode != 0 or verbose_ptxas:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode != 0:
            failed = True
            sys.stderr.write(f"FAILED: {' '.join(cmd)}\n")
    if failed:
        raise RuntimeError("nvcc failed while building thingy_b200")
    out = lib_path()
    if force or todo or not out.exists():
        tmp = out.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("linking libcutie_b200.so failed")
        os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas, jobs=args.jobs))


if __name__ == "__main__":
    main()
