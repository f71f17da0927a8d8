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


BINDING_SRC = CSRC / "torch_binding.cpp"


def binding_path() -> Path:
    import sysconfig

    return PKG / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_binding(force: bool = False) -> Path:
    """Compile the torch binding (csrc/torch_binding.cpp) against libcutie_b200.so.

    A thin pybind11 module over the C ABI that takes at::Tensor arguments,
    so a call costs a few microseconds instead of the ~15 us of ctypes plus
    Python-side checks. Built in-tree next to the package.
    """
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    out = binding_path()
    deps = [BINDING_SRC, INCLUDE / "cutie.h", lib_path(), Path(__file__)]
    if not force and not _stale(out, deps):
        return out
    cxx = shutil.which("g++") or "g++"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    inc += [f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}", "-I/usr/local/cuda/include"]
    torch_lib = cpp_extension.library_paths()[0]
    tmp = out.with_suffix(".tmp.so")
    cmd = [
        cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
        "-DTORCH_API_INCLUDE_EXTENSION_H", *inc, str(BINDING_SRC), "-o", str(tmp),
        f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
        "-ltorch_python", f"-L{LIB_DIR}", "-lcutie_b200",
        "-Wl,-rpath,$ORIGIN/lib", f"-Wl,-rpath,{torch_lib}",
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the torch binding failed")
    os.replace(tmp, out)
    return out


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
    build_torch_binding(force=force)
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
