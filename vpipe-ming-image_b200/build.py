"""Build recipe for libmingproj.so (sm_100a) — the mingproj C-ABI library.

Run as a script or call build(). Compiles every .cu under csrc/ with nvcc for
sm_100a only, links the CUDA runtime statically (so the library loads on a
machine without a GPU and its exports can be checked there), and writes
mingproj/libmingproj.so next to the Python bindings.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "mingproj" / "libmingproj.so"
BUILD = HERE / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    return cand if Path(cand).exists() else "nvcc"


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link; returns the path of the shared library."""
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        deps = [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [
            HERE.parent / "include" / "mingproj.h"]
        fresh = obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps)
        if not fresh:
            cmd = [_nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
        objs.append(obj)
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
           "-cudart", "static", "-o", str(OUT), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
