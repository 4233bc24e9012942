"""Build recipe for libzengpu_b200.so (sm_100a).

Run ``python -m zengpu_b200.build`` (or ``__graft_entry__.build()``).  The
library is built in-tree next to this file so it travels with the source
tree; nvcc cross-compiles for sm_100a without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libzengpu_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build zengpu_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def build_library(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every kernel and the runtime into one shared library."""
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if LIB.stat().st_mtime >= newest:
            return LIB
    cmd = [
        _nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--cudart", "static",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
        "-I", str(ROOT / "include"), "-I", str(CSRC),
        "-o", str(LIB), *map(str, srcs),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    if verbose:
        sys.stderr.write(proc.stdout + proc.stderr)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build_library(verbose=v, force="-f" in sys.argv))
