"""Build recipe for libsa_b200.so (sm_100a), in-tree.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links one
shared library next to this file. cudart is linked statically (nvcc's
default), so the library depends only on the driver at run time. Object
files go to ``<repo>/_build/`` and are rebuilt when a source or
header is newer.
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
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libsa_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsa_b200.so")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    objects = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if _stale(obj, [src] + headers + [Path(__file__)]):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
