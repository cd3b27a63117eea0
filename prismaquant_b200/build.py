"""Build libprismaquant_b200.so in-tree with nvcc for sm_100a.

    python -m prismaquant_b200.build

The library is one translation unit (csrc/pq_lib.cu).  No --use_fast_math:
the kernels rely on IEEE division, denormals and round-to-nearest products to
reproduce the reference bit for bit.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
SRC = PKG / "csrc" / "pq_lib.cu"
OUT = PKG / "libprismaquant_b200.so"
SOURCES = sorted((PKG / "csrc").glob("*.cu")) + sorted((PKG / "csrc").glob("*.cuh")) + \
    sorted((PKG / "csrc").glob("*.h")) + [REPO / "include" / "prismaquant_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in SOURCES if s.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{REPO / 'include'}", f"-I{PKG / 'csrc'}", "-o", str(OUT), str(SRC)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
