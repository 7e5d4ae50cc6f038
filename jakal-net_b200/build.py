"""Builds libjakal_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

Usage: python jakal-net_b200/build.py [--force]
The library lands next to the Python package (jakal_net_b200/libjakal_b200.so) so that
it ships with the source tree; no JIT cache is involved.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "jakal_net_b200" / "libjakal_b200.so"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libjakal_b200.so")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "jakal_b200.h"]


def needs_build() -> bool:
    if not OUT.exists():
        return True
    mtime = OUT.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra or []), "-I", str(INCLUDE), str(CSRC / "jk_lib.cu"), "-o", str(OUT) + ".tmp", "-lcudart"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose=True, extra=["-Xptxas", "-v"] if a.ptxas_verbose else None)
    print(OUT)
