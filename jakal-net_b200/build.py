"""Builds libjakal_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

Usage: python jakal-net_b200/build.py [--force] [--ptxas-verbose]

Every csrc/*.cu file is its own translation unit (no relocatable device code: each unit
has its own device error word, see csrc/jk_host.h). Units are compiled in parallel into
jakal-net_b200/_build/ and linked into jakal_net_b200/libjakal_b200.so, which ships with the
source tree; no JIT cache is involved. A unit is recompiled when the content hash of its
source, the shared headers and the compiler flags changes (timestamps are not trusted: a
checkout or a copy can make a stale object look new).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "jakal_net_b200" / "libjakal_b200.so"
INCLUDE = HERE.parent / "include"
OBJ_DIR = HERE / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libjakal_b200.so")
    return cand


def units() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "jakal_b200.h"]


def sources() -> list[Path]:
    return units() + headers()


def _hash(paths: list[Path], flags: list[str]) -> str:
    h = hashlib.sha256()
    for p in paths:
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(flags).encode())
    return h.hexdigest()


def _compile(unit: Path, flags: list[str], force: bool, verbose: bool) -> Path:
    obj = OBJ_DIR / (unit.stem + ".o")
    stamp = obj.with_suffix(".sha256")
    digest = _hash([unit] + headers(), flags)
    if not force and obj.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return obj
    cmd = [nvcc_path(), *flags, "-I", str(INCLUDE), "-c", str(unit), "-o", str(obj) + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(obj) + ".tmp", obj)
    stamp.write_text(digest + "\n")
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    flags = NVCC_FLAGS + list(extra or [])
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    with ThreadPoolExecutor(max_workers=max(1, min(len(units()), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(lambda u: _compile(u, flags, force, verbose), units()))
    stamp = OUT.with_name(OUT.name + ".sha256")
    digest = _hash(objs, flags)
    if not force and OUT.exists() and stamp.exists() and stamp.read_text().strip() == digest:
        return OUT
    cmd = [nvcc_path(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *[str(o) for o in objs],
           "-o", str(OUT) + ".tmp", "-lcudart"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(OUT) + ".tmp", OUT)
    stamp.write_text(digest + "\n")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose=True, extra=["-Xptxas", "-v"] if a.ptxas_verbose else None)
    print(OUT)
