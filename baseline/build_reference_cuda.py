"""Builds the reference's own CUDA extension, unchanged, into baseline/_ref/native_cuda/.

    python baseline/build_reference_cuda.py [--src PATH_TO_REFERENCE_CHECKOUT]

This is the reference's own build recipe (scripts/build_native_extension.py: ``native/
jakal_net_native.cpp`` plus ``native/jakal_net_native_cuda.cu`` with ``-DWITH_CUDA``,
torch.utils.cpp_extension) with the GPU architecture fixed to sm_100a; nvcc cross-compiles
it without a GPU. The output is the reference install next to the staged Python package
(git-ignored, shipped with the tree to the GPU host): the same-box GPU reference that
bench.py times beside this backend, and the reference backend the GPU parity tests compare
against on identical inputs. The product package never imports it.
"""
from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "native_cuda"
DEFAULT_SRC = Path("/root/reference")
MODULE = "jakal_net_native"


def build(src: Path = DEFAULT_SRC, verbose: bool = False) -> Path:
    from torch.utils.cpp_extension import load

    native = src / "native"
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    load(name=MODULE, sources=[str(native / "jakal_net_native.cpp"), str(native / "jakal_net_native_cuda.cu")],
         build_directory=str(OUT), verbose=verbose, with_cuda=True, extra_include_paths=[str(native)],
         extra_cflags=["-std=c++17", "-O3", "-DWITH_CUDA"],
         extra_cuda_cflags=["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a"])
    return OUT / f"{MODULE}.so"


def available() -> bool:
    return (OUT / f"{MODULE}.so").exists()


def load_built():
    """Imports the built extension (no compiler or reference checkout needed)."""
    import torch  # noqa: F401  (the extension links against torch's libraries)

    path = OUT / f"{MODULE}.so"
    if not path.exists():
        raise ImportError(f"{path} not built (python baseline/build_reference_cuda.py)")
    if MODULE in sys.modules and getattr(sys.modules[MODULE], "__file__", "") == str(path):
        return sys.modules[MODULE]
    loader = importlib.machinery.ExtensionFileLoader(MODULE, str(path))
    spec = importlib.util.spec_from_loader(MODULE, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[MODULE] = mod
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", type=Path, default=DEFAULT_SRC)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.src, a.verbose))
