"""Builds the reference's own native extension (CPU) from its sources into oracle/_ref/cpu/.

    python oracle/build_ref.py [--src PATH_TO_REFERENCE_CHECKOUT]

Test infrastructure (a checker): nothing in the product package imports what this builds.

* ``native/jakal_net_native.cpp`` compiled CPU-only with torch.utils.cpp_extension,
  plus a two-function stub. The .cpp calls two availability probes that only the .cu defines
  (``jakal_net_low_rank_dense_scores_tf32_cuda_available`` and
  ``jakal_net_low_rank_propagation_dense_tf32_forward_cuda_available``, referenced outside its
  ``#ifdef WITH_CUDA``); the stub answers ``false`` for both, which is what a CPU-only build
  means. Module name ``jakal_net_native`` (backend "aten_cpp_cpu"). Its per-query transition
  (jakal_net_native.cpp:7089-7246) generates the fixtures that pin the oracle's
  transition_query_topk (tests/golden/make_golden_native.py).
Nothing in the reference tree is modified; outputs go to oracle/_ref/cpu/ only (git-ignored,
shipped with the tree to the GPU host like the product library). The reference's CUDA build
is baseline/build_reference_cuda.py.
"""
from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
DEFAULT_SRC = Path("/root/reference")
STUB = """// CPU-only build of the reference extension: the two CUDA availability probes the .cpp
// references outside its WITH_CUDA guard answer "not available".
bool jakal_net_low_rank_dense_scores_tf32_cuda_available() { return false; }
bool jakal_net_low_rank_propagation_dense_tf32_forward_cuda_available() { return false; }
"""


def build(kind: str = "cpu", src: Path = DEFAULT_SRC, verbose: bool = False) -> Path:
    from torch.utils.cpp_extension import load

    native = src / "native"
    out = REF_OUT / kind
    out.mkdir(parents=True, exist_ok=True)
    stub = out / "cuda_probe_stub.cpp"
    stub.write_text(STUB)
    load(name="jakal_net_native", sources=[str(native / "jakal_net_native.cpp"), str(stub)],
         build_directory=str(out), verbose=verbose, with_cuda=False, extra_include_paths=[str(native)],
         extra_cflags=["-std=c++17", "-O3"])
    return out / "jakal_net_native.so"


def load_built(kind: str):
    """Imports a module built by build() (no compiler, no reference checkout needed)."""
    import torch  # noqa: F401  (the extension links against torch's libraries)

    path = REF_OUT / kind / "jakal_net_native.so"
    if not path.exists():
        raise ImportError(f"{path} not built (python oracle/build_ref.py --{kind})")
    name = "jakal_net_native"
    if name in sys.modules and getattr(sys.modules[name], "__file__", "") == str(path):
        return sys.modules[name]
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def available(kind: str) -> bool:
    return (REF_OUT / kind / "jakal_net_native.so").exists()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", type=Path, default=DEFAULT_SRC)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build("cpu", a.src, a.verbose))
