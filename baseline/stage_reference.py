"""Stages the reference Jakal-Net sources into baseline/_ref/ (git-ignored).

The reference checkout has neither setup.py nor pyproject.toml, so
``pip install --target baseline/_ref`` refuses it ("Directory ... is not installable").
This recipe does what that install would do: it copies the importable package
``src/jakal_net``, the model script ``scripts/progressive_b_example.py`` and the reference's
native-backend test suite ``tests/test_native_backend.py`` unchanged into ``baseline/_ref/``. The folder is git-ignored (never committed) but travels with the tree
to the GPU host, where the reference checkout itself does not exist.

Only tests/ and bench.py's reference arm import what lands there (through
``baseline/reference_shim.py``); the product package never does.

Usage: python baseline/stage_reference.py [--src PATH_TO_REFERENCE_CHECKOUT]
"""
from __future__ import annotations

import argparse
import shutil
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref"
DEFAULT_SRC = Path("/root/reference")
ITEMS = (("src/jakal_net", "jakal_net"), ("scripts/progressive_b_example.py", "progressive_b_example.py"),
         ("tests/test_native_backend.py", "reference_tests/test_native_backend.py"))


def stage(src: Path = DEFAULT_SRC, dest: Path = DEST) -> bool:
    """Copies the reference package into ``dest``; returns False when ``src`` is absent."""
    if not (src / "src" / "jakal_net").is_dir():
        return False
    dest.mkdir(parents=True, exist_ok=True)
    for rel, name in ITEMS:
        s, d = src / rel, dest / name
        if s.is_dir():
            if d.exists():
                shutil.rmtree(d)
            shutil.copytree(s, d, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        else:
            d.parent.mkdir(parents=True, exist_ok=True)
            shutil.copy2(s, d)
    return True


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", type=Path, default=DEFAULT_SRC)
    a = ap.parse_args()
    print("staged" if stage(a.src) else f"reference checkout not found at {a.src}", DEST)
