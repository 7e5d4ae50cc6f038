"""Imports the reference Jakal-Net package from a source checkout (fixture generation only).

The shipped package fails to import: ``jakal_net/transition.py`` imports
``unit_normalize_values`` from ``jakal_net/_architectural_common.py``, which only defines
``normalize_value_directions``. The shim pre-loads that module through a stub package,
aliases the missing name and then imports the real package. Nothing in the reference tree
is modified. Used by make_golden.py only; never at test or run time.
"""
from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path


def import_reference(src: Path):
    pkg_dir = src / "jakal_net"
    stub = types.ModuleType("jakal_net")
    stub.__path__ = [str(pkg_dir)]
    sys.modules["jakal_net"] = stub
    common = importlib.import_module("jakal_net._architectural_common")
    if not hasattr(common, "unit_normalize_values"):
        common.unit_normalize_values = common.normalize_value_directions
    del sys.modules["jakal_net"]
    for name in list(sys.modules):
        if name.startswith("jakal_net.") and name != "jakal_net._architectural_common":
            del sys.modules[name]
    sys.path.insert(0, str(src))
    pkg = importlib.import_module("jakal_net")
    return pkg
