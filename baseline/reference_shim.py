"""Imports the staged reference Jakal-Net package (test and baseline infrastructure only).

The shipped package fails to import: ``jakal_net/transition.py`` imports
``unit_normalize_values`` from ``jakal_net/_architectural_common.py``, which only defines
``normalize_value_directions``. ``import_reference`` pre-loads that module through a stub
package, aliases the missing name and then imports the real package. Nothing in the
reference tree is modified.

Callers: tests (the drop-in tests through the reference's loader, fixture generation) and
bench.py's reference arm. The product package never imports the reference.
"""
from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

STAGED = Path(__file__).resolve().parent / "_ref"


def available(src: Path = STAGED) -> bool:
    return (src / "jakal_net" / "__init__.py").is_file()


def import_reference(src: Path = STAGED):
    """Returns the imported ``jakal_net`` package from ``src`` (a folder holding
    ``jakal_net/``), applying the import-name alias described above."""
    pkg_dir = src / "jakal_net"
    if "jakal_net" in sys.modules and getattr(sys.modules["jakal_net"], "__file__", None):
        return sys.modules["jakal_net"]
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
    if str(src) not in sys.path:
        sys.path.insert(0, str(src))
    pkg = importlib.import_module("jakal_net")
    # The pre-loaded _architectural_common still holds the classes of the stub-time import of
    # jakal_net.modules; re-executing it in place binds the package's own classes (functions
    # other modules imported from it read its globals, so they follow), and keeps the alias.
    common = importlib.reload(sys.modules["jakal_net._architectural_common"])
    if not hasattr(common, "unit_normalize_values"):
        common.unit_normalize_values = common.normalize_value_directions
    return pkg


def import_progressive_b(src: Path = STAGED):
    """Imports the staged ``progressive_b_example`` model script (needs the package)."""
    import_reference(src)
    if str(src) not in sys.path:
        sys.path.insert(0, str(src))
    return importlib.import_module("progressive_b_example")
