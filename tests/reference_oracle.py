"""Access to the installed reference package (``baseline/_ref``) as an oracle.

When the package is missing it is installed once, the way the benchmark's
reference arm does it (``bench.ensure_reference``: the unmodified reference
tree, ``pip install --no-index --target baseline/_ref``); tests that compare
against the reference skip only when that is impossible on this machine.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


_INSTALL = {}


def _install_once():
    """None when the reference package is (now) installed, else why not."""
    if "reason" not in _INSTALL:
        if ROOT not in sys.path:
            sys.path.insert(0, ROOT)
        import bench
        _INSTALL["reason"] = bench.ensure_reference()
    return _INSTALL["reason"]


def require_reference():
    if not os.path.isdir(os.path.join(REF, "optimizer_design")):
        reason = _install_once()
        if reason is not None or not os.path.isdir(os.path.join(REF, "optimizer_design")):
            pytest.skip(f"reference package not installed in baseline/_ref ({reason})")
    os.environ["RATIONAL_OPT_TORCH_FALLBACK"] = "1"
    if REF not in sys.path:
        sys.path.append(REF)
    return {
        "train": importlib.import_module("training.train"),
        "entry": importlib.import_module("experiments.protocol.method_entrypoint"),
        "core": importlib.import_module("optimizer_design._tiller.core"),
        "tiller": importlib.import_module("optimizer_design._tiller"),
        "rational": importlib.import_module("rational_opt.rational"),
    }
