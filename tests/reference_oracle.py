"""Access to the installed reference package (``baseline/_ref``) as an oracle.

Tests that compare against the reference skip when it is not installed.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def require_reference():
    if not os.path.isdir(os.path.join(REF, "optimizer_design")):
        pytest.skip("reference package not installed in baseline/_ref")
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
