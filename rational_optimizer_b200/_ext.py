"""Loader for the in-tree sm_100a extension (``rational_optimizer_b200._C``;
``rational_optimizer_b200._C_checked``, the bounds-checked build, when
``RO_CHECKED=1``).

CUDA tensors always go through the native kernels: if the extension is
missing on a machine with a GPU, :func:`ext` raises instead of silently
falling back to PyTorch.  CPU tensors use the PyTorch reference paths, which
double as the fp32 oracles of the test-suite.
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return
    try:
        import torch  # noqa: F401  (loads libc10 / libtorch that the extension links against)
        _C = importlib.import_module(module_name())
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERR = exc


def module_name() -> str:
    checked = os.environ.get("RO_CHECKED", "0") == "1"
    return "rational_optimizer_b200._C_checked" if checked else "rational_optimizer_b200._C"


def available() -> bool:
    _load()
    return _C is not None


def ext():
    """Return the compiled module or raise a descriptive error."""
    _load()
    if _C is None:
        raise RuntimeError(
            f"{module_name()} is not built; run `python setup.py build_ext --inplace` (sm_100a; "
            "with RO_BOUNDS_CHECK=1 for the checked build) before using CUDA tensors"
        ) from _ERR
    return _C


DTYPE_CODE = {"float32": 0, "bfloat16": 1}


def dtype_code(dtype) -> int:
    import torch

    if dtype == torch.float32:
        return 0
    if dtype == torch.bfloat16:
        return 1
    raise TypeError(f"unsupported dtype {dtype}")
