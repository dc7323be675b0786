"""Loader for the in-tree sm_100a extension (``rational_optimizer_b200._C``).

CUDA tensors always go through the native kernels: if the extension is
missing on a machine with a GPU, :func:`ext` raises instead of silently
falling back to PyTorch.  CPU tensors use the PyTorch reference paths, which
double as the fp32 oracles of the test-suite.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return
    try:
        _C = importlib.import_module("rational_optimizer_b200._C")
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERR = exc


def available() -> bool:
    _load()
    return _C is not None


def ext():
    """Return the compiled module or raise a descriptive error."""
    _load()
    if _C is None:
        raise RuntimeError(
            "rational_optimizer_b200._C is not built; run "
            "`python setup.py build_ext --inplace` (sm_100a) before using CUDA tensors"
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
