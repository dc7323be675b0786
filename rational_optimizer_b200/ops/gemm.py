"""GEMM entry points used by the model and the optimizers.

``matmul_nt(a, b)`` = a @ b^T, ``matmul_nn(a, b)`` = a @ b,
``matmul_tn(a, b)`` = a^T @ b, and the batched ``bmm``/``baddbmm`` forms used
by Newton-Schulz.  Shapes the tcgen05 kernel (``csrc/gemm_sm100.cu``)
supports are routed to it; anything else uses cuBLAS through PyTorch.
"""
from __future__ import annotations

import os
import warnings

import torch

from .. import _ext

_NATIVE = os.environ.get("RO_NATIVE_GEMM", "0") == "1"


def _native():
    if not _NATIVE or not _ext.available():
        return None
    C = _ext.ext()
    return C if hasattr(C, "gemm_bf16") else None


def _native_ok(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16)


def matmul_nt(a: torch.Tensor, b: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """a [M, K] @ b[N, K]^T -> [M, N]."""
    C = _native()
    if C is not None and _native_ok(a, b):
        out = C.gemm_bf16(a, b, False, True, out_dtype is torch.float32)
        if out is not None:
            return out
    if out_dtype is not None and out_dtype != a.dtype and a.is_cuda:
        return torch.mm(a, b.t(), out_dtype=out_dtype)
    out = a @ b.t()
    return out if out_dtype is None else out.to(out_dtype)


def matmul_nn(a: torch.Tensor, b: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """a [M, K] @ b [K, N] -> [M, N]."""
    C = _native()
    if C is not None and _native_ok(a, b):
        out = C.gemm_bf16(a, b, False, False, out_dtype is torch.float32)
        if out is not None:
            return out
    if out_dtype is not None and out_dtype != a.dtype and a.is_cuda:
        return torch.mm(a, b, out_dtype=out_dtype)
    out = a @ b
    return out if out_dtype is None else out.to(out_dtype)


def matmul_tn(a: torch.Tensor, b: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """a [K, M]^T @ b [K, N] -> [M, N] (weight gradients: dy^T x)."""
    C = _native()
    if C is not None and _native_ok(a, b):
        out = C.gemm_bf16(a, b, True, False, out_dtype is torch.float32)
        if out is not None:
            return out
    if out_dtype is not None and out_dtype != a.dtype and a.is_cuda:
        return torch.mm(a.t(), b, out_dtype=out_dtype)
    out = a.t() @ b
    return out if out_dtype is None else out.to(out_dtype)


_ADDMM_DTYPE_OUT = True
# Which form the last CUDA weight-gradient accumulation took: "addmm_fp32_out"
# (one GEMM with beta = 1 writing fp32 in place) or "gemm_then_add" (a
# separate fp32 GEMM output added into the buffer: 8 more bytes per element).
ACCUMULATE_PATH = None


def matmul_tn_accumulate_(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``out += a^T @ b`` with bf16 operands and an fp32 ``out`` (weight-gradient
    accumulation straight into a gradient buffer, beta = 1 in the GEMM)."""
    global _ADDMM_DTYPE_OUT, ACCUMULATE_PATH
    if _ADDMM_DTYPE_OUT and a.is_cuda and out.dtype == torch.float32 and a.dtype != torch.float32:
        try:
            result = torch.addmm(out, a.t(), b, out_dtype=torch.float32, out=out)
            ACCUMULATE_PATH = "addmm_fp32_out"
            return result
        except (RuntimeError, TypeError) as exc:
            _ADDMM_DTYPE_OUT = False
            warnings.warn(f"fp32-output addmm is unavailable ({exc}); weight gradients fall back to a "
                          "separate GEMM and an add", RuntimeWarning)
    if a.is_cuda:
        ACCUMULATE_PATH = "gemm_then_add"
    return out.add_(matmul_tn(a, b, out_dtype=out.dtype))
