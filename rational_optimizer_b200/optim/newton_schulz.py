"""Newton-Schulz (quintic, 5 steps) polar maps used by Muon and TILLER.

Semantics follow the reference exactly:
  * 2-D literal Muon path (optimizer_design/_tiller/core.py:12-26): bf16,
    transpose tall matrices, divide by the Frobenius norm, 5 iterations of
    ``X <- a X + (b A + c A^2) X`` with ``A = X X^T`` and (a, b, c) =
    (3.4445, -4.775, 2.0315);
  * batched path (core.py:571-585), the fp32 norm is taken of the bf16 copy;
  * rational-group blocks (core.py:3303-3325): one NS5 per ``[w, d]`` (or
    ``[d, w]``) GRAIN group block, rescaled by sqrt(global_rank / (G*block_rank));
  * attention head groups (core.py:3327-3344): QKV as 3 x 4 blocks of 4 heads
    (x 1/sqrt(3)), the output projection as 4 column blocks.
On CUDA the batched GEMMs go through :mod:`rational_optimizer_b200.ops.gemm`
(batched tcgen05 kernel when built for the shape).
"""
from __future__ import annotations

import math
import os

import torch

from .. import _ext

NS_COEFFICIENTS = (3.4445, -4.775, 2.0315)
LAST_PATH = None  # "native" (tcgen05 GEMMs) or "cublas": the last CUDA ns5_grouped_bf16
NS_EPS = 1e-7
ATTENTION_HEADS = 16
ATTENTION_HEAD_GROUP_SIZE = 4


def match_rms_adamw_adjustment(shape) -> float:
    if len(shape) != 2:
        raise RuntimeError("TILLER Muon adjustment requires a matrix")
    return 0.2 * math.sqrt(float(max(shape)))


def zeropower_via_newton_schulz(matrix: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """Literal torch.optim.Muon NS5 on one matrix (bf16 result)."""
    if matrix.ndim != 2 or steps != 5:
        raise RuntimeError("TILLER requires a 2D NS5 input")
    a, b, c = NS_COEFFICIENTS
    value = matrix.bfloat16()
    transposed = value.shape[0] > value.shape[1]
    if transposed:
        value = value.T
    value = value / value.norm().clamp(min=NS_EPS)
    for _ in range(steps):
        gram = value @ value.T
        update = torch.addmm(gram, gram, gram, beta=b, alpha=c)
        value = torch.addmm(value, update, value, beta=a)
    return value.T if transposed else value


def _ns5_torch_bf16(work: torch.Tensor) -> torch.Tensor:
    a, b, c = NS_COEFFICIENTS
    for _ in range(5):
        gram = torch.bmm(work, work.transpose(1, 2))
        poly = torch.baddbmm(gram, gram, gram, beta=b, alpha=c)
        work = torch.baddbmm(work, poly, work, beta=a)
    return work


def ns5_grouped_bf16(x16: torch.Tensor, *, native: bool | None = None) -> torch.Tensor:
    """NS5 of a contiguous bf16 batch ``[B, r, c]`` with ``r <= c`` (bf16 result).

    CUDA: the Frobenius normalisation kernel followed by, per iteration,
    ``A = X X^T``; ``P = b A + c A A``; ``X = a X + P X``.  ``native`` selects
    the package's batched tcgen05 GEMMs, whose epilogue reads the addend
    directly (the default; ``RO_NATIVE_NS=0`` selects cuBLAS batched GEMMs,
    which first copy the addend into the output).  Shapes the kernel does
    not take (row strides that are not a multiple of 16 bytes) use cuBLAS;
    :data:`LAST_PATH` records which ran last.
    """
    global LAST_PATH
    if x16.shape[-2] > x16.shape[-1]:
        raise RuntimeError("ns5_grouped_bf16 expects wide blocks")
    if _ext.available() and x16.is_cuda and hasattr(_ext.ext(), "ns_normalize"):
        C = _ext.ext()
        work = C.ns_normalize(x16.contiguous())
        if native is None:
            native = _native_ns_enabled()
        if native and hasattr(C, "gemm_bf16_ex"):
            out = _ns5_native_bf16(C, work)
            if out is not None:
                LAST_PATH = "native"
                return out
        LAST_PATH = "cublas"
        return _ns5_torch_bf16(work)
    work = x16.to(torch.bfloat16)
    norm = torch.linalg.vector_norm(work.float(), dim=(-2, -1), keepdim=True).clamp_min(NS_EPS)
    return _ns5_torch_bf16(work / norm.to(work.dtype))


def _ns5_native_bf16(C, work):
    a, b, c = NS_COEFFICIENTS
    for _ in range(5):
        gram = C.gemm_bf16(work, work, False, True, False)
        poly = C.gemm_bf16_ex(gram, gram, False, True, False, gram, c, b) if gram is not None else None
        nxt = C.gemm_bf16_ex(poly, work, False, False, False, work, 1.0, a) if poly is not None else None
        if nxt is None:
            return None
        work = nxt
    return work


def _native_ns_enabled() -> bool:
    return os.environ.get("RO_NATIVE_NS", "1") == "1"


def _native_gemm_enabled() -> bool:
    from ..ops import gemm as _g
    return _g._NATIVE and hasattr(_ext.ext(), "gemm_bf16")


def batched_zero_power(momentum: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """NS5 on ``[batch, rows, cols]`` (bf16 result, same shape)."""
    if momentum.ndim != 3:
        raise RuntimeError(f"expected [batch, rows, cols], got {tuple(momentum.shape)}")
    transposed = momentum.shape[-2] > momentum.shape[-1]
    work = momentum.transpose(-2, -1) if transposed else momentum
    if work.is_cuda and int(steps) == 5:
        # normalisation kernel + batched GEMMs (same arithmetic as below)
        out = ns5_grouped_bf16(work.to(dtype=torch.bfloat16).contiguous())
        return out.transpose(-2, -1) if transposed else out
    work = work.to(dtype=torch.bfloat16)
    norm = torch.linalg.vector_norm(work.float(), dim=(-2, -1), keepdim=True).clamp_min(NS_EPS)
    work = work / norm.to(dtype=work.dtype)
    a, b, c = NS_COEFFICIENTS
    for _ in range(int(steps)):
        gram = torch.bmm(work, work.transpose(1, 2))
        poly = torch.baddbmm(gram, gram, gram, beta=b, alpha=c)
        work = torch.baddbmm(work, poly, work, beta=a)
    return work.transpose(-2, -1) if transposed else work


def rational_group_zero_power(source: torch.Tensor, steps: int, *, groups: int,
                              width: int) -> torch.Tensor:
    """NS5 per GRAIN group block of ``[L, rows, cols]`` (incoming or outgoing)."""
    if source.ndim != 3 or int(steps) != 5:
        raise RuntimeError("rational-group polar requires [layers,rows,cols] NS5")
    layers, rows, cols = map(int, source.shape)
    groups, width = int(groups), int(width)
    if groups <= 0 or width <= 0:
        raise ValueError("rational-group polar dimensions must be positive")
    hidden = groups * width
    if rows == hidden:
        blocks = source.reshape(layers * groups, width, cols)
        polar = batched_zero_power(blocks, steps).reshape(layers, rows, cols)
        block_rank = min(width, cols)
    elif cols == hidden:
        blocks = source.reshape(layers, rows, groups, width).permute(0, 2, 1, 3)
        blocks = blocks.reshape(layers * groups, rows, width)
        polar = batched_zero_power(blocks, steps).reshape(layers, groups, rows, width)
        polar = polar.permute(0, 2, 1, 3).reshape(layers, rows, cols)
        block_rank = min(rows, width)
    else:
        raise RuntimeError("rational-group polar cannot identify grouped axis")
    global_rank = min(rows, cols)
    return polar.mul(math.sqrt(float(global_rank) / float(groups * block_rank)))


def attention_head_group_zero_power(source: torch.Tensor, steps: int, *,
                                    heads: int = ATTENTION_HEADS,
                                    head_group_size: int = ATTENTION_HEAD_GROUP_SIZE) -> torch.Tensor:
    """NS5 per group of ``head_group_size`` heads for QKV ``[L,3d,d]`` or out ``[L,d,d]``."""
    if source.ndim != 3 or int(steps) != 5:
        raise RuntimeError("attention head-group polar requires batched NS5")
    layers, rows, cols = map(int, source.shape)
    if cols % int(heads) or int(heads) % int(head_group_size):
        raise RuntimeError("attention head-group inventory is not divisible")
    head_width = cols // int(heads)
    group_count = int(heads) // int(head_group_size)
    block = int(head_group_size) * head_width
    if rows == 3 * cols:
        blocks = source.reshape(layers * 3 * group_count, block, cols)
        polar = batched_zero_power(blocks, steps).reshape(layers, rows, cols)
        return polar.mul(1.0 / math.sqrt(3.0))
    if rows == cols:
        blocks = source.reshape(layers, rows, group_count, block).permute(0, 2, 1, 3)
        blocks = blocks.reshape(layers * group_count, rows, block)
        polar = batched_zero_power(blocks, steps).reshape(layers, group_count, rows, block)
        return polar.permute(0, 2, 1, 3).reshape(layers, rows, cols)
    raise RuntimeError("attention head-group polar supports only QKV/output roles")
