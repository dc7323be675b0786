"""Fused ``lm_head`` projection + mean cross-entropy.

The logits of a row chunk are produced by one GEMM, a single kernel turns
them into ``(softmax - onehot) / N`` in place while emitting the row losses,
and the two gradient GEMMs consume the chunk immediately, so the full
``[N, vocab]`` logit tensor (3.3 GB at N=32768, V=50304 in bf16) never
exists.  Equivalent to ``F.cross_entropy(h @ W^T, y)`` (training/train.py:
2868-2870); the backward only rescales the stored gradients by the upstream
scalar.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._ext import ext
from . import gemm
from .linear import managed_grad, report_ready

DEFAULT_CHUNK_ROWS = 8192


class _LinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, w_compute, target, chunk_rows, ignore_index):
        C = ext()
        n = h.shape[0]
        valid = n if ignore_index is None else int((target != ignore_index).sum().item())
        scale = 1.0 / max(valid, 1)
        ign = -100 if ignore_index is None else int(ignore_index)
        hc = h if h.dtype == w_compute.dtype else h.to(w_compute.dtype)
        dh = torch.empty_like(hc)
        dw = None
        loss_rows = torch.empty(n, device=h.device, dtype=torch.float32)
        for start in range(0, n, chunk_rows):
            stop = min(n, start + chunk_rows)
            hs = hc[start:stop]
            logits = gemm.matmul_nt(hs, w_compute)
            loss_rows[start:stop] = C.cross_entropy_fwd_bwd(logits, target[start:stop].contiguous(),
                                                            scale, ign)
            dh[start:stop] = gemm.matmul_nn(logits, w_compute)
            # the first chunk writes the fp32 weight gradient, later ones add to
            # it inside the GEMM (no zero fill, no temporaries, no separate adds)
            if dw is None:
                dw = gemm.matmul_tn(logits, hs, out_dtype=torch.float32)
            else:
                gemm.matmul_tn_accumulate_(dw, logits, hs)
        if dw is None:
            dw = torch.zeros(weight.shape, device=h.device, dtype=torch.float32)
        ctx.save_for_backward(dh, dw)
        ctx.weight = weight
        ctx.h_dtype = h.dtype
        ctx.w_dtype = weight.dtype
        return loss_rows.sum() * scale

    @staticmethod
    def backward(ctx, go):
        dh, dw = ctx.saved_tensors
        gh = (dh * go.to(dh.dtype)).to(ctx.h_dtype) if ctx.needs_input_grad[0] else None
        if not ctx.needs_input_grad[1]:
            return gh, None, None, None, None, None
        buf = managed_grad(ctx.weight)
        if buf is not None and ctx.w_dtype == torch.float32:
            # grad += dw * go in one pass over the managed fp32 gradient buffer
            buf.addcmul_(dw, go.to(buf.dtype))
            report_ready(ctx.weight)
            return gh, None, None, None, None, None
        return gh, (dw * go).to(ctx.w_dtype), None, None, None, None


def linear_cross_entropy(h, weight, target, *, w_compute=None, chunk_rows=DEFAULT_CHUNK_ROWS,
                         ignore_index=None):
    """mean CE of ``h @ weight^T`` against ``target`` (h: [N, d], target: [N])."""
    if not h.is_cuda:
        logits = h.float() @ weight.float().t()
        if ignore_index is None:
            return F.cross_entropy(logits, target)
        return F.cross_entropy(logits, target, ignore_index=ignore_index)
    if w_compute is None:
        w_compute = weight.detach().to(torch.bfloat16)
    return _LinearCrossEntropy.apply(h, weight, w_compute, target, int(chunk_rows), ignore_index)
