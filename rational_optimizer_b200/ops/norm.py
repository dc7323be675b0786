"""RMSNorm ``y = w * x * rsqrt(mean(x^2) + eps)`` (training/train.py:24-31).

CUDA: one fused kernel each way (``csrc/nn_ops.cu``); the residual stream can
stay fp32 while the normalised output is written in bf16 for the next GEMM.
The weight gradient uses a deterministic two-stage column reduction.
"""
from __future__ import annotations

import torch

from .._ext import dtype_code, ext


class _RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype):
        d = x.shape[-1]
        x2 = x.reshape(-1, d).contiguous()
        w = weight.detach().float().contiguous()
        y, rstd = ext().rmsnorm_forward(x2, w, float(eps), dtype_code(out_dtype))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        ctx.wdtype = weight.dtype
        return y.reshape(*x.shape[:-1], d)

    @staticmethod
    def backward(ctx, gy):
        x2, w, rstd = ctx.saved_tensors
        g2 = gy.reshape(-1, x2.shape[-1]).contiguous()
        dx, dw = ext().rmsnorm_backward(g2, x2, w, rstd)
        return dx.reshape(ctx.shape), dw.to(ctx.wdtype), None, None


def rms_norm_reference(x, weight, eps):
    return weight * x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)


def rms_norm(x, weight, eps=1e-6, out_dtype=None):
    if not x.is_cuda:
        y = rms_norm_reference(x, weight, eps)
        return y if out_dtype is None else y.to(out_dtype)
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if x.dtype == torch.bfloat16 and out_dtype == torch.float32:
        x = x.float()
    return _RMSNormFunction.apply(x, weight, eps, out_dtype)
