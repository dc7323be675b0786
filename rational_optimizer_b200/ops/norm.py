"""RMSNorm ``y = w * x * rsqrt(mean(x^2) + eps)`` (training/train.py:24-31).

CUDA: one fused kernel each way (``csrc/nn_ops.cu``); the residual stream can
stay fp32 while the normalised output is written in bf16 for the next GEMM.
The weight gradient uses a deterministic two-stage column reduction.
"""
from __future__ import annotations

import torch

from .linear import managed_grad, report_ready
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


class _AddRMSNormFunction(torch.autograd.Function):
    """(x_new, y) = (x + delta, rmsnorm(x + delta)); x fp32, delta/y bf16."""

    @staticmethod
    def forward(ctx, x, delta, weight, eps):
        d = x.shape[-1]
        x2 = x.reshape(-1, d).contiguous()
        dl = delta.reshape(-1, d).contiguous()
        w = weight.detach().float().contiguous()
        x_new, y, rstd = ext().add_rmsnorm_forward(x2, dl, w, float(eps))
        ctx.save_for_backward(x_new, w, rstd)
        ctx.shape = x.shape
        ctx.wdtype = weight.dtype
        ctx.weight = weight
        return x_new.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, dx_new, dy):
        x_new, w, rstd = ctx.saved_tensors
        d = x_new.shape[-1]
        if dy is None:
            dy = torch.zeros(x_new.shape, device=x_new.device, dtype=torch.bfloat16)
        dres = None if dx_new is None else dx_new.reshape(-1, d).float().contiguous()
        into = managed_grad(ctx.weight) if ctx.needs_input_grad[2] else None
        dx, ddelta, dw = ext().add_rmsnorm_backward(dy.reshape(-1, d).to(torch.bfloat16).contiguous(),
                                                    dres, x_new, w, rstd, True, into)
        if into is not None:
            # the weight gradient was added into the managed buffer by the reduction
            report_ready(ctx.weight)
            return dx.view(ctx.shape), ddelta.view(ctx.shape), None, None
        return dx.view(ctx.shape), ddelta.view(ctx.shape), dw.to(ctx.wdtype), None


def add_rms_norm(x, delta, weight, eps=1e-6):
    """Fused ``x_new = x + delta`` and ``rmsnorm(x_new)`` (bf16 output) on CUDA."""
    if delta is None:
        return x, rms_norm(x, weight, eps, torch.bfloat16 if x.is_cuda else None)
    if not x.is_cuda:
        x_new = x + delta
        return x_new, rms_norm_reference(x_new, weight, eps)
    return _AddRMSNormFunction.apply(x.float(), delta.to(torch.bfloat16), weight, eps)


def fused_add_norm_supported(x) -> bool:
    return x.is_cuda and x.shape[-1] % 256 == 0 and x.shape[-1] <= 1024


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
