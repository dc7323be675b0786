"""Muon with batched Newton-Schulz (reference baseline: ``torch.optim.Muon``,
training/train.py:1808-1850).

Same constructor, defaults, parameter-group keys and ``momentum_buffer``
state as ``torch.optim.Muon``; the step groups parameters of equal shape and
runs one batched NS5 per shape
(:func:`~rational_optimizer_b200.optim.newton_schulz.batched_zero_power`)
instead of one small NS5 per matrix.
"""
from __future__ import annotations

import torch

from .newton_schulz import batched_zero_power


def adjust_lr(lr, adjust_lr_fn, shape):
    a, b = shape[:2]
    if adjust_lr_fn is None or adjust_lr_fn == "original":
        return lr * max(1.0, a / b) ** 0.5
    if adjust_lr_fn == "match_rms_adamw":
        return lr * 0.2 * max(a, b) ** 0.5
    return lr


class Muon(torch.optim.Muon):
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr = float(group["lr"])
            wd = float(group["weight_decay"])
            mu = float(group["momentum"])
            by_shape = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.ndim != 2:
                    raise ValueError("Param gradient must be a 2D matrix")
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p.grad, memory_format=torch.preserve_format)
                by_shape.setdefault(tuple(p.shape), []).append(p)
            for shape, ps in by_shape.items():
                grads = [p.grad for p in ps]
                bufs = [self.state[p]["momentum_buffer"] for p in ps]
                torch._foreach_lerp_(bufs, grads, 1.0 - mu)
                upd = torch._foreach_lerp(grads, bufs, mu) if group["nesterov"] else bufs
                polar = batched_zero_power(torch.stack(upd), int(group["ns_steps"]))
                alr = adjust_lr(lr, group["adjust_lr_fn"], shape)
                torch._foreach_mul_(ps, 1.0 - lr * wd)
                torch._foreach_add_(ps, list(polar.to(ps[0].dtype).unbind(0)), alpha=-alr)
        return loss
