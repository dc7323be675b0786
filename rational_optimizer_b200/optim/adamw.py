"""AdamW with a single multi-tensor sm_100a kernel on CUDA.

State layout and hyper-parameters are exactly ``torch.optim.AdamW``'s
(``step``, ``exp_avg``, ``exp_avg_sq``; decoupled weight decay
``p <- p (1 - lr wd)``; bias-corrected ``m / (sqrt(v / bc2) + eps)``) so
checkpoints interchange with the reference, which uses torch's AdamW
(training/train.py:1737-1743).  On CUDA every parameter of every group is
updated by one launch of ``adamw_multi_tensor`` (csrc/optim.cu); on CPU the
torch implementation runs.
"""
from __future__ import annotations

import torch
from torch.autograd.graph import increment_version

from .. import _ext


class FusedAdamW(torch.optim.AdamW):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, **kw):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                         foreach=False, **kw)

    def eager_step_required(self):
        """No probes are recorded in the forward/backward: always graph-eligible."""
        return False

    def _native(self):
        if not _ext.available():
            return None
        C = _ext.ext()
        return C if hasattr(C, "adamw_multi_tensor") else None

    @torch.no_grad()
    def step(self, closure=None):
        C = self._native()
        params = [p for g in self.param_groups for p in g["params"] if p.grad is not None]
        if C is None or not params or not params[0].is_cuda:
            return super().step(closure)
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            ps, gs, ms, vs = [], [], [], []
            step_value = None
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if len(st) == 0:
                    st["step"] = torch.tensor(0.0, dtype=torch.float32)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                step_value = float(st["step"])
                ps.append(p)
                gs.append(p.grad)
                ms.append(st["exp_avg"])
                vs.append(st["exp_avg_sq"])
            if not ps:
                continue
            beta1, beta2 = group["betas"]
            C.adamw_multi_tensor(ps, gs, ms, vs, float(group["lr"]), float(beta1), float(beta2),
                                 float(group["eps"]), float(group["weight_decay"]), step_value)
            # the kernel wrote the parameters in place: bump their version counters
            # so version-keyed caches (the bf16 weight casts) see the update
            for p in ps:
                increment_version(p)
        return loss
