"""Published optimizer baselines: Lion, AdEMAMix, Schedule-Free AdamW,
CAME-style AdamW and SOAP-style AdamW (reference
training/baseline_optimizers.py:56-460, constructed by training/train.py:1726-1806).

Update rules, hyper-parameter names, defaults and per-parameter state keys
are those of the reference, so checkpoints interchange and the trainer flags
(``--ademamix-*``, ``--came-*``, ``--soap-*``, ``--schedule-free-*``,
``--factored-*``) mean the same thing.  Execution differs: every elementwise
rule runs as multi-tensor ``torch._foreach_*`` kernels over a whole parameter
group (one launch per arithmetic stage for all tensors, instead of one per
tensor), and the matrix rules (CAME's factored moments, SOAP's rotations)
batch their GEMMs per parameter on the tensor cores.
"""
from __future__ import annotations

import math

import torch
from torch.optim import Optimizer


def _decoupled_decay_(params, lr, weight_decay):
    if weight_decay != 0.0 and params:
        torch._foreach_mul_(params, 1.0 - lr * weight_decay)


def _factored_second_moment(row, col, eps):
    """Rank-one second-moment estimate row_mean * col_mean / global_mean."""
    row_mean = row.mean(dim=-1, keepdim=True).clamp_min(eps)
    col_mean = col.mean(dim=-2, keepdim=True).clamp_min(eps)
    global_mean = row_mean.mean().clamp_min(eps)
    return row_mean * col_mean / global_mean


def ademamix_linear_warmup(step, value_end, value_start, warmup_steps):
    """alpha schedule: linear from ``value_start`` to ``value_end`` over the warm-up."""
    if warmup_steps is None or int(warmup_steps) <= 0 or step >= int(warmup_steps):
        return float(value_end)
    mix = float(step) / float(warmup_steps)
    return (1.0 - mix) * float(value_start) + mix * float(value_end)


def ademamix_half_life_warmup(step, beta_end, beta_start, warmup_steps):
    """beta3 schedule: the EMA half-life moves linearly from beta_start's to beta_end's."""
    if warmup_steps is None or int(warmup_steps) <= 0 or step >= int(warmup_steps):
        return float(beta_end)

    def half_life(beta):
        beta = min(max(float(beta), 1e-8), 1.0 - 1e-12)
        return math.log(0.5) / math.log(beta) - 1.0

    mix = float(step) / float(warmup_steps)
    h = (1.0 - mix) * half_life(beta_start) + mix * half_life(beta_end)
    return math.pow(0.5, 1.0 / (h + 1.0))


def resolve_ademamix_warmup(value, steps):
    """Negative: 15% of the run (at least one step); 0 or None: off; else as given
    (training/train.py:1716-1723)."""
    if value is None:
        return None
    value = int(value)
    if value < 0:
        return max(1, int(round(0.15 * int(steps))))
    return value if value > 0 else None


def _with_grads(group):
    params, grads = [], []
    for p in group["params"]:
        if p.grad is None:
            continue
        if p.grad.is_sparse:
            raise RuntimeError("sparse gradients are not supported")
        params.append(p)
        grads.append(p.grad)
    return params, grads


class Lion(Optimizer):
    """Lion: sign of an interpolated momentum, decoupled weight decay."""

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.99), weight_decay=0.0):
        super().__init__(params, dict(lr=lr, betas=betas, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            params, grads = _with_grads(group)
            if not params:
                continue
            lr = float(group["lr"])
            beta1, beta2 = group["betas"]
            bufs = []
            for p in params:
                st = self.state[p]
                if not st:
                    st["exp_avg"] = torch.zeros_like(p)
                bufs.append(st["exp_avg"])
            _decoupled_decay_(params, lr, float(group["weight_decay"]))
            upd = torch._foreach_mul(bufs, beta1)
            torch._foreach_add_(upd, grads, alpha=1.0 - beta1)
            torch._foreach_sign_(upd)
            torch._foreach_add_(params, upd, alpha=-lr)
            torch._foreach_mul_(bufs, beta2)
            torch._foreach_add_(bufs, grads, alpha=1.0 - beta2)
        return loss


class AdEMAMix(Optimizer):
    """AdEMAMix: Adam plus an un-bias-corrected slow EMA weighted by ``alpha``.

    ``alpha_warmup`` ramps alpha linearly from 0; ``beta3_warmup`` moves the
    slow EMA's half-life from beta1's to beta3's.
    """

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.999, 0.9999), eps=1e-8, weight_decay=0.0,
                 alpha=5.0, beta3_warmup=None, alpha_warmup=None):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      alpha=alpha, beta3_warmup=beta3_warmup,
                                      alpha_warmup=alpha_warmup))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            params, grads = _with_grads(group)
            if not params:
                continue
            lr = float(group["lr"])
            beta1, beta2, beta3_final = group["betas"]
            eps = float(group["eps"])
            # tensors that share a step count are updated together
            by_step = {}
            for p, g in zip(params, grads):
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg_fast"] = torch.zeros_like(p) if beta1 != 0.0 else None
                    st["exp_avg_slow"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                st["step"] += 1
                by_step.setdefault(int(st["step"]), []).append((p, g, st))
            for step, items in by_step.items():
                ps = [i[0] for i in items]
                gs = [i[1] for i in items]
                slow = [i[2]["exp_avg_slow"] for i in items]
                sq = [i[2]["exp_avg_sq"] for i in items]
                alpha = ademamix_linear_warmup(step, float(group["alpha"]), 0.0, group.get("alpha_warmup"))
                beta3 = ademamix_half_life_warmup(step, beta3_final, beta1, group.get("beta3_warmup"))
                _decoupled_decay_(ps, lr, float(group["weight_decay"]))
                if beta1 != 0.0:
                    fast = [i[2]["exp_avg_fast"] for i in items]
                    torch._foreach_mul_(fast, beta1)
                    torch._foreach_add_(fast, gs, alpha=1.0 - beta1)
                    upd = torch._foreach_div(fast, 1.0 - beta1 ** step)
                else:
                    upd = [g.clone() for g in gs]
                torch._foreach_mul_(slow, beta3)
                torch._foreach_add_(slow, gs, alpha=1.0 - beta3)
                torch._foreach_mul_(sq, beta2)
                torch._foreach_addcmul_(sq, gs, gs, value=1.0 - beta2)
                denom = torch._foreach_sqrt(sq)
                torch._foreach_div_(denom, math.sqrt(1.0 - beta2 ** step))
                torch._foreach_add_(denom, eps)
                torch._foreach_add_(upd, slow, alpha=alpha)
                torch._foreach_addcdiv_(ps, upd, denom, value=-lr)
        return loss


class ScheduleFreeAdamW(Optimizer):
    """Schedule-free AdamW with Polyak interpolation.

    The optimizer keeps the AdamW sequence ``z`` and its running average;
    gradients are taken at ``param = lerp(z, avg, beta1)``.
    """

    def __init__(self, params, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
                 warmup_steps=0):
        super().__init__(params, dict(lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                                      weight_decay=weight_decay, warmup_steps=warmup_steps))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            params, grads = _with_grads(group)
            if not params:
                continue
            lr = float(group["lr"])
            beta1, beta2 = float(group["beta1"]), float(group["beta2"])
            eps = float(group["eps"])
            warmup = int(group["warmup_steps"])
            by_step = {}
            for p, g in zip(params, grads):
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["z"] = p.detach().clone()
                    st["avg"] = p.detach().clone()
                    st["exp_avg_sq"] = torch.zeros_like(p)
                st["step"] += 1
                by_step.setdefault(int(st["step"]), []).append((p, g, st))
            for step, items in by_step.items():
                ps = [i[0] for i in items]
                gs = [i[1] for i in items]
                z = [i[2]["z"] for i in items]
                avg = [i[2]["avg"] for i in items]
                sq = [i[2]["exp_avg_sq"] for i in items]
                _decoupled_decay_(z, lr, float(group["weight_decay"]))
                torch._foreach_mul_(sq, beta2)
                torch._foreach_addcmul_(sq, gs, gs, value=1.0 - beta2)
                denom = torch._foreach_sqrt(sq)
                torch._foreach_div_(denom, math.sqrt(1.0 - beta2 ** step))
                torch._foreach_add_(denom, eps)
                torch._foreach_addcdiv_(z, gs, denom, value=-lr)
                if warmup > 0 and step <= warmup:
                    weight = 1.0 / float(step)
                else:
                    weight = 1.0 / float(max(1, step - warmup + 1))
                torch._foreach_mul_(avg, 1.0 - weight)
                torch._foreach_add_(avg, z, alpha=weight)
                torch._foreach_copy_(ps, torch._foreach_lerp(z, avg, beta1))
        return loss


class CAMEStyleAdamW(Optimizer):
    """AdamW with Adafactor-style factored second moments and a CAME
    confidence factor ``clamp(rsqrt(1 + scale * instability))``."""

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.999, 0.999), eps=1e-8, weight_decay=0.0,
                 factored_min_dim=128, clip_threshold=1.0, confidence_scale=1.0,
                 confidence_min=0.25, confidence_max=4.0):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      factored_min_dim=factored_min_dim,
                                      clip_threshold=clip_threshold,
                                      confidence_scale=confidence_scale,
                                      confidence_min=confidence_min,
                                      confidence_max=confidence_max))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr = float(group["lr"])
            beta1, beta2, beta3 = group["betas"]
            eps = float(group["eps"])
            wd = float(group["weight_decay"])
            min_dim = int(group["factored_min_dim"])
            clip = float(group["clip_threshold"])
            cscale = float(group["confidence_scale"])
            cmin, cmax = float(group["confidence_min"]), float(group["confidence_max"])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("CAMEStyleAdamW does not support sparse gradients")
                factored = p.dim() == 2 and min(p.shape) >= min_dim
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                    if factored:
                        kw = dict(device=p.device, dtype=torch.float32)
                        st["exp_avg_sq_row"] = torch.zeros(p.shape[0], 1, **kw)
                        st["exp_avg_sq_col"] = torch.zeros(1, p.shape[1], **kw)
                        st["instability_row"] = torch.zeros(p.shape[0], 1, **kw)
                        st["instability_col"] = torch.zeros(1, p.shape[1], **kw)
                    else:
                        st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
                        st["instability"] = torch.zeros_like(p, dtype=torch.float32)
                st["step"] += 1
                step = int(st["step"])
                b1, b2, b3 = 1.0 - beta1 ** step, 1.0 - beta2 ** step, 1.0 - beta3 ** step
                g = p.grad.detach().float()
                m = st["exp_avg"]
                m.mul_(beta1).add_(g, alpha=1.0 - beta1)
                g2 = g.square().add_(eps)
                if factored:
                    row, col = st["exp_avg_sq_row"], st["exp_avg_sq_col"]
                    row.mul_(beta2).add_(g2.mean(dim=1, keepdim=True), alpha=1.0 - beta2)
                    col.mul_(beta2).add_(g2.mean(dim=0, keepdim=True), alpha=1.0 - beta2)
                    v = _factored_second_moment(row / b2, col / b2, eps)
                    resid = (g2 - v).abs() / v.clamp_min(eps)
                    irow, icol = st["instability_row"], st["instability_col"]
                    irow.mul_(beta3).add_(resid.mean(dim=1, keepdim=True), alpha=1.0 - beta3)
                    icol.mul_(beta3).add_(resid.mean(dim=0, keepdim=True), alpha=1.0 - beta3)
                    inst = _factored_second_moment(irow / b3, icol / b3, eps)
                else:
                    sq = st["exp_avg_sq"]
                    sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
                    v = sq / b2
                    resid = (g2 - v).abs() / v.clamp_min(eps)
                    ist = st["instability"]
                    ist.mul_(beta3).add_(resid, alpha=1.0 - beta3)
                    inst = ist / b3
                upd = (m / b1) / v.sqrt().add(eps)
                upd = upd * (1.0 + cscale * inst).rsqrt().clamp(cmin, cmax)
                if clip > 0:
                    rms = torch.sqrt(upd.square().mean()).clamp_min(eps)
                    upd = upd / torch.clamp(rms / clip, min=1.0)
                if wd != 0.0:
                    p.mul_(1.0 - lr * wd)
                p.add_(upd.to(dtype=p.dtype), alpha=-lr)
        return loss


class SOAPStyleAdamW(Optimizer):
    """AdamW in the eigenbasis of Shampoo's factored preconditioners.

    Matrices whose larger side is at most ``large_side_identity_threshold``
    rotate their moments into the eigenbases of ``EMA(G G^T)`` and
    ``EMA(G^T G)`` (refreshed every ``precondition_frequency`` steps, moments
    carried across the basis change); all other tensors take plain AdamW.
    """

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0,
                 precondition_frequency=50, large_side_identity_threshold=2048, one_sided=False):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      precondition_frequency=precondition_frequency,
                                      large_side_identity_threshold=large_side_identity_threshold,
                                      one_sided=one_sided))

    @staticmethod
    def _eigenbasis(matrix, eps):
        m = matrix.float()
        m = 0.5 * (m + m.transpose(-1, -2))
        eye = torch.eye(m.shape[0], device=m.device, dtype=m.dtype)
        try:
            return torch.linalg.eigh(m + eps * eye)[1]
        except RuntimeError:
            return eye

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr = float(group["lr"])
            beta1, beta2 = group["betas"]
            eps = float(group["eps"])
            wd = float(group["weight_decay"])
            freq = max(1, int(group["precondition_frequency"]))
            limit = int(group["large_side_identity_threshold"])
            one_sided = bool(group["one_sided"])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("SOAPStyleAdamW does not support sparse gradients")
                soap = p.dim() == 2 and max(p.shape) <= limit and min(p.shape) > 1
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                    st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
                    if soap:
                        r, c = p.shape
                        kw = dict(device=p.device, dtype=torch.float32)
                        st["left_precond"] = torch.zeros(r, r, **kw)
                        st["right_precond"] = torch.zeros(c, c, **kw)
                        st["left_basis"] = torch.eye(r, **kw)
                        st["right_basis"] = torch.eye(c, **kw)
                st["step"] += 1
                step = int(st["step"])
                if wd != 0.0:
                    p.mul_(1.0 - lr * wd)
                b1, b2 = 1.0 - beta1 ** step, 1.0 - beta2 ** step
                m, v = st["exp_avg"], st["exp_avg_sq"]
                g = p.grad.detach().float()
                if not soap:
                    m.mul_(beta1).add_(g, alpha=1.0 - beta1)
                    v.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
                    denom = v.sqrt().div_(math.sqrt(b2)).add_(eps)
                    p.add_(((m / b1) / denom).to(dtype=p.dtype), alpha=-lr)
                    continue
                left, right = st["left_precond"], st["right_precond"]
                left.mul_(beta2).add_(g @ g.t(), alpha=1.0 - beta2)
                if not one_sided:
                    right.mul_(beta2).add_(g.t() @ g, alpha=1.0 - beta2)
                if step == 1 or step % freq == 0:
                    old_l, old_r = st["left_basis"], st["right_basis"]
                    new_l = self._eigenbasis(left, eps).to(device=p.device)
                    new_r = old_r if one_sided else self._eigenbasis(right, eps).to(device=p.device)
                    raw = old_l @ m @ old_r.t()
                    m.copy_(new_l.t() @ raw @ new_r)
                    v.zero_()
                    st["left_basis"], st["right_basis"] = new_l, new_r
                lb = st["left_basis"].to(device=p.device, dtype=torch.float32)
                rb = st["right_basis"].to(device=p.device, dtype=torch.float32)
                gr = lb.t() @ g @ rb
                m.mul_(beta1).add_(gr, alpha=1.0 - beta1)
                v.mul_(beta2).addcmul_(gr, gr, value=1.0 - beta2)
                upd = m.div(b1) / v.sqrt().div(math.sqrt(b2)).add(eps)
                p.add_((lb @ upd.float() @ rb.t()).to(dtype=p.dtype), alpha=-lr)
        return loss


def build(name, groups, args):
    """Construct the baseline named by the trainer's ``--optimizer`` flag."""
    if name == "lion":
        return Lion(groups, lr=args.lr, betas=(args.beta1, args.beta2), weight_decay=args.weight_decay)
    if name == "ademamix":
        return AdEMAMix(groups, lr=args.lr, betas=(args.beta1, args.beta2, args.ademamix_beta3),
                        eps=args.eps, weight_decay=args.weight_decay, alpha=args.ademamix_alpha,
                        beta3_warmup=resolve_ademamix_warmup(args.ademamix_beta3_warmup_steps, args.steps),
                        alpha_warmup=resolve_ademamix_warmup(args.ademamix_alpha_warmup_steps, args.steps))
    if name == "schedule_free_adamw":
        return ScheduleFreeAdamW(groups, lr=args.lr, beta1=args.schedule_free_beta1, beta2=args.beta2,
                                 eps=args.eps, weight_decay=args.weight_decay,
                                 warmup_steps=args.schedule_free_warmup_steps)
    if name == "adafactor_came":
        return CAMEStyleAdamW(groups, lr=args.lr, betas=(args.beta1, args.beta2, args.came_beta3),
                              eps=args.eps, weight_decay=args.weight_decay,
                              factored_min_dim=args.factored_min_dim,
                              clip_threshold=args.factored_clip_threshold,
                              confidence_scale=args.came_confidence_scale,
                              confidence_min=args.came_confidence_min,
                              confidence_max=args.came_confidence_max)
    if name == "soap_adamw":
        return SOAPStyleAdamW(groups, lr=args.lr, betas=(args.beta1, args.beta2), eps=args.eps,
                              weight_decay=args.weight_decay,
                              precondition_frequency=args.soap_precondition_frequency,
                              large_side_identity_threshold=args.soap_large_side_identity_threshold,
                              one_sided=args.soap_one_sided)
    raise ValueError(f"unknown baseline optimizer {name!r}")
