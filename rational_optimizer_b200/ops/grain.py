"""GRAIN operators: grouped RMS-normalised P5/Q4 rational activation.

Public functions mirror activation/rational_opt/rational.py:110-239 of the
reference (``rational_local_basis`` with numerator/denominator, local-basis
atoms, ``coeff_limit``, ``eps``, ``hidden_dim``, ``groups``).  CUDA tensors run
the sm_100a kernels of ``csrc/grain.cu`` (fp32 math, fp32 or bf16 storage);
CPU tensors run :func:`grain_reference`, the PyTorch oracle used by tests.
The legacy ungrouped operators (reference K1-K5: ``forward``/``backward`` and
``version_a_forward``/``version_a_backward``), the affine statistics (K9) and
the restricted backward (K10) are exposed as well.
"""
from __future__ import annotations

import os

import torch

from .._ext import dtype_code, ext
from .linear import weight_grad

# SiLU fit of P5/Q4 on [-5, 5] (the published GRAIN initializer; the values
# must be identical for checkpoints and the parameter-count contract).
GRAIN_NUMERATOR = (
    2.4915714620520875e-05,
    0.5000668663485823,
    0.2499441908995771,
    0.0526200910151016,
    0.005525765640115002,
    0.00024199321178747251,
)
GRAIN_DENOMINATOR = (
    0.00022554017910995938,
    0.10511420350691994,
    2.8656992394109812e-05,
    0.0004816962110562025,
)
MAX_GROUP_WIDTH = 256
MAX_BASIS = 4


def torch_fallback_requested() -> bool:
    """``RATIONAL_OPT_TORCH_FALLBACK`` selects the PyTorch path (reference switch)."""
    return os.environ.get("RATIONAL_OPT_TORCH_FALLBACK", "0") in {"1", "true", "True", "yes"}


def grain_reference(x, numerator, denominator, coeff_logits, centers, beta, coeff_limit, eps,
                    hidden_dim, groups):
    """PyTorch GRAIN (fp32 math) used on CPU and as the numerical oracle."""
    shape = x.shape
    groups = int(groups)
    width = int(hidden_dim) // groups
    work = x.float().reshape(*shape[:-1], groups, width)
    rho = torch.sqrt(work.square().mean(dim=-1, keepdim=True) + float(eps))
    t = work / rho
    cshape = (1,) * (work.dim() - 2) + (groups, 1)
    a = numerator.float()
    b = denominator.float().abs()
    coef = lambda m, j: m[:, j].reshape(cshape)
    # Same expression graph as the reference fallback so CPU gradients agree
    # bit for bit (each |t| is its own node; Horner from the top coefficient).
    t2 = t.square()
    t4 = t2.square()
    p = ((((coef(a, 5) * t + coef(a, 4)) * t + coef(a, 3)) * t + coef(a, 2)) * t
         + coef(a, 1)) * t + coef(a, 0)
    q = (1.0 + coef(b, 0) * t.abs() + coef(b, 1) * t2 + coef(b, 2) * t.abs() * t2
         + coef(b, 3) * t4)
    f = p / q.clamp_min(torch.finfo(torch.float32).tiny)
    nb = int(centers.shape[1]) if centers.dim() == 2 else 0
    delta = torch.zeros_like(t)
    if nb:
        weights = float(coeff_limit) * torch.tanh(coeff_logits.float())
        for k in range(nb):
            c = centers[:, k].float().reshape(cshape)
            be = beta[:, k].float().reshape(cshape)
            u = t - c
            den = 1.0 + be * u.square()
            zero = 1.0 / (1.0 + be * c.square())
            delta = delta + weights[:, k, 0].reshape(cshape) * (u / den)
            delta = delta + weights[:, k, 1].reshape(cshape) * (1.0 / den - zero)
    f = f + delta
    return (f * rho).reshape(shape).to(x.dtype)


class _GrainFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, numerator, denominator, coeff_logits, centers, beta, coeff_limit, eps,
                hidden_dim, groups):
        C = ext()
        xw = x.contiguous()
        num = numerator.detach().float().contiguous()
        den = denominator.detach().float().contiguous()
        log = coeff_logits.detach().float().contiguous()
        cen = centers.detach().float().contiguous()
        bet = beta.detach().float().contiguous()
        (y,) = C.grain_forward(xw, num, den, log, cen, bet, float(coeff_limit), float(eps),
                               int(hidden_dim), int(groups), -1, False)
        ctx.save_for_backward(xw, num, den, log, cen, bet)
        ctx.meta = (float(coeff_limit), float(eps), int(hidden_dim), int(groups),
                    numerator.dtype, denominator.dtype, coeff_logits.dtype)
        return y

    @staticmethod
    def backward(ctx, gy):
        C = ext()
        xw, num, den, log, cen, bet = ctx.saved_tensors
        coeff_limit, eps, hidden, groups, ndt, ddt, ldt = ctx.meta
        gy = gy.contiguous()
        if gy.dtype != xw.dtype:
            gy = gy.to(xw.dtype)
        gx, gnum, gden, gcoef = C.grain_backward(gy, xw, num, den, log, cen, bet, coeff_limit, eps,
                                                 hidden, groups, None, None)
        return (gx, gnum.to(ndt), gden.to(ddt), gcoef.to(ldt), None, None, None, None, None, None)


class _GrainMLPFunction(torch.autograd.Function):
    """``out_proj(GRAIN(in_proj(x)))`` with GRAIN inside the GEMM epilogues.

    Forward: ``grain_in_proj_forward`` (csrc/gemm2_sm100.cu) is one 2-SM
    tcgen05 GEMM whose epilogue stores the pre-activation ``h`` and the
    activation ``y``; the out-projection follows.  Backward: the out-
    projection's input gradient and the GRAIN backward are one GEMM
    (``grain_out_proj_backward``: ``gy = dO W_out`` stays in tensor memory,
    the epilogue emits ``dh`` and the coefficient partials), then the
    in-projection's gradients.  Weight gradients accumulate inside the GEMM
    when the weight's ``.grad`` is a managed fp32 buffer (as in
    ``ops.linear``).  ``h`` and ``y`` are also returned (non-differentiable)
    for the activation module's forward hooks.
    """

    @staticmethod
    def forward(ctx, x, w_in, w_in_c, numerator, denominator, w_out, w_out_c, w_out_t_c, eps, groups):
        from . import gemm
        C = ext()
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != w_in_c.dtype:
            x2 = x2.to(w_in_c.dtype)
        x2 = x2.contiguous()
        num = numerator.detach().float().contiguous()
        den = denominator.detach().float().contiguous()
        out = C.grain_in_proj_forward(x2, w_in_c, num, den, float(eps))
        if out is None:
            raise RuntimeError("fused GRAIN in-projection rejected a supported shape")
        h, y = out
        o = gemm.matmul_nt(y, w_out_c)
        ctx.save_for_backward(x2, w_in_c, h, y, num, den, w_out_c, w_out_t_c)
        ctx.weights = (w_in, w_out)
        ctx.coefs = (numerator, denominator)
        ctx.meta = (float(eps), int(groups), x.shape, x.dtype, numerator.dtype, denominator.dtype)
        ctx.mark_non_differentiable(h, y)
        # h and y never receive gradients: skip materialising two zero tensors
        # of the activation's size for them in the backward
        ctx.set_materialize_grads(False)
        lead = tuple(x.shape[:-1])
        return o.view(lead + (o.shape[-1],)), h.view(lead + (h.shape[-1],)), y.view(lead + (y.shape[-1],))

    @staticmethod
    def backward(ctx, go, _gh, _gy):
        from . import gemm
        C = ext()
        x2, w_in_c, h, y, num, den, w_out_c, w_out_t_c = ctx.saved_tensors
        eps, groups, in_shape, x_dtype, ndt, ddt = ctx.meta
        w_in, w_out = ctx.weights
        hidden = h.shape[-1]
        if go is None:
            go = torch.zeros(tuple(in_shape[:-1]) + (w_out_c.shape[0],), device=h.device, dtype=w_out_c.dtype)
        g2 = go.reshape(-1, go.shape[-1])
        if g2.dtype != w_out_c.dtype:
            g2 = g2.to(w_out_c.dtype)
        g2 = g2.contiguous()
        gw_out = weight_grad(w_out, g2, y, ctx.needs_input_grad[5])
        res = None
        coef_into = None
        if os.environ.get("RO_FUSED_GRAIN_BWD", "1") != "0":
            from .linear import managed_grad
            gn_buf = managed_grad(ctx.coefs[0]) if ctx.needs_input_grad[3] else None
            gd_buf = managed_grad(ctx.coefs[1]) if ctx.needs_input_grad[4] else None
            if gn_buf is not None and gd_buf is not None:
                coef_into = (gn_buf, gd_buf)
            res = C.grain_out_proj_backward(g2, w_out_t_c, h, num, den, float(eps),
                                            *(coef_into if coef_into else (None, None)))
            if res is None:
                coef_into = None
        if res is None:
            gy = gemm.matmul_nn(g2, w_out_c)
            e = num.new_empty(groups, 0)
            gh, gnum, gden, _ = C.grain_backward(gy, h, num, den, num.new_empty(groups, 0, 2), e, e, 0.0, eps,
                                                 hidden, groups, None, None)
        else:
            gh, gnum, gden = res
        gx = None
        if ctx.needs_input_grad[0]:
            gx = gemm.matmul_nn(gh, w_in_c).reshape(in_shape)
            if gx.dtype != x_dtype:
                gx = gx.to(x_dtype)
        gw_in = weight_grad(w_in, gh, x2, ctx.needs_input_grad[1])
        if coef_into is not None:
            # coefficient gradients were added into the managed buffers by the reduction
            from .linear import report_ready
            report_ready(ctx.coefs[0])
            report_ready(ctx.coefs[1])
            return gx, gw_in, None, None, None, gw_out, None, None, None, None
        return gx, gw_in, None, gnum.to(ndt), gden.to(ddt), gw_out, None, None, None, None


def in_proj_grain_supported(x, hidden_dim, groups) -> bool:
    """Whether the fused in-projection + GRAIN path applies (CUDA bf16, groups of 256)."""
    if not (x.is_cuda and x.dtype == torch.bfloat16) or torch_fallback_requested():
        return False
    if int(hidden_dim) != 256 * int(groups):
        return False
    if os.environ.get("RO_FUSED_GRAIN", "1") == "0":
        return False
    return hasattr(ext(), "grain_in_proj_forward")


def grain_mlp(x, w_in, w_in_c, numerator, denominator, w_out, w_out_c, w_out_t_c, eps, groups):
    """``(o, h, y)``: the GRAIN MLP output and, without gradient, its pre-activation and activation."""
    return _GrainMLPFunction.apply(x, w_in, w_in_c, numerator, denominator, w_out, w_out_c, w_out_t_c, eps,
                                   groups)


def _validate(x, hidden_dim, groups, centers):
    hidden_dim = int(hidden_dim)
    groups = int(groups)
    if groups <= 0 or hidden_dim % groups:
        raise ValueError("hidden_dim must be divisible by groups")
    if hidden_dim // groups > MAX_GROUP_WIDTH:
        raise ValueError("GRAIN supports group width <= 256")
    if x.size(-1) != hidden_dim:
        raise ValueError(f"expected last dimension {hidden_dim}, got {x.size(-1)}")
    if centers.dim() == 2 and centers.shape[1] > MAX_BASIS:
        raise ValueError("GRAIN supports at most 4 local basis atoms")


def rational_local_basis(x, numerator, denominator, coeff_logits, centers, beta, coeff_limit, eps,
                         hidden_dim, groups):
    """Apply GRAIN (reference API ``rational_local_basis``, rational.py:195-239)."""
    _validate(x, hidden_dim, groups, centers)
    if not x.is_cuda or torch_fallback_requested():
        return grain_reference(x, numerator, denominator, coeff_logits, centers, beta,
                               coeff_limit, eps, hidden_dim, groups)
    return _GrainFunction.apply(x, numerator, denominator, coeff_logits, centers, beta,
                                coeff_limit, eps, hidden_dim, groups)


def local_basis_forward(x, numerator, denominator, coeff_logits, centers, beta, coeff_limit, eps,
                        hidden_dim, groups, out_dtype=None, want_rho=False):
    """Raw kernel forward (no autograd); returns ``y`` or ``(y, rho[rows, G])``."""
    code = -1 if out_dtype is None else dtype_code(out_dtype)
    out = ext().grain_forward(x.contiguous(), numerator.float().contiguous(),
                              denominator.float().contiguous(), coeff_logits.float().contiguous(),
                              centers.float().contiguous(), beta.float().contiguous(),
                              float(coeff_limit), float(eps), int(hidden_dim), int(groups), code,
                              bool(want_rho))
    return tuple(out) if want_rho else out[0]


def local_basis_backward(grad_output, x, numerator, denominator, coeff_logits, centers, beta,
                         coeff_limit, eps, hidden_dim, groups):
    """Raw kernel backward: ``(grad_x, grad_numerator, grad_denominator, grad_coeff_logits)``."""
    return tuple(ext().grain_backward(
        grad_output.contiguous(), x.contiguous(), numerator.float().contiguous(),
        denominator.float().contiguous(), coeff_logits.float().contiguous(),
        centers.float().contiguous(), beta.float().contiguous(), float(coeff_limit), float(eps),
        int(hidden_dim), int(groups), None, None))


def local_basis_restricted_backward(grad_output, x, numerator, denominator, coeff_logits, centers,
                                    beta, affine_alpha, affine_beta, coeff_limit, eps, hidden_dim,
                                    groups):
    """Restricted-morphology backward (reference K10).

    Returns ``(nonlinear_y, nonlinear_grad_x, grad_numerator, grad_denominator,
    grad_coeff_logits)`` where the per-group affine part ``z*alpha + rho*beta``
    is removed from the output and its gradient.
    """
    if not x.is_cuda:
        return _restricted_backward_reference(grad_output, x, numerator, denominator, coeff_logits,
                                              centers, beta, affine_alpha, affine_beta,
                                              coeff_limit, eps, hidden_dim, groups)
    return tuple(ext().grain_backward(
        grad_output.contiguous(), x.contiguous(), numerator.float().contiguous(),
        denominator.float().contiguous(), coeff_logits.float().contiguous(),
        centers.float().contiguous(), beta.float().contiguous(), float(coeff_limit), float(eps),
        int(hidden_dim), int(groups), affine_alpha.float().contiguous(),
        affine_beta.float().contiguous()))


def local_basis_affine_statistics(x, feature, eps, hidden_dim, groups):
    """Per-(row, group) ``rho`` and fp64 group sums [count, Σt, Σt², Σh/ρ, Σt·h/ρ] (K9)."""
    if not x.is_cuda:
        return _affine_statistics_reference(x, feature, eps, hidden_dim, groups)
    stats, rho = ext().grain_affine_statistics(x.contiguous(), feature.contiguous(), float(eps),
                                               int(hidden_dim), int(groups))
    return stats, rho


def _affine_statistics_reference(x, feature, eps, hidden_dim, groups):
    groups = int(groups)
    width = int(hidden_dim) // groups
    z = x.float().reshape(-1, groups, width)
    h = feature.float().reshape(-1, groups, width)
    rho = torch.sqrt(z.square().mean(dim=-1, keepdim=True) + float(eps))
    t = z / rho
    fn = h / rho
    count = torch.full((groups,), float(z.shape[0] * width), dtype=torch.float64)
    stats = torch.stack((count.to(x.device), t.double().sum(dim=(0, 2)),
                         t.double().square().sum(dim=(0, 2)), fn.double().sum(dim=(0, 2)),
                         (t.double() * fn.double()).sum(dim=(0, 2))), dim=1)
    return stats, rho


def _restricted_backward_reference(gy, x, numerator, denominator, coeff_logits, centers, beta,
                                   alpha, abeta, coeff_limit, eps, hidden_dim, groups):
    groups = int(groups)
    width = int(hidden_dim) // groups
    xr = x.detach().float().requires_grad_(True)
    num = numerator.detach().float().requires_grad_(True)
    den = denominator.detach().float().requires_grad_(True)
    log = coeff_logits.detach().float().requires_grad_(True)
    y = grain_reference(xr, num, den, log, centers, beta, coeff_limit, eps, hidden_dim, groups)
    grads = torch.autograd.grad(y, (xr, num, den, log), gy.float(), allow_unused=True)
    gx, gnum, gden, glog = [g if g is not None else torch.zeros_like(v)
                            for g, v in zip(grads, (xr, num, den, log))]
    z = x.float().reshape(-1, groups, width)
    rho = torch.sqrt(z.square().mean(dim=-1, keepdim=True) + float(eps))
    t = z / rho
    a = alpha.float().view(1, groups, 1)
    bb = abeta.float().view(1, groups, 1)
    g = gy.float().reshape(-1, groups, width)
    nonlinear = y.detach().reshape(-1, groups, width) - z * a - rho * bb
    gx = gx.reshape(-1, groups, width) - g * a - (t / width) * bb * g.sum(dim=-1, keepdim=True)
    return (nonlinear.reshape(x.shape), gx.reshape(x.shape), gnum, gden, glog)


# ---------------------------------------------------------------------------
# Legacy ungrouped rationals (reference K1-K5).

def _legacy_reference(x, a, b, signed):
    xf = x.float()
    p = torch.zeros_like(xf)
    for j in (5, 4, 3, 2, 1, 0):
        p = p * xf + a[j].float()
    if signed:
        q = torch.zeros_like(xf)
        for j in (3, 2, 1, 0):
            q = q * xf + b[j].float()
        q = q * xf + 1.0
    else:
        bb = b.float().abs()
        ax = xf.abs()
        q = 1.0 + bb[0] * ax + bb[1] * xf * xf + bb[2] * ax * xf * xf + bb[3] * xf ** 4
    return p / q


class _LegacyFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, a, b, signed):
        xw = x.float().contiguous()
        aw = a.detach().float().contiguous()
        bw = b.detach().float().contiguous()
        y = ext().legacy_forward(xw, aw, bw, bool(signed))
        ctx.save_for_backward(xw, aw, bw)
        ctx.signed = bool(signed)
        return y

    @staticmethod
    def backward(ctx, gy):
        xw, aw, bw = ctx.saved_tensors
        gx, ga, gb = ext().legacy_backward(gy.float().contiguous(), xw, aw, bw, ctx.signed)
        return gx, ga, gb, None


def rational_forward(x, numerator, denominator):
    """Legacy ungrouped P5/Q4 with signed denominator (reference ``_C.forward``)."""
    if not x.is_cuda:
        return _legacy_reference(x, numerator, denominator, True)
    return _LegacyFunction.apply(x, numerator, denominator, True)


def version_a_forward(x, numerator, denominator):
    """Legacy ungrouped P5/Q4 with |b| denominator (reference ``_C.version_a_forward``)."""
    if not x.is_cuda:
        return _legacy_reference(x, numerator, denominator, False)
    return _LegacyFunction.apply(x, numerator, denominator, False)


def rational_backward(grad_output, x, numerator, denominator, *, version_a=False):
    """Kernel backward of the legacy operators: ``(grad_x, grad_num, grad_den)``."""
    if not x.is_cuda:
        xr = x.detach().float().requires_grad_(True)
        a = numerator.detach().float().requires_grad_(True)
        b = denominator.detach().float().requires_grad_(True)
        y = _legacy_reference(xr, a, b, not version_a)
        return torch.autograd.grad(y, (xr, a, b), grad_output.float())
    return tuple(ext().legacy_backward(grad_output.float().contiguous(), x.float().contiguous(),
                                       numerator.float().contiguous(),
                                       denominator.float().contiguous(), not version_a))
