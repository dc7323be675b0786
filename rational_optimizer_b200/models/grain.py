"""GRAIN ``nn.Module`` (Groupwise Rational Activation with Internal Normalization).

Same constructor, parameters and persistent buffers as the reference module
(activation/rational_opt/rational.py:242-289): ``numerator [G, 6]`` and
``denominator [G, 4]`` initialised to the SiLU@5 fit, plus the empty
``_empty_coeff [G, 0, 2]``, ``_empty_centers [G, 0]`` and ``_empty_beta [G, 0]``
buffers that appear in checkpoints.  The optional optimizer telemetry
(rational.py:291-437) is reproduced by :meth:`GRAIN._update_optimizer_stats`.
"""
from __future__ import annotations

import torch
from torch import nn

from ..ops.grain import (GRAIN_DENOMINATOR, GRAIN_NUMERATOR, MAX_GROUP_WIDTH,
                         rational_local_basis)


class GRAIN(nn.Module):
    """Groupwise Rational Activation with Internal Normalization."""

    def __init__(self, hidden_dim, groups, init="silu", fit_range=5.0, eps=1e-6):
        super().__init__()
        hidden_dim = int(hidden_dim)
        groups = int(groups)
        if hidden_dim <= 0:
            raise ValueError("hidden_dim must be positive")
        if groups <= 0:
            raise ValueError("groups must be positive")
        if hidden_dim % groups != 0:
            raise ValueError("hidden_dim must be divisible by groups")
        if hidden_dim // groups > MAX_GROUP_WIDTH:
            raise ValueError("GRAIN supports group width <= 256")
        if init != "silu" or float(fit_range) != 5.0:
            raise ValueError("GRAIN requires the published silu@5 initializer")
        self.hidden_dim = hidden_dim
        self.groups = groups
        self.init_name = init
        self.fit_range = float(fit_range)
        self.eps = float(eps)
        self.numerator = nn.Parameter(
            torch.tensor(GRAIN_NUMERATOR, dtype=torch.float32).repeat(groups, 1))
        self.denominator = nn.Parameter(
            torch.tensor(GRAIN_DENOMINATOR, dtype=torch.float32).repeat(groups, 1))
        self.register_buffer("_empty_coeff", torch.empty(groups, 0, 2, dtype=torch.float32))
        self.register_buffer("_empty_centers", torch.empty(groups, 0, dtype=torch.float32))
        self.register_buffer("_empty_beta", torch.empty(groups, 0, dtype=torch.float32))

    @torch.no_grad()
    def _update_optimizer_stats(self, x):
        if not bool(getattr(self, "_rlb_optimizer_track_stats", False)):
            return
        if bool(getattr(self, "_rlb_optimizer_stats_training_only", False)) and not self.training:
            return
        stat_every = int(getattr(self, "_rlb_optimizer_stat_every", 1))
        counter = int(getattr(self, "_rlb_optimizer_stat_counter", 0)) + 1
        self._rlb_optimizer_stat_counter = counter
        if stat_every > 1 and counter % stat_every != 0 and hasattr(self, "_rlb_optimizer_stats"):
            return
        self._rlb_optimizer_stats = grain_statistics(
            x, self.numerator, self.denominator, self.groups, self.hidden_dim, self.eps,
            int(getattr(self, "_rlb_optimizer_stat_samples", 512)))
        version = int(getattr(self, "_rlb_optimizer_stat_version", 0)) + 1
        self._rlb_optimizer_stat_version = version
        self._rlb_optimizer_stats["stat_version"] = version

    def forward(self, x, precomputed=None):
        """GRAIN(x).  ``precomputed``: the activation already evaluated by a fused
        producer (the in-projection GEMM epilogue); the module then only records
        its statistics and hands it on, so its hooks still see (x, GRAIN(x))."""
        if x.size(-1) != self.hidden_dim:
            raise ValueError(f"expected last dimension {self.hidden_dim}, got {x.size(-1)}")
        self._update_optimizer_stats(x)
        if precomputed is not None:
            return precomputed
        return rational_local_basis(x, self.numerator, self.denominator, self._empty_coeff,
                                    self._empty_centers, self._empty_beta, 0.0, self.eps,
                                    self.hidden_dim, self.groups)

    def extra_repr(self):
        return (f"hidden_dim={self.hidden_dim}, groups={self.groups}, "
                f"init={self.init_name!r}, fit_range={self.fit_range:g}")


@torch.no_grad()
def grain_statistics(x, numerator, denominator, groups, hidden_dim, eps, max_samples=512):
    """Moments, feature Grams and output/derivative RMS of GRAIN on sampled rows."""
    flat = x.detach().reshape(-1, hidden_dim)
    if max_samples > 0 and flat.size(0) > max_samples:
        index = torch.linspace(0, flat.size(0) - 1, max_samples, device=flat.device).long()
        flat = flat.index_select(0, index)
    width = hidden_dim // groups
    grouped = flat.float().view(-1, groups, width)
    rms = torch.sqrt(grouped.square().mean(dim=-1, keepdim=True) + eps)
    t = grouped / rms
    abs_t = t.abs()
    moments = [torch.ones(groups, device=t.device)]
    signed = [torch.ones(groups, device=t.device)]
    ap = torch.ones_like(abs_t)
    sp = torch.ones_like(t)
    for _ in range(1, 11):
        ap = ap * abs_t
        sp = sp * t
        moments.append(ap.mean(dim=(0, 2)))
        signed.append(sp.mean(dim=(0, 2)))
    t2 = t.square()
    t3 = t2 * t
    t4 = t2.square()
    t5 = t4 * t
    ax3 = abs_t * t2
    num = numerator.detach().float().view(1, groups, 1, 6)
    den = denominator.detach().float()
    den_abs = den.abs().view(1, groups, 1, 4)
    den_sign = torch.where(den >= 0.0, 1.0, -1.0).view(1, groups, 1, 4)
    powers = torch.stack((torch.ones_like(t), t, t2, t3, t4, t5), dim=-1)
    den_powers = torch.stack((abs_t, t2, ax3, t4), dim=-1)
    q = (1.0 + den_abs[..., 0] * abs_t + den_abs[..., 1] * t2 + den_abs[..., 2] * ax3
         + den_abs[..., 3] * t4)
    poly = (num * powers).sum(dim=-1)
    dpoly = (num[..., 1] + 2.0 * num[..., 2] * t + 3.0 * num[..., 3] * t2
             + 4.0 * num[..., 4] * t3 + 5.0 * num[..., 5] * t4)
    dq = (den_abs[..., 0] * torch.sign(t) + 2.0 * den_abs[..., 1] * t
          + 3.0 * den_abs[..., 2] * t * abs_t + 4.0 * den_abs[..., 3] * t3)
    output = poly / q.clamp_min(eps)
    derivative = (dpoly * q - poly * dq) / q.square().clamp_min(eps)
    num_features = powers / q.unsqueeze(-1).clamp_min(eps)
    den_features = (-poly.unsqueeze(-1) * den_sign * den_powers
                    / q.square().unsqueeze(-1).clamp_min(eps))
    num_flat = num_features.permute(1, 0, 2, 3).reshape(groups, -1, 6)
    den_flat = den_features.permute(1, 0, 2, 3).reshape(groups, -1, 4)
    num_gram = torch.einsum("gni,gnj->gij", num_flat, num_flat) / max(1, num_flat.size(1))
    den_gram = torch.einsum("gni,gnj->gij", den_flat, den_flat) / max(1, den_flat.size(1))
    return {
        "abs_moments": torch.stack(moments, dim=1),
        "raw_moments": torch.stack(signed, dim=1),
        "num_gram": num_gram,
        "den_gram": den_gram,
        "output_rms": torch.sqrt(output.square().mean(dim=(0, 2)) + eps),
        "derivative_rms": torch.sqrt(derivative.square().mean(dim=(0, 2)) + eps),
        "output_sq_sum": output.square().sum(dim=(0, 2)),
        "derivative_sq_sum": derivative.square().sum(dim=(0, 2)),
        "sample_count": torch.full((groups,), float(output.size(0) * output.size(2)),
                                   device=output.device),
    }
