"""TILLER for a fixed SwiGLU MLP (no GRAIN): the separately named extension of
experiments/swiglu_tiller/tiller_swiglu.py:1-525 (checkpoint version
``tiller_swiglu_fixed_v1``).

Method.  With a fixed activation the response congruence is exactly one, so
the chord's response-drift rotation vanishes.  What remains per update:

* a participation route from trace ratios of ``J = [diag(dg), diag(dv)]``
  and of the features ``h = silu(g) * v`` on the probe rows (refresh steps,
  every eighth update; cached in between);
* per role the Nesterov momentum, its rational-group polar factor, and the
  factorized adaptive-tangent chord (:func:`tiller_math.adaptive_tangent_chord`);
* the functional loss ledger and equal-budget transaction of the GRAIN router
  (:meth:`TILLERRouter._advance_rows` / :meth:`TILLERRouter._transaction`,
  shared, not re-implemented), with the gate and value matrices forming one
  logical incoming role and the down projection the outgoing role.

Structure of this module.

* Probe rows are recorded through the SwiGLU module's ``tap`` instrumentation
  point (:class:`~rational_optimizer_b200.mha.model.SwiGLU`): one callback per
  layer receives the input, both projections, the features and the output of
  the forward that actually ran, and attaches the cotangent hook.
  :class:`ProbeTap` owns that bookkeeping.
* :class:`SwiGLURouter` is the optimizer over the gate/value/down matrices;
  its ``step`` is split into the route, the role directions, the functional
  scores and the apply.
* :class:`SwiGLUTILLER` wires router, the standard TILLER attention optimizer
  (congruence one, q/k/v handled as one logical matrix through
  :class:`~rational_optimizer_b200.mha.optim.QKVBundle`) and an AdamW for the
  remaining parameters, and runs an update from explicit per-token loss masks:
  ``zero_grad()``, ``begin_step(masks)``, one ``backward(per_token_losses)``
  per micro-batch, ``step()`` (outside autocast).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import tiller_math as tm
from .newton_schulz import match_rms_adamw_adjustment, rational_group_zero_power
from .tiller import TILLERAttentionOptimizer, TILLERRouter, foreach_apply, foreach_nesterov

VERSION = "tiller_swiglu_fixed_v1"
REFRESH_EVERY = 8
# the fixed optimizer cell of the extension (LR is scheduled by the caller)
CELL = dict(weight_decay=0.1, momentum=0.95, ns_steps=5, beta2=0.95, eps=1e-8)
AUX_BETAS = (0.9, 0.95)


# -- SwiGLU calculus -----------------------------------------------------------
def swiglu_factors(gate, value):
    """(features, d features / d gate, d features / d value) of ``silu(gate) * value``."""
    s = torch.sigmoid(gate)
    silu = F.silu(gate)
    return silu * value, value * s * (1 + gate * (1 - s)), silu


def group_scores(inputs, gate, value, features, cotangent, down_weight, gate_direction,
                 value_direction, down_direction, group_width):
    """Cotangent-contracted JVP of the MLP along a direction, one column per channel group.

    ``<c, d y>`` with ``d y = down (dg * (x dWg^T) + dv * (x dWv^T)) + dWdown h``.
    """
    _, dg, dv = swiglu_factors(gate, value)
    back = cotangent @ down_weight
    tangent_in = (inputs @ gate_direction.T) * dg + (inputs @ value_direction.T) * dv
    per_channel = tangent_in * back + features * (cotangent @ down_direction)
    return per_channel.reshape(inputs.shape[0], -1, group_width).sum(-1)


def participation_statistics(gate, value, features, cotangent, down_weight, width):
    """[groups, 4]: weighted trace-ratio numerators and weights for the incoming and
    outgoing roles (sum them over probe rows and ranks before dividing)."""
    _, dg, dv = swiglu_factors(gate, value)
    rows = gate.shape[0]
    jac = (dg.square() + dv.square()).reshape(rows, -1, width)
    feat = features.square().reshape(rows, -1, width)
    floor = torch.finfo(gate.dtype).tiny

    def trace_ratio(e):
        return e.sum(-1).square() / (width * e.square().sum(-1)).clamp_min(floor)

    w_in = (jac * (cotangent @ down_weight).reshape(rows, -1, width).square()).mean(-1)
    w_out = cotangent.square().mean(-1, keepdim=True).expand_as(w_in)
    return torch.stack(((trace_ratio(jac) * w_in).sum(0), w_in.sum(0),
                        (trace_ratio(feat) * w_out).sum(0), w_out.sum(0)), -1)


# -- probe recording -------------------------------------------------------------
@dataclass
class _Probe:
    x: torch.Tensor
    gate: torch.Tensor
    value: torch.Tensor
    h: torch.Tensor
    cotangent: torch.Tensor | None = None


@dataclass
class _LayerLog:
    forwards: int = 0
    probes: list = field(default_factory=list)


class ProbeTap:
    """Records the probe rows of every layer's SwiGLU forward and backward.

    Installed as ``mlp.tap`` on each layer.  ``arm`` opens an update with the
    per-micro-batch row indices to record (empty when the update does not
    refresh); every training forward of a layer consumes the next
    micro-batch's indices.
    """

    def __init__(self, mlps, hidden, external):
        self.mlps = list(mlps)
        self.hidden, self.external = int(hidden), int(external)
        self.rows = None          # [micro-batch] -> LongTensor of local rows, or None when idle
        self.rows_per_micro = None
        self.recording = False
        self.logs = []
        for layer, mlp in enumerate(self.mlps):
            if getattr(mlp, "tap", None) is not None:
                raise RuntimeError(f"layer {layer}'s SwiGLU already has an instrumentation tap")
            mlp.tap = self._callback(layer)

    def remove(self):
        for mlp in self.mlps:
            mlp.tap = None
        self.mlps = []

    def arm(self, rows_per_micro, row_indices, recording):
        self.rows_per_micro = list(rows_per_micro)
        self.rows = list(row_indices)
        self.recording = bool(recording)
        self.logs = [_LayerLog() for _ in self.mlps]

    def disarm(self):
        self.rows = None
        self.logs = []

    def _callback(self, layer):
        def tap(mlp, x, gate, value, h, y):
            if not mlp.training:
                return
            if self.rows is None:
                raise RuntimeError("a training forward ran outside begin_step()/step()")
            log = self.logs[layer]
            micro = log.forwards
            if micro >= len(self.rows):
                raise RuntimeError(f"layer {layer} ran more forwards than declared micro-batches "
                                   "(re-entrant or checkpointed MLP forwards are not supported)")
            flat_x = x.detach().reshape(-1, self.external)
            if flat_x.shape[0] != self.rows_per_micro[micro]:
                raise RuntimeError(f"layer {layer} saw {flat_x.shape[0]} rows, loss mask declares "
                                   f"{self.rows_per_micro[micro]}")
            log.forwards += 1
            if not self.recording:
                return
            with torch.no_grad():
                idx = self.rows[micro]
                pick = lambda t, w: t.detach().reshape(-1, w).index_select(0, idx).float()
                probe = _Probe(pick(x, self.external), pick(gate, self.hidden), pick(value, self.hidden),
                               pick(h, self.hidden))
            if not y.requires_grad:
                raise RuntimeError("SwiGLU output is not differentiable; probes need its cotangent")
            log.probes.append(probe)

            def on_cotangent(grad):
                if probe.cotangent is not None:
                    raise RuntimeError("a probed SwiGLU output received two cotangents")
                probe.cotangent = grad.detach().reshape(-1, self.external).index_select(0, idx).float()
                return grad
            y.register_hook(on_cotangent)
        return tap

    def forwards_complete(self):
        return all(log.forwards == len(self.rows) for log in self.logs)

    def packets(self, cotangent_scale):
        """Per layer: [x, gate, value, h, scaled cotangent] over all micro-batches."""
        out = []
        for layer, log in enumerate(self.logs):
            if len(log.probes) != len(self.rows) or any(p.cotangent is None for p in log.probes):
                raise RuntimeError(f"layer {layer}: probe backward incomplete")
            cat = lambda name: torch.cat([getattr(p, name) for p in log.probes])
            out.append([cat("x"), cat("gate"), cat("value"), cat("h"),
                        cat("cotangent") * cotangent_scale])
        return out


# -- router ----------------------------------------------------------------------
class SwiGLURouter(torch.optim.Optimizer):
    """Gate/value/down matrices of every layer (two logical roles: gate+value, down)."""

    # ledger + transaction of the GRAIN router, used unchanged
    _previous_ledger = TILLERRouter._previous_ledger
    _advance_rows = TILLERRouter._advance_rows
    _transaction = TILLERRouter._transaction
    momentum = CELL["momentum"]
    ns_steps = CELL["ns_steps"]
    strict = True

    _AXIS = {"gate": "rows", "value": "rows", "down": "columns"}

    def __init__(self, blocks, group_width, process_group=None):
        self.pairs = blocks
        self.loss_probe_group = process_group
        self.width = int(group_width)
        self.hidden, self.external = blocks[0]["in_weight"].shape
        self.groups = self.hidden // self.width
        self.roles = {"gate": [b["in_weight"] for b in blocks],
                      "value": [b["value_weight"] for b in blocks],
                      "down": [b["out_weight"] for b in blocks]}
        params = [p for ps in self.roles.values() for p in ps]
        super().__init__([{"params": params, "lr": 3e-4, "weight_decay": CELL["weight_decay"],
                           "version": VERSION}], {})
        self.tap = ProbeTap([b["mlp"] for b in blocks], self.hidden, self.external)
        self._attention_consumed = True
        self._attention_update = 0
        self._clip_factor = None
        self._capture_telemetry_next_step = False
        self._rfd_rows = self._rfd_selection = None
        self._rfd_gradient_scale = self._rfd_decay_derivative = None
        self.refresh = False
        self.loss_denominator = None
        self.last_metrics = {}

    @property
    def anchor(self):
        return self.state[self.pairs[0]["in_weight"]]

    @property
    def completed_steps(self):
        return int(self.anchor.get("factorized_rfd_step", 0))

    @property
    def active(self):
        return self.tap.rows is not None

    def begin(self, masks, indices, loss_denominator):
        if self.active or not self._attention_consumed:
            raise RuntimeError("the previous router/attention update has not finished")
        self.refresh = self.completed_steps % REFRESH_EVERY == 0
        self.loss_denominator = float(loss_denominator)
        self._clip_factor = None
        self.tap.arm([m.numel() for m in masks], indices, self.refresh)

    def consume_response_homotopy(self):
        if self._attention_consumed:
            raise RuntimeError("the attention optimizer already took this update's route")
        self._attention_consumed = True
        route = self.anchor["swiglu_participation"]
        intrinsic = (route[..., 0].mean(-1) * route[..., 1].mean(-1)).clamp(0, 1).sqrt()
        return intrinsic, torch.ones_like(intrinsic), self._attention_update

    # -- pieces of a step ---------------------------------------------------
    def _refresh_route(self, packets):
        stats = torch.stack([participation_statistics(g, v, h, c, b["out_weight"].detach().float(),
                                                      self.width)
                             for b, (_x, g, v, h, c) in zip(self.pairs, packets)])
        if dist.is_initialized():
            dist.all_reduce(stats, group=self.loss_probe_group)
        ratio, weight = stats[..., (0, 2)], stats[..., (1, 3)]
        self.anchor["swiglu_participation"] = torch.where(
            weight > 0, ratio / weight.clamp_min(1e-38), torch.ones_like(ratio)).clamp(0, 1)

    def _moments(self, parent, axis, key):
        """Row / column second moments of the role's chord (created at zero)."""
        shape = tm.grouped_shape(parent, groups=self.groups, width=self.width, axis=axis)
        want = {key + "_row_second_moment": shape[:-1],
                key + "_column_second_moment": shape[:2] + shape[-1:]}
        for name, sz in want.items():
            if name not in self.anchor:
                self.anchor[name] = torch.zeros(sz, device=parent.device, dtype=torch.float32)
        return tuple(self.anchor[name] for name in want)

    def _role_direction(self, role, params, route, step):
        """Selected direction [L, out, in] and its per-group contractions with
        the gradient, the momentum and itself."""
        axis = self._AXIS[role]
        view = lambda t: tm.group_view(t, groups=self.groups, width=self.width, axis=axis)
        momentum = foreach_nesterov(self, params, self.momentum)
        grad = torch.stack([p.grad for p in params]).float()
        parent = rational_group_zero_power(momentum, self.ns_steps, groups=self.groups,
                                           width=self.width).float()
        rows, cols = self._moments(parent, axis, "swiglu_" + role)
        parent_g, restore = view(parent)
        part = route[..., 1 if role == "down" else 0]
        chosen, _ = tm.adaptive_tangent_chord(parent_g, view(momentum)[0], view(grad)[0], rows, cols,
                                              part, torch.ones_like(part), step)
        direction = restore(chosen) * match_rms_adamw_adjustment(params[0].shape)
        d = view(direction)[0]
        contract = lambda t: (d * view(t)[0]).sum((-2, -1)).flatten()
        return direction, contract(grad), contract(momentum), d.square().sum((-2, -1)).flatten()

    def _functional_scores(self, packets, directions, wd):
        """[32 global probes, L*G + 1]: group scores of the direction, then the decay column."""
        score_cols, decay = [], []
        for layer, (b, packet) in enumerate(zip(self.pairs, packets)):
            base = (*packet, b["out_weight"].detach().float())
            score_cols.append(group_scores(*base, *(directions[r][layer] for r in self.roles),
                                           self.width))
            decay_dir = [b[k].detach().float() * wd for k in ("in_weight", "value_weight", "out_weight")]
            decay.append(group_scores(*base, *decay_dir, self.width).sum(-1))
        local = torch.cat((torch.stack(score_cols, 1).flatten(1), torch.stack(decay).sum(0)[:, None]), 1)
        return _gather_probe_rows(local, expected=tm.GLOBAL_PROBE_COUNT, group=self.loss_probe_group)

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("the probe batch is declared by begin_step; closures are not supported")
        if not self.active:
            raise RuntimeError("step() without begin_step()")
        if not self._attention_consumed or self._clip_factor is None:
            raise RuntimeError("step() needs the clip factor and the previous attention update")
        if not self.tap.forwards_complete():
            raise RuntimeError("some layer ran fewer forwards than declared micro-batches")
        step = self.completed_steps + 1
        lr = float(self.param_groups[0]["lr"])
        wd = float(self.param_groups[0]["weight_decay"])
        packets = self.tap.packets(self.loss_denominator * self._clip_factor) if self.refresh else None
        if self.refresh:
            self._refresh_route(packets)
        route = self.anchor["swiglu_participation"]
        directions, exact, moment, energies = {}, {}, {}, []
        for role, params in self.roles.items():
            directions[role], exact[role], moment[role], e = self._role_direction(role, params, route, step)
            energies.append(e)
        energy = torch.stack(energies).sum(0)
        self._rfd_rows = None
        self._rfd_gradient_scale = None
        self._rfd_decay_derivative = sum((p.grad * p).sum() * wd for ps in self.roles.values() for p in ps)
        if self.refresh:
            rows = self._functional_scores(packets, directions, wd)
            self._advance_rows(rows[:, :-1], rows[:, -1], functional=True)
        layer_ids = torch.arange(len(self.pairs), device=energy.device).repeat_interleave(self.groups)
        self._transaction(torch.stack((exact["gate"] + exact["value"], exact["down"])),
                          torch.stack((moment["gate"] + moment["value"], moment["down"])),
                          energy, layer_ids, eta=lr)
        coeff = self._rfd_selection.coefficients.reshape(len(self.pairs), self.groups)
        for role, params in self.roles.items():
            blocks, restore = tm.group_view(directions[role], groups=self.groups, width=self.width,
                                            axis=self._AXIS[role])
            foreach_apply(params, restore(blocks * coeff[..., None, None]), decay=1 - lr * wd, alpha=-lr)
        self._attention_update = step
        self._attention_consumed = False
        self.last_metrics = self._metrics(step, coeff)
        self.tap.disarm()
        self._clip_factor = None

    def _metrics(self, step, coeff):
        sel = self._rfd_selection
        dev = (coeff - 1).abs()
        return {"version": VERSION, "step": step, "functional_refresh": self.refresh,
                "ledger_step": self.completed_steps, "beta2": CELL["beta2"],
                "fixed_activation_congruence": 1.0, "response_departure_energy": 0.0,
                "proposal_accepted": bool(sel.accepted.item()),
                "coefficient_abs_deviation_mean": float(dev.mean()),
                "coefficient_abs_deviation_max": float(dev.max()),
                "budget_residual": float(sel.budget_residual.item()),
                "ledger_measurement": "functional" if self.refresh else "gradient_surrogate"}

    def close(self):
        self.tap.remove()


def _gather_probe_rows(local, *, expected, group=None):
    """All ranks' probe rows in rank order (ranks hold different counts; ``expected`` in total)."""
    if not (dist.is_available() and dist.is_initialized()):
        if local.shape[0] != expected:
            raise RuntimeError(f"{local.shape[0]} probe rows, the global layout has {expected}")
        return local
    world = dist.get_world_size(group)
    mine = torch.tensor([local.shape[0]], device=local.device, dtype=torch.int64)
    counts = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(counts, mine, group=group)
    counts = [int(c.item()) for c in counts]
    if sum(counts) != expected:
        raise RuntimeError(f"{sum(counts)} probe rows over all ranks, the global layout has {expected}")
    padded = local.new_zeros((max(counts), local.shape[1]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)])


# -- model inspection --------------------------------------------------------------
def _inspect_model(model, group_width):
    """(blocks, QKV bundles, auxiliary parameters) of a fixed-SwiGLU MHA decoder,
    or ValueError naming every requirement the model misses."""
    from ..mha.model import SwiGLU
    from ..mha.optim import AttentionLayout, QKVBundle

    c = getattr(model, "config", None)
    problems = []
    if getattr(model, "grain", True) or not isinstance(c, dict):
        raise ValueError("SwiGLU TILLER needs the fixed-SwiGLU MHA decoder (grain=False)")
    d, h = c["hidden_size"], c["intermediate_size"]
    if not (c["num_attention_heads"] == c["num_key_value_heads"] == 16 and 16 * c["head_dim"] == d):
        problems.append("attention must have 16 query and 16 key/value heads of width hidden/16")
    if type(group_width) is not int or group_width < 1 or h % group_width:
        problems.append(f"group width {group_width!r} does not divide the SwiGLU width {h}")
    elif len(model.layers) * (h // group_width) < 2:
        problems.append("fewer than two (layer, group) coordinates to coordinate")
    if h <= d:
        problems.append(f"SwiGLU width {h} is not wider than the residual width {d}")
    params = list(model.parameters())
    device = params[0].device
    if any(p.dtype != torch.float32 or p.device != device or not p.requires_grad for p in params):
        problems.append("every parameter must be a trainable fp32 tensor on one device")
    if problems:
        raise ValueError("SwiGLU TILLER cannot drive this model: " + "; ".join(problems))
    layout = AttentionLayout(d, 16, 16, c["head_dim"])
    want = [(h, d), (h, d), (d, h)] + [(d, d)] * 4
    blocks, bundles, structural = [], [], set()
    for i, layer in enumerate(model.layers):
        mlp, attn = layer.mlp, layer.attn
        mods = (mlp.gate, mlp.value, mlp.down, attn.q_proj, attn.k_proj, attn.v_proj, attn.out)
        if not isinstance(mlp, SwiGLU):
            raise ValueError(f"layer {i}: the MLP is {type(mlp).__name__}, not SwiGLU")
        if any(getattr(m, "bias", None) is not None for m in mods):
            raise ValueError(f"layer {i}: projections must be bias-free")
        if [tuple(m.weight.shape) for m in mods] != want:
            raise ValueError(f"layer {i}: projection shapes differ from the configuration")
        structural.update(id(m.weight) for m in mods)
        bundle = QKVBundle((attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight), layout)
        bundles.append(bundle)
        blocks.append({"layer_index": i, "mlp": mlp, "in_weight": mlp.gate.weight,
                       "value_weight": mlp.value.weight, "out_weight": mlp.down.weight,
                       "qkv_weight": bundle.logical, "attn_out_weight": attn.out.weight})
    if len(structural) != 7 * len(blocks):
        raise ValueError("a projection matrix is shared between layers or roles")
    embeddings = {id(m.weight) for m in model.modules() if isinstance(m, torch.nn.Embedding)}
    aux = [p for p in params if id(p) not in structural]
    stray = [n for n, p in model.named_parameters()
             if id(p) not in structural and p.ndim > 1 and id(p) not in embeddings]
    if stray:
        raise ValueError(f"matrices with no optimizer role: {stray[:4]}")
    return blocks, bundles, aux


# -- the optimizer ---------------------------------------------------------------
class SwiGLUTILLER:
    """Router + TILLER attention + AdamW for a fixed-SwiGLU MHA decoder, driven by loss masks.

    fp32 parameters; the forward/backward may run under autocast, ``step``
    may not.  A DistributedDataParallel model is accepted (its process group
    carries the probe statistics); no gradient scaler, activation
    checkpointing or model sharding.
    """

    def __init__(self, model, *, group_width=256):
        ddp = isinstance(model, torch.nn.parallel.DistributedDataParallel)
        self.process_group = model.process_group if ddp else None
        self.world = dist.get_world_size(self.process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.process_group) if dist.is_initialized() else 0
        if self.world > 1 and not ddp:
            raise ValueError("with several ranks pass the DistributedDataParallel-wrapped model")
        if self.world > tm.GLOBAL_PROBE_COUNT:
            raise ValueError(f"at most {tm.GLOBAL_PROBE_COUNT} data-parallel ranks (one probe each)")
        model = model.module if ddp else model
        self.model = model
        self.group_width = group_width
        self.blocks, self.bundles, aux = _inspect_model(model, group_width)
        self.parameters = list(model.parameters())
        self.device = self.parameters[0].device
        self.inventory = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
        self.router = SwiGLURouter(self.blocks, group_width, self.process_group)
        cell = {k: CELL[k] for k in ("weight_decay", "momentum", "ns_steps", "beta2", "eps")}
        self.attention = TILLERAttentionOptimizer(self.blocks, self.router, lr=3e-4,
                                                  adjust_lr_fn="match_rms_adamw", **cell)
        self.auxiliary = torch.optim.AdamW(aux, lr=3e-4, betas=AUX_BETAS, eps=CELL["eps"],
                                           weight_decay=0.0)
        self.children = (self.router, self.attention, self.auxiliary)
        self.total_loss_tokens = 0
        self.batch = None

    @property
    def param_groups(self):
        return [g for child in self.children for g in child.param_groups]

    @property
    def completed_steps(self):
        return self.router.completed_steps

    def zero_grad(self):
        if self.batch is not None:
            raise RuntimeError("zero_grad() inside an update (between begin_step and step)")
        for p in self.parameters:
            p.grad = None
        for b in self.bundles:
            b.logical.grad = None

    def _probe_rows(self, masks, probe_indices):
        """This rank's probe positions (flat over the update) and the global loss-token count."""
        valid = torch.cat([m.flatten() for m in masks]).nonzero().flatten()
        want = tm.fixed_global_probe_layout(tm.GLOBAL_PROBE_COUNT, self.rank, self.world).local_probe_count
        counts = torch.tensor([valid.numel(), int(valid.numel() < want)], dtype=torch.int64,
                              device=self.device)
        if dist.is_initialized():
            dist.all_reduce(counts, group=self.process_group)
        if counts[1].item():
            raise ValueError(f"a rank has fewer than its {want} probes' worth of loss-bearing tokens")
        if probe_indices is None:
            probe_indices = valid[tm.evenly_spaced_indices(valid.numel(), want, device=self.device)]
        ok = (probe_indices.dtype == torch.int64 and probe_indices.device == self.device
              and tuple(probe_indices.shape) == (want,)
              and bool(torch.isin(probe_indices, valid).all())
              and (want < 2 or bool((probe_indices[1:] > probe_indices[:-1]).all())))
        bad = torch.tensor(int(not ok), device=self.device)
        if dist.is_initialized():
            dist.all_reduce(bad, group=self.process_group)
        if bad.item():
            raise ValueError(f"probe_indices must be {want} increasing loss-bearing positions of this "
                             "rank's update")
        return probe_indices, int(counts[0].item())

    def begin_step(self, loss_masks, *, probe_indices=None):
        """Open an update: one boolean loss mask per local micro-batch, before any forward.

        ``probe_indices`` (optional): this rank's probe positions, flattened
        over the update's micro-batches; sorted, unique and loss-bearing.
        """
        if self.batch is not None:
            raise RuntimeError("begin_step() twice without step()")
        if not self.model.training:
            raise RuntimeError("begin_step() needs model.train()")
        if any(p.grad is not None for p in self.parameters):
            raise RuntimeError("gradients present: call zero_grad() first")
        masks = [m.detach().clone() for m in loss_masks]
        if not masks or any(m.dtype != torch.bool or m.device != self.device for m in masks):
            raise ValueError("loss_masks: a non-empty list of bool tensors on the model's device")
        probes, total = self._probe_rows(masks, probe_indices)
        per_micro, start = [], 0
        for m in masks:
            here = (probes >= start) & (probes < start + m.numel())
            per_micro.append(probes[here] - start)
            start += m.numel()
        self.batch = {"masks": masks, "backwards": 0, "global_tokens": total}
        self.router.begin(masks, per_micro, total / self.world)

    def backward(self, per_token_losses):
        """Backward of one micro-batch's unreduced per-token losses (in micro-batch order)."""
        if self.batch is None or self.batch["backwards"] >= len(self.batch["masks"]):
            raise RuntimeError("backward() needs begin_step() and at most one call per micro-batch")
        mask = self.batch["masks"][self.batch["backwards"]]
        if per_token_losses.shape != mask.shape or not per_token_losses.requires_grad:
            raise ValueError(f"per-token losses of shape {tuple(mask.shape)} with grad required")
        scale = self.world / self.batch["global_tokens"]
        (per_token_losses[mask].sum() * scale).backward()
        self.batch["backwards"] += 1

    def step(self):
        if torch.is_autocast_enabled(self.device.type):
            raise RuntimeError("step() must run outside autocast")
        if self.batch is None or self.batch["backwards"] != len(self.batch["masks"]):
            raise RuntimeError("step() before every micro-batch's backward()")
        if any(p.grad is None for p in self.parameters):
            raise RuntimeError("a parameter received no gradient")
        self._check_cell()
        lrs = {float(g["lr"]) for g in self.param_groups}
        lr = next(iter(lrs))
        if len(lrs) != 1 or not math.isfinite(lr) or lr <= 0:
            raise ValueError(f"every child needs the same positive scheduled LR, got {sorted(lrs)}")
        norm = torch.nn.utils.clip_grad_norm_(self.parameters, 1.0, error_if_nonfinite=True)
        self.router._clip_factor = min(1.0, 1.0 / (float(norm) + 1e-6))
        self.router.step()
        for b in self.bundles:
            b.gather()
        self.attention.step()
        for b in self.bundles:
            b.scatter()
        self.auxiliary.step()
        tokens = self.batch["global_tokens"]
        self.total_loss_tokens += tokens
        self.batch = None
        return dict(self.router.last_metrics, total_loss_tokens=self.total_loss_tokens,
                    loss_tokens_this_update=tokens, lr=lr, preclip_norm=float(norm))

    def _check_cell(self):
        r, a = self.router.param_groups[0], self.attention.param_groups[0]
        drift = [r.get("version") != VERSION, r["weight_decay"] != CELL["weight_decay"],
                 a["weight_decay"] != CELL["weight_decay"]]
        drift += [g["weight_decay"] != 0.0 or tuple(g["betas"]) != AUX_BETAS or g["eps"] != CELL["eps"]
                  for g in self.auxiliary.param_groups]
        if any(drift):
            raise ValueError("the fixed SwiGLU TILLER hyper-parameters were changed")

    # -- checkpoints -------------------------------------------------------------
    def state_dict(self):
        if self.batch is not None or not self.router._attention_consumed:
            raise RuntimeError("state_dict() only between updates")
        return {"version": VERSION, "group_width": self.group_width, "world_size": self.world,
                "inventory": self.inventory, "completed_steps": self.completed_steps,
                "total_loss_tokens": self.total_loss_tokens,
                "children": [c.state_dict() for c in self.children]}

    def load_state_dict(self, state):
        if self.batch is not None:
            raise RuntimeError("load_state_dict() inside an update")
        identity = {"version": VERSION, "group_width": self.group_width, "world_size": self.world,
                    "inventory": self.inventory}
        wrong = [k for k, v in identity.items() if state.get(k) != v]
        if wrong or len(state.get("children", ())) != len(self.children):
            raise ValueError(f"checkpoint belongs to another SwiGLU TILLER set-up ({wrong or 'children'})")
        steps, tokens = state.get("completed_steps"), state.get("total_loss_tokens")
        if not (type(steps) is int and type(tokens) is int and steps >= 0 and tokens >= 0
                and (steps == 0) == (tokens == 0)):
            raise ValueError(f"bad counters in checkpoint: steps={steps!r} tokens={tokens!r}")
        for child, saved in zip(self.children, state["children"]):
            child.load_state_dict(saved)
        if steps != self.completed_steps:
            raise ValueError(f"checkpoint says {steps} updates, the router ledger {self.completed_steps}")
        if steps:
            self._check_restored(steps)
        self.router._attention_update = steps
        self.router._attention_consumed = True
        self.total_loss_tokens = tokens
        self._check_cell()

    def _check_restored(self, steps):
        """State every child must hold after ``steps`` updates (finite, right shapes)."""
        L, G = len(self.blocks), self.router.groups

        def fine(t, shape, nonneg=False):
            return (torch.is_tensor(t) and tuple(t.shape) == tuple(shape) and t.dtype == torch.float32
                    and bool(torch.isfinite(t).all()) and (not nonneg or bool((t >= 0).all())))

        anchor = self.router.anchor
        self.router._previous_ledger()  # validates the persistent ledger rows
        failures = []
        route = anchor.get("swiglu_participation")
        if not (fine(route, (L, G, 2), True) and bool((route <= 1).all())):
            failures.append("cached participation route")
        ref = anchor.get("factorized_rfd_reference_row_norm")
        if not (torch.is_tensor(ref) and ref.numel() == 1 and bool(torch.isfinite(ref).all())
                and bool((ref >= 0).all())):
            failures.append("functional calibration")
        for role, params in self.router.roles.items():
            if not all(fine(self.router.state[p].get("momentum_buffer"), p.shape) for p in params):
                failures.append(f"{role} momentum")
            for axis, size in (("row", self.router.width), ("column", self.router.external)):
                if not fine(anchor.get(f"swiglu_{role}_{axis}_second_moment"), (L, G, size), True):
                    failures.append(f"{role} {axis} moments")
        att = self.attention.state[self.attention.role_parameters["qkv"][0]]
        counters = [att.get("compact_response_homotopy_router_update"),
                    att.get("factorized_adaptive_tangent_updates")]
        counters += [int(self.auxiliary.state[p]["step"]) for g in self.auxiliary.param_groups
                     for p in g["params"]]
        if any(c != steps for c in counters):
            failures.append("child update counters")
        for role, params in self.attention.role_parameters.items():
            if not all(fine(self.attention.state[p].get("momentum_buffer"), p.shape) for p in params):
                failures.append(f"attention {role} momentum")
            key = "qkv" if role == "qkv" else "attention_output"
            for axis, size in (("row", params[0].shape[0]), ("column", params[0].shape[1])):
                if not fine(att.get(f"factorized_adaptive_tangent_{key}_{axis}_second_moment"),
                            (L, 1, size), True):
                    failures.append(f"attention {role} {axis} moments")
        for g in self.auxiliary.param_groups:
            for p in g["params"]:
                if not all(fine(self.auxiliary.state[p].get(k), p.shape) for k in ("exp_avg", "exp_avg_sq")):
                    failures.append("AdamW moments")
                    break
        if failures:
            raise ValueError("restored optimizer state is invalid: " + ", ".join(sorted(set(failures))))

    def close(self):
        self.router.close()
