"""TILLER for a fixed SwiGLU MLP (no GRAIN) - the separately named extension of
reference experiments/swiglu_tiller/tiller_swiglu.py:1-525.

With a fixed activation the response congruence is exactly one, so the
response-drift rotation of the chord vanishes; what remains is the
participation route (trace-ratio statistics of ``J = [diag(dg), diag(dv)]``
and of the features), the factorized adaptive-tangent chord, and the same
functional loss ledger and equal-budget transaction as the GRAIN router
(:meth:`TILLERRouter._advance_rows` / :meth:`TILLERRouter._transaction` are
shared, not re-implemented).  Three native matrices form two logical roles:
the joint gate/value incoming role (rows grouped by channel group) and the
down projection (columns grouped).  The attention matrices are driven by the
standard :class:`TILLERAttentionOptimizer` with congruence one.

Use: ``opt = SwiGLUTILLER(model)``; per update ``opt.zero_grad()``,
``opt.begin_step(masks)``, one ``opt.backward(per_token_losses)`` per
micro-batch, ``opt.step()`` (outside autocast).  Checkpoints carry the
version ``tiller_swiglu_fixed_v1`` and are validated on load.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import tiller_math as tm
from .newton_schulz import match_rms_adamw_adjustment, rational_group_zero_power
from .tiller import TILLERAttentionOptimizer, TILLERRouter, foreach_apply, foreach_nesterov

VERSION = "tiller_swiglu_fixed_v1"


def swiglu_factors(gate, value):
    """(features, d features / d gate, d features / d value) of silu(gate) * value."""
    sig = gate.sigmoid()
    silu = F.silu(gate)
    return silu * value, value * sig * (1 + gate * (1 - sig)), silu


def group_scores(inputs, gate, value, features, cotangent, down_weight, gate_direction, value_direction,
                 down_direction, group_width):
    """Loss-cotangent-contracted JVP of the MLP, one column per channel group."""
    _, dg, dv = swiglu_factors(gate, value)
    pull = cotangent @ down_weight
    incoming = ((inputs @ gate_direction.T) * dg + (inputs @ value_direction.T) * dv) * pull
    outgoing = features * (cotangent @ down_direction)
    return (incoming + outgoing).reshape(len(inputs), -1, group_width).sum(-1)


def participation_statistics(gate, value, features, cotangent, down_weight, width):
    """Weighted trace-ratio participation numerators/denominators (reduce before dividing)."""
    _, dg, dv = swiglu_factors(gate, value)
    energy = (dg.square() + dv.square()).reshape(len(gate), -1, width)
    h2 = features.square().reshape_as(energy)
    tiny = torch.finfo(gate.dtype).tiny
    incoming = energy.sum(-1).square() / (width * energy.square().sum(-1)).clamp_min(tiny)
    outgoing = h2.sum(-1).square() / (width * h2.square().sum(-1)).clamp_min(tiny)
    pulled = (cotangent @ down_weight).reshape_as(energy)
    in_w = (energy * pulled.square()).mean(-1)
    out_w = cotangent.square().mean(-1, keepdim=True).expand_as(in_w)
    return torch.stack(((incoming * in_w).sum(0), in_w.sum(0), (outgoing * out_w).sum(0), out_w.sum(0)), -1)


class SwiGLURouter(torch.optim.Optimizer):
    """Gate/value/down matrices of every layer; ledger and transaction shared with TILLER."""

    _previous_ledger = TILLERRouter._previous_ledger
    _advance_rows = TILLERRouter._advance_rows
    _transaction = TILLERRouter._transaction
    momentum = 0.95
    ns_steps = 5
    strict = True

    def __init__(self, blocks, group_width, process_group=None):
        self.pairs = blocks
        self.loss_probe_group = process_group
        self.width = int(group_width)
        self.hidden, self.external = blocks[0]["in_weight"].shape
        self.groups = self.hidden // self.width
        self.roles = {"gate": [b["in_weight"] for b in blocks], "value": [b["value_weight"] for b in blocks],
                      "down": [b["out_weight"] for b in blocks]}
        super().__init__([{"params": [p for ps in self.roles.values() for p in ps], "lr": 3e-4,
                           "weight_decay": 0.1, "version": VERSION}], {})
        self._attention_consumed = True
        self._attention_update = 0
        self._clip_factor = None
        self._capture_telemetry_next_step = False
        self._rfd_rows = self._rfd_selection = None
        self._rfd_gradient_scale = self._rfd_decay_derivative = None
        self.active = False
        self.last_metrics = {}
        self.handles = []
        for i, b in enumerate(blocks):
            self.handles.append(b["mlp"].register_forward_pre_hook(self._input_hook(i)))
            for role in ("gate", "value"):
                self.handles.append(b[role].register_forward_hook(self._projection_hook(i, role)))
            self.handles.append(b["down"].register_forward_pre_hook(self._feature_hook(i)))
            self.handles.append(b["mlp"].register_forward_hook(self._output_hook(i)))

    @property
    def anchor(self):
        return self.state[self.pairs[0]["in_weight"]]

    @property
    def completed_steps(self):
        return int(self.anchor.get("factorized_rfd_step", 0))

    def begin(self, masks, indices, loss_denominator):
        if self.active or not self._attention_consumed:
            raise RuntimeError("finish the previous optimizer/attention update first")
        self.active = True
        self.refresh = self.completed_steps % 8 == 0
        self.masks, self.indices, self.loss_denominator = masks, indices, loss_denominator
        self.calls = [0] * len(self.pairs)
        self.records = [[] for _ in self.pairs]
        self.pending = [None] * len(self.pairs)
        self._clip_factor = None

    # -- probe capture -------------------------------------------------------
    def _input_hook(self, layer):
        @torch.no_grad()
        def capture(module, args):
            if not module.training:
                return
            if not self.active:
                raise RuntimeError("call begin_step before a training forward")
            micro = self.calls[layer]
            if micro >= len(self.masks) or self.pending[layer] is not None:
                raise RuntimeError("reentrant/checkpointed MLP forwards are not supported")
            x = args[0].detach().reshape(-1, self.external)
            if len(x) != self.masks[micro].numel():
                raise RuntimeError("MLP rows differ from the declared loss mask")
            self.calls[layer] += 1
            if self.refresh:
                ids = self.indices[micro]
                self.pending[layer] = {"indices": ids, "x": x[ids].clone()}
        return capture

    def _projection_hook(self, layer, role):
        @torch.no_grad()
        def capture(module, args, output):
            if self.active and self.refresh:
                rec = self.pending[layer]
                if rec is None or role in rec:
                    raise RuntimeError("SwiGLU projection capture is unaligned")
                rec[role] = output.detach().reshape(-1, self.hidden)[rec["indices"]].float().clone()
        return capture

    def _feature_hook(self, layer):
        @torch.no_grad()
        def capture(module, args):
            if self.active and self.refresh:
                rec = self.pending[layer]
                rec["h"] = args[0].detach().reshape(-1, self.hidden)[rec["indices"]].float().clone()
        return capture

    def _output_hook(self, layer):
        def capture(module, args, output):
            if self.active and self.refresh:
                rec = self.pending[layer]
                if rec is None or "h" not in rec or not output.requires_grad:
                    raise RuntimeError("missing differentiable SwiGLU output")
                self.records[layer].append(rec)
                self.pending[layer] = None

                def backward(gradient):
                    if "cotangent" in rec:
                        raise RuntimeError("a probe was backpropagated twice")
                    rec["cotangent"] = gradient.detach().reshape(-1, self.external)[rec["indices"]].float().clone()
                    return gradient
                output.register_hook(backward)
        return capture

    def _packets(self):
        out = []
        for recs in self.records:
            if len(recs) != len(self.masks) or any("cotangent" not in r for r in recs):
                raise RuntimeError("incomplete functional probe backward")
            packet = [torch.cat([r[k] for r in recs]).float() for k in ("x", "gate", "value", "h", "cotangent")]
            packet[-1].mul_(self.loss_denominator * self._clip_factor)
            out.append(packet)
        return out

    def consume_response_homotopy(self):
        if self._attention_consumed:
            raise RuntimeError("attention route consumed twice")
        self._attention_consumed = True
        route = self.anchor["swiglu_participation"]
        intrinsic = (route[..., 0].mean(-1) * route[..., 1].mean(-1)).clamp(0, 1).sqrt()
        return intrinsic, torch.ones_like(intrinsic), self._attention_update

    def _chord_state(self, parent, axis, key_prefix):
        shape = tm.grouped_shape(parent, groups=self.groups, width=self.width, axis=axis)
        rk, ck = key_prefix + "_row_second_moment", key_prefix + "_column_second_moment"
        a = self.anchor
        if rk not in a:
            a[rk] = torch.zeros(shape[:-1], device=parent.device, dtype=torch.float32)
        if ck not in a:
            a[ck] = torch.zeros(shape[:2] + shape[-1:], device=parent.device, dtype=torch.float32)
        return a[rk], a[ck]

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("closures are incompatible with the explicit probe batch")
        if not self.active or not self._attention_consumed or self._clip_factor is None:
            raise RuntimeError("missing batch, synchronized clipping, or attention update")
        if any(n != len(self.masks) for n in self.calls):
            raise RuntimeError("missing MLP micro-batch forwards")
        step = self.completed_steps + 1
        lr, wd = (float(self.param_groups[0][k]) for k in ("lr", "weight_decay"))
        packets = self._packets() if self.refresh else None
        if self.refresh:
            stats = torch.stack([participation_statistics(g, v, h, c, b["out_weight"].detach().float(), self.width)
                                 for b, (x, g, v, h, c) in zip(self.pairs, packets)])
            if dist.is_initialized():
                dist.all_reduce(stats, group=self.loss_probe_group)
            nums, dens = stats[..., (0, 2)], stats[..., (1, 3)]
            self.anchor["swiglu_participation"] = torch.where(
                dens > 0, nums / dens.clamp_min(1e-38), torch.ones_like(nums)).clamp(0, 1)
        route = self.anchor["swiglu_participation"]
        directions, exact, moment, energies = {}, {}, {}, []
        for role, params in self.roles.items():
            axis = "columns" if role == "down" else "rows"
            momentum = foreach_nesterov(self, params, self.momentum)
            grad = torch.stack([p.grad for p in params]).float()
            parent = rational_group_zero_power(momentum, 5, groups=self.groups, width=self.width).float()
            row, col = self._chord_state(parent, axis, "swiglu_" + role)
            pg, restore = tm.group_view(parent, groups=self.groups, width=self.width, axis=axis)
            mg, _ = tm.group_view(momentum, groups=self.groups, width=self.width, axis=axis)
            gg, _ = tm.group_view(grad, groups=self.groups, width=self.width, axis=axis)
            part = route[..., 1 if role == "down" else 0]
            sel_g, _ = tm.adaptive_tangent_chord(pg, mg, gg, row, col, part, torch.ones_like(part), step)
            selected = restore(sel_g) * match_rms_adamw_adjustment(params[0].shape)
            directions[role] = selected
            d, _ = tm.group_view(selected, groups=self.groups, width=self.width, axis=axis)
            exact[role] = (d * gg).sum((-2, -1)).flatten()
            moment[role] = (d * mg).sum((-2, -1)).flatten()
            energies.append(d.square().sum((-2, -1)).flatten())
        # the incoming logical role is the gate/value pair
        exact_by_role = torch.stack((exact["gate"] + exact["value"], exact["down"]))
        momentum_by_role = torch.stack((moment["gate"] + moment["value"], moment["down"]))
        weights = torch.stack(energies).sum(0)
        self._rfd_rows = None
        self._rfd_gradient_scale = None
        self._rfd_decay_derivative = sum((p.grad * p).sum() * wd for ps in self.roles.values() for p in ps)
        if self.refresh:
            scores, decay = [], []
            for layer, (b, packet) in enumerate(zip(self.pairs, packets)):
                args = (*packet, b["out_weight"].detach().float())
                scores.append(group_scores(*args, *(directions[r][layer] for r in self.roles), self.width))
                decay.append(group_scores(*args, b["in_weight"].detach().float() * wd,
                                          b["value_weight"].detach().float() * wd,
                                          b["out_weight"].detach().float() * wd, self.width).sum(-1))
            local = torch.cat((torch.stack(scores, 1).flatten(1), torch.stack(decay).sum(0)[:, None]), 1)
            rows = _gather_probe_rows(local, expected=tm.GLOBAL_PROBE_COUNT, group=self.loss_probe_group)
            self._advance_rows(rows[:, :-1], rows[:, -1], functional=True)
        layer_ids = torch.arange(len(self.pairs), device=weights.device).repeat_interleave(self.groups)
        self._transaction(exact_by_role, momentum_by_role, weights, layer_ids, eta=lr)
        coeff = self._rfd_selection.coefficients.reshape(len(self.pairs), self.groups)
        for role, params in self.roles.items():
            axis = "columns" if role == "down" else "rows"
            blocks, restore = tm.group_view(directions[role], groups=self.groups, width=self.width, axis=axis)
            foreach_apply(params, restore(blocks * coeff[..., None, None]), decay=1 - lr * wd, alpha=-lr)
        self._attention_update = step
        self._attention_consumed = False
        sel = self._rfd_selection
        self.last_metrics = dict(version=VERSION, step=step, functional_refresh=self.refresh,
                                 ledger_step=self.completed_steps, beta2=0.95, fixed_activation_congruence=1.0,
                                 response_departure_energy=0.0, proposal_accepted=bool(sel.accepted.item()),
                                 coefficient_abs_deviation_mean=float((coeff - 1).abs().mean()),
                                 coefficient_abs_deviation_max=float((coeff - 1).abs().max()),
                                 budget_residual=float(sel.budget_residual.item()),
                                 ledger_measurement="functional" if self.refresh else "gradient_surrogate")
        self.active = False
        self.records, self.pending = [], []
        self._clip_factor = None

    def close(self):
        for h in self.handles:
            h.remove()
        self.handles.clear()


def _gather_probe_rows(local, *, expected, group=None):
    """All ranks' probe rows in rank order (variable local counts, ``expected`` in total)."""
    if not (dist.is_available() and dist.is_initialized()):
        if local.shape[0] != expected:
            raise RuntimeError("probe row count differs from the global probe layout")
        return local
    world = dist.get_world_size(group)
    count = torch.tensor([local.shape[0]], device=local.device, dtype=torch.int64)
    counts = [torch.zeros_like(count) for _ in range(world)]
    dist.all_gather(counts, count, group=group)
    counts = [int(c.item()) for c in counts]
    if sum(counts) != expected:
        raise RuntimeError("probe row count differs from the global probe layout")
    width = max(counts)
    padded = local.new_zeros((width, local.shape[1]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)])


class SwiGLUTILLER:
    """Router + attention + AdamW for a fixed-SwiGLU MHA decoder with explicit loss masks."""

    def __init__(self, model, *, group_width=256):
        from ..mha.optim import AttentionLayout, QKVBundle
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        model = model.module if hasattr(model, "module") else model
        c = model.config
        if getattr(model, "grain", True) or not isinstance(c, dict):
            raise ValueError("requires the fixed-SwiGLU MHA decoder")
        if c["num_attention_heads"] != 16 or c["num_key_value_heads"] != 16 or c["head_dim"] * 16 != c["hidden_size"]:
            raise ValueError("requires sixteen equal heads with a square output")
        if type(group_width) is not int or group_width < 1 or c["intermediate_size"] % group_width:
            raise ValueError("the group width must divide the SwiGLU intermediate width")
        if c["intermediate_size"] <= c["hidden_size"]:
            raise ValueError("requires an expanded SwiGLU hidden width")
        if len(model.layers) * (c["intermediate_size"] // group_width) < 2:
            raise ValueError("TILLER needs at least two coordination coordinates")
        self.parameters = list(model.parameters())
        self.model = model
        device = self.parameters[0].device
        if any(p.dtype != torch.float32 or p.device != device or not p.requires_grad for p in self.parameters):
            raise ValueError("all model parameters must be trainable fp32 on one device")
        self.device = device
        self.inventory = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
        self.group_width = group_width
        self.blocks, self.bundles, structural = [], [], []
        layout = AttentionLayout(c["hidden_size"], 16, 16, c["head_dim"])
        for i, layer in enumerate(model.layers):
            mlp, attn = layer.mlp, layer.attn
            mods = [mlp.gate, mlp.value, mlp.down, attn.q_proj, attn.k_proj, attn.v_proj, attn.out]
            d, h = c["hidden_size"], c["intermediate_size"]
            if [tuple(m.weight.shape) for m in mods] != [(h, d), (h, d), (d, h)] + [(d, d)] * 4:
                raise ValueError("projection shapes differ from the model configuration")
            structural.extend(m.weight for m in mods)
            bundle = QKVBundle((attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight), layout)
            self.bundles.append(bundle)
            self.blocks.append(dict(layer_index=i, mlp=mlp, gate=mlp.gate, value=mlp.value, down=mlp.down,
                                    in_weight=mlp.gate.weight, value_weight=mlp.value.weight,
                                    out_weight=mlp.down.weight, qkv_weight=bundle.logical,
                                    attn_out_weight=attn.out.weight))
        ids = {id(p) for p in structural}
        aux = [p for p in self.parameters if id(p) not in ids]
        embeds = {id(m.weight) for m in model.modules() if isinstance(m, torch.nn.Embedding)}
        if any(p.ndim > 1 and id(p) not in embeds for p in aux):
            raise ValueError("unrecognized auxiliary matrix; explicit routing is required")
        self.router = SwiGLURouter(self.blocks, group_width)
        kw = dict(lr=3e-4, weight_decay=0.1, momentum=0.95, ns_steps=5, beta2=0.95, eps=1e-8)
        self.attention = TILLERAttentionOptimizer(self.blocks, self.router, adjust_lr_fn="match_rms_adamw", **kw)
        self.auxiliary = torch.optim.AdamW(aux, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
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
            raise RuntimeError("cannot discard an unfinished update")
        for p in self.parameters:
            p.grad = None
        for b in self.bundles:
            b.logical.grad = None

    def begin_step(self, loss_masks, *, probe_indices=None):
        """Declare every local micro-batch's loss mask before any forward."""
        if self.batch is not None:
            raise RuntimeError("optimizer update already active")
        if not self.model.training:
            raise RuntimeError("call model.train() before begin_step")
        if any(p.grad is not None for p in self.parameters):
            raise RuntimeError("call zero_grad before begin_step")
        masks = [m.detach().clone() for m in loss_masks]
        if not masks or any(m.dtype != torch.bool or m.device != self.device for m in masks):
            raise ValueError("a nonempty list of boolean masks on the model device is required")
        valid = torch.cat([m.flatten() for m in masks]).nonzero().flatten()
        count = tm.fixed_global_probe_layout(tm.GLOBAL_PROBE_COUNT, self.rank, self.world).local_probe_count
        counts = torch.tensor([len(valid), int(len(valid) < count)], dtype=torch.int64, device=self.device)
        if dist.is_initialized():
            dist.all_reduce(counts)
        if counts[1].item():
            raise ValueError("each rank needs enough loss-bearing positions for its probes")
        total = int(counts[0].item())
        if probe_indices is None:
            probe_indices = valid[tm.evenly_spaced_indices(len(valid), count, device=self.device)]
        ok = not (probe_indices.dtype != torch.int64 or probe_indices.device != self.device
                  or tuple(probe_indices.shape) != (count,) or not bool(torch.isin(probe_indices, valid).all())
                  or (count > 1 and not bool((probe_indices[1:] > probe_indices[:-1]).all())))
        if not ok:
            raise ValueError("probe identities must be sorted, unique, local loss-bearing positions")
        indices, offset = [], 0
        for m in masks:
            indices.append(probe_indices[(probe_indices >= offset) & (probe_indices < offset + m.numel())] - offset)
            offset += m.numel()
        self.batch = dict(masks=masks, next_backward=0, global_tokens=total)
        self.router.begin(masks, indices, total / self.world)

    def backward(self, per_token_losses):
        if self.batch is None or self.batch["next_backward"] >= len(self.batch["masks"]):
            raise RuntimeError("begin_step and exactly one backward per micro-batch are required")
        mask = self.batch["masks"][self.batch["next_backward"]]
        if per_token_losses.shape != mask.shape or not per_token_losses.requires_grad:
            raise ValueError("pass differentiable unreduced per-token losses matching the mask")
        (per_token_losses[mask].sum() * (self.world / self.batch["global_tokens"])).backward()
        self.batch["next_backward"] += 1

    def step(self):
        if torch.is_autocast_enabled(self.device.type):
            raise RuntimeError("optimizer.step must run outside autocast")
        if self.batch is None or self.batch["next_backward"] != len(self.batch["masks"]):
            raise RuntimeError("the update has incomplete backwards")
        if any(p.grad is None for p in self.parameters):
            raise RuntimeError("missing parameter gradient")
        lrs = [float(g["lr"]) for g in self.param_groups]
        if any(not math.isfinite(lr) or lr <= 0 for lr in lrs) or len(set(lrs)) != 1:
            raise ValueError("all optimizer children require the same positive scheduled LR")
        norm = torch.nn.utils.clip_grad_norm_(self.parameters, 1.0, error_if_nonfinite=True)
        self.router._clip_factor = min(1.0, 1.0 / (float(norm) + 1e-6))
        self.router.step()
        for b in self.bundles:
            b.gather()
        self.attention.step()
        for b in self.bundles:
            b.scatter()
        self.auxiliary.step()
        self.total_loss_tokens += self.batch["global_tokens"]
        metrics = dict(self.router.last_metrics, total_loss_tokens=self.total_loss_tokens,
                       loss_tokens_this_update=self.batch["global_tokens"], lr=lrs[0], preclip_norm=float(norm))
        self.batch = None
        return metrics

    def state_dict(self):
        if self.batch is not None or not self.router._attention_consumed:
            raise RuntimeError("checkpoint only at a completed optimizer boundary")
        return dict(version=VERSION, group_width=self.group_width, world_size=self.world,
                    inventory=self.inventory, completed_steps=self.completed_steps,
                    total_loss_tokens=self.total_loss_tokens, children=[c.state_dict() for c in self.children])

    def load_state_dict(self, state):
        if self.batch is not None:
            raise RuntimeError("cannot restore in the middle of an update")
        if (state.get("version") != VERSION or state.get("group_width") != self.group_width
                or state.get("world_size") != self.world or state.get("inventory") != self.inventory
                or len(state.get("children", ())) != 3):
            raise ValueError("SwiGLU TILLER checkpoint identity/inventory mismatch")
        steps, tokens = state.get("completed_steps"), state.get("total_loss_tokens")
        if (type(steps) is not int or steps < 0 or type(tokens) is not int or tokens < 0
                or (steps == 0) != (tokens == 0)):
            raise ValueError("invalid persisted optimizer counters")
        for child, saved in zip(self.children, state["children"]):
            child.load_state_dict(saved)
        if steps != self.completed_steps:
            raise ValueError("ledger and optimizer counters disagree")
        if steps:
            anchor = self.router.anchor
            route = anchor.get("swiglu_participation")
            if (route is None or tuple(route.shape) != (len(self.blocks), self.router.groups, 2)
                    or not bool(torch.isfinite(route).all() & (route >= 0).all() & (route <= 1).all())):
                raise ValueError("invalid cached response route")
            ref = anchor.get("factorized_rfd_reference_row_norm")
            if ref is None or ref.numel() != 1 or not bool(torch.isfinite(ref).all() & (ref >= 0).all()):
                raise ValueError("invalid functional calibration")
            attn = self.attention.state[self.attention.role_parameters["qkv"][0]]
            if (attn.get("compact_response_homotopy_router_update") != steps
                    or attn.get("factorized_adaptive_tangent_updates") != steps):
                raise ValueError("optimizer-child counters disagree")
        self.router._attention_update = steps
        self.router._attention_consumed = True
        self.total_loss_tokens = tokens

    def close(self):
        self.router.close()
