"""Optimizer composition of the MHA study (reference experiments/mha_1b_tokens/
optim.py:1-190, packing.py:1-34, tiller_then_muon.py:1-130).

All structural matrices decay at 0.1; tied embeddings, norm vectors and
GRAIN coefficients take AdamW without decay; AdamW uses (0.9, 0.95), eps
1e-8; Muon/TILLER use momentum 0.95, NS5 and the match-RMS LR adjustment.
Clipping is one global norm at 1.0 after gradient synchronisation and the
realised norm is handed to TILLER.  TILLER's attention role expects the
fused ``[3d, d]`` QKV matrix; :class:`QKVBundle` packs the native Q/K/V
weights (and gradients) into that view before the attention step and
scatters the result back after it.  ``grain_tiller100_muon`` runs TILLER for
100 updates, then hands its momentum to Muon (Q/K/V split back per owner),
keeps the AdamW child, removes TILLER's hooks and validates the handoff in
checkpoints.
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass

import torch

from ..optim.adamw import FusedAdamW
from ..optim.muon import Muon
from ..optim.tiller import TILLERAttentionOptimizer, TILLERRouter, configure_microbatch_count
from ..train.engine import clip_grad_norm
from . import config as C
from .config import CONDITIONS, MHA_MUON, MHA_SWITCH, MHA_TILLER, SWITCH_CONDITIONS, SWITCH_UPDATE

POLICY = {
    "version": "tiller100_then_native_muon_v1", "tiller_updates": SWITCH_UPDATE, "tiller_beta2": 0.95,
    "functional_probe_interval_steps": 8, "functional_probe_count": 32, "sketch_rank": 64,
    "tiller_variant": "original_grain_tiller",
    "momentum_transfer": "exact; unpack logical QKV into native Q/K/V",
    "auxiliary": "retain AdamW object, moments, counters and hyperparameters",
    "model": "GRAIN throughout; no activation or parameter conversion",
}


@dataclass(frozen=True)
class AttentionLayout:
    residual_width: int
    q_heads: int
    kv_heads: int
    head_dim: int

    def __post_init__(self):
        if self.q_heads != 16 or self.kv_heads != 16 or self.head_dim * 16 != self.residual_width:
            raise ValueError("TILLER attention requires 16 equal heads and a square output")

    @property
    def widths(self):
        return (self.residual_width,) * 3


class QKVBundle:
    """Packing workspace; the native Q/K/V parameters remain the only owners."""

    def __init__(self, parameters, layout):
        self.parameters, self.layout = tuple(parameters), layout
        if len(self.parameters) != 3 or any(tuple(p.shape) != (w, layout.residual_width)
                                            for p, w in zip(self.parameters, layout.widths)):
            raise ValueError("native Q/K/V packing inventory mismatch")
        if len({id(p) for p in self.parameters}) != 3:
            raise ValueError("duplicated Q/K/V owner")
        if any(p.dtype != torch.float32 or p.device != self.parameters[0].device for p in self.parameters):
            raise ValueError("native attention parameters must share one device and fp32 master precision")
        self.logical = torch.cat([p.detach() for p in self.parameters], dim=0)

    @torch.no_grad()
    def gather(self):
        if any(p.grad is None for p in self.parameters):
            raise RuntimeError("missing native attention gradient")
        self.logical.copy_(torch.cat([p.detach() for p in self.parameters], dim=0))
        self.logical.grad = torch.cat([p.grad.detach() for p in self.parameters], dim=0)

    @torch.no_grad()
    def scatter(self):
        for p, value in zip(self.parameters, self.logical.split(self.layout.widths, dim=0)):
            p.copy_(value)


def collect_blocks(model):
    cfg = model.config
    layout = AttentionLayout(cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"],
                             cfg["head_dim"])
    blocks = []
    for index, block in enumerate(model.layers):
        mlp, act = block.mlp, block.mlp.rlb_activation
        bundle = QKVBundle((block.attn.q_proj.weight, block.attn.k_proj.weight, block.attn.v_proj.weight), layout)
        blocks.append(dict(layer_index=index, num_layers=len(model.layers), block=block, mlp=mlp, module=act,
                           in_weight=mlp.in_proj.weight, out_weight=mlp.out_proj.weight,
                           qkv_weight=bundle.logical, qkv_bundle=bundle, attention_layout=layout,
                           attn_out_weight=block.attn.out.weight, numerator=act.numerator,
                           denominator=act.denominator, coeff_logits=None, centers=None, beta=None,
                           coeff_limit=0.0, groups=act.groups, hidden_dim=act.hidden_dim, eps=act.eps))
    return blocks


class CampaignOptimizer:
    schema = "portable_mha_optimizer_v1"

    def __init__(self, model, condition, accumulation, children, roles, inventory, router=None, attention=None,
                 bundles=()):
        self.condition, self.accumulation = condition, accumulation
        self.children, self.roles = tuple(children), tuple(roles)
        self.parameter_inventory = inventory
        self.parameters = tuple(p for p in model.parameters() if p.requires_grad)
        self.router, self.attention, self.bundles = router, attention, tuple(bundles)
        self.completed_steps = 0
        self.last_clipping = None
        self._clipping_recorded = False

    @property
    def param_groups(self):
        return [g for child in self.children for g in child.param_groups]

    def zero_grad(self, set_to_none=True):
        if self._clipping_recorded:
            raise RuntimeError("cannot discard gradients after clipping before step")
        for p in self.parameters:
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.detach_()
                    p.grad.zero_()
        for child in self.children:
            child.zero_grad(set_to_none=set_to_none)

    def record_realized_clipping(self, preclip_norm, max_norm=1.0):
        norm = float(preclip_norm)
        if self._clipping_recorded or max_norm != 1.0 or not math.isfinite(norm) or norm < 0:
            raise ValueError("one finite realized clipping norm at max_norm=1 is required")
        if self.router is not None:
            self.router.record_realized_clipping(norm, max_norm)
        self.last_clipping = dict(preclip_norm=norm, max_norm=float(max_norm), factor=min(1.0, max_norm / (norm + 1e-6)))
        self._clipping_recorded = True

    def clip_grad_norm(self, max_norm=1.0):
        if max_norm != 1.0 or self._clipping_recorded:
            raise ValueError("exactly one clipping operation at max_norm=1 is required")
        norm = clip_grad_norm(self.parameters, max_norm)
        if not torch.isfinite(norm):
            raise RuntimeError("non-finite gradient norm")
        self.record_realized_clipping(norm, max_norm)
        return norm

    def step(self):
        if not self._clipping_recorded:
            raise RuntimeError("record clipping after synchronized backward and before optimizer step")
        for child in self.children:
            if child is self.attention:
                for b in self.bundles:
                    b.gather()
            child.step()
            if child is self.attention:
                for b in self.bundles:
                    b.scatter()
        self.completed_steps += 1
        self._clipping_recorded = False

    def state_dict(self):
        if self._clipping_recorded:
            raise RuntimeError("checkpoint only at completed optimizer boundaries")
        if self.router is not None and self.completed_steps == 0:
            raise RuntimeError("a TILLER checkpoint requires at least one completed optimizer step")
        return dict(schema=self.schema, condition=self.condition, accumulation=self.accumulation, roles=self.roles,
                    inventory=self.parameter_inventory, completed_steps=self.completed_steps,
                    last_clipping=self.last_clipping, children=[c.state_dict() for c in self.children])

    def load_state_dict(self, state):
        if (state.get("schema") != self.schema or state.get("condition") != self.condition
                or state.get("accumulation") != self.accumulation or tuple(state.get("roles", ())) != self.roles
                or state.get("inventory") != self.parameter_inventory
                or len(state.get("children", ())) != len(self.children)):
            raise ValueError("campaign optimizer checkpoint configuration/inventory mismatch")
        if type(state.get("completed_steps")) is not int or state["completed_steps"] < 0:
            raise ValueError("invalid optimizer step counter")
        if self.router is not None and state["completed_steps"] == 0:
            raise ValueError("a TILLER checkpoint requires at least one completed optimizer step")
        for child, saved in zip(self.children, state["children"]):
            child.load_state_dict(saved)
        self.completed_steps = state["completed_steps"]
        self.last_clipping = state["last_clipping"]
        self._clipping_recorded = False


def build_optimizer(model, condition, lr=3e-4, accumulation=4):
    if condition not in CONDITIONS or type(accumulation) is not int or accumulation < 1:
        raise ValueError("invalid campaign condition or accumulation")
    if not math.isfinite(lr) or lr <= 0:
        raise ValueError("optimizer LR must be finite and positive")
    model = model.module if hasattr(model, "module") else model
    if condition in SWITCH_CONDITIONS:
        if not model.grain:
            raise ValueError("the switch experiment requires GRAIN throughout")
        return TillerThenMuon(model, lr, accumulation, condition=condition)
    if bool(model.grain) != (condition == MHA_TILLER):
        raise ValueError("condition does not match model activation")
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    structural, children, roles, bundles = [], [], [], []
    router = attention = None
    if condition == MHA_TILLER:
        configure_microbatch_count(accumulation)
        blocks = collect_blocks(model)
        bundles = [b["qkv_bundle"] for b in blocks]
        structural = [b[k] for b in blocks for k in ("in_weight", "out_weight", "attn_out_weight")]
        structural += [p for bundle in bundles for p in bundle.parameters]
        kw = dict(lr=3e-4, weight_decay=0.1, momentum=0.95, ns_steps=5, beta2=0.95, eps=1e-8)
        router = TILLERRouter(blocks, **kw)
        attention = TILLERAttentionOptimizer(blocks, router, adjust_lr_fn="match_rms_adamw", **kw)
        roles += ["tiller_router", "tiller_attention_mha_reference"]
        children += [router, attention]
    elif condition == MHA_MUON:
        structural = [p for n, p in named if p.ndim == 2 and n != "embed_tokens.weight"]
        children.append(Muon(structural, lr=lr, weight_decay=0.1, momentum=0.95, ns_steps=5,
                             adjust_lr_fn="match_rms_adamw"))
        roles.append("muon")
    sid = {id(p) for p in structural}
    if len(sid) != len(structural):
        raise RuntimeError("structural parameter ownership overlaps")
    decay, no_decay = [], []
    for name, p in named:
        if id(p) not in sid:
            (no_decay if p.ndim < 2 or ".rlb_activation." in name or name == "embed_tokens.weight" else decay).append(p)
    groups = ([dict(params=decay, weight_decay=0.1)] if decay else []) + (
        [dict(params=no_decay, weight_decay=0.0)] if no_decay else [])
    children.append(FusedAdamW(groups, lr=lr, betas=(0.9, 0.95), eps=1e-8))
    roles.append("adamw")
    owner = {}
    for role, child in zip(roles, children):
        for g in child.param_groups:
            g["lr"] = lr
            for p in g["params"]:
                bundle = next((b for b in bundles if b.logical is p), None)
                for real in (bundle.parameters if bundle else (p,)):
                    if id(real) in owner:
                        raise RuntimeError("optimizer parameter ownership overlaps")
                    owner[id(real)] = (role, g["weight_decay"])
    if set(owner) != {id(p) for _, p in named}:
        raise RuntimeError("optimizer parameter coverage is incomplete")
    inventory = [dict(name=n, shape=list(p.shape), role=owner[id(p)][0], weight_decay=owner[id(p)][1])
                 for n, p in named]
    return CampaignOptimizer(model, condition, accumulation, children, roles, inventory, router, attention, bundles)


class TillerThenMuon:
    """TILLER for ``SWITCH_UPDATE`` updates, then native Muon on the same GRAIN model."""

    schema = "portable_mha_tiller100_muon_v1"

    def __init__(self, model, lr, accumulation, *, condition=MHA_SWITCH):
        if condition not in SWITCH_CONDITIONS:
            raise ValueError("unsupported switch identity")
        self._condition, self.model, self.lr, self.accumulation = condition, model, lr, accumulation
        self.phase, self.handoff = "tiller", None
        self.inner = build_optimizer(model, MHA_TILLER, lr, accumulation)

    @property
    def condition(self):
        return self._condition

    def __getattr__(self, name):
        if name == "inner":
            raise AttributeError(name)
        return getattr(self.inner, name)

    @property
    def param_groups(self):
        return self.inner.param_groups

    def _remove_hooks(self):
        if self.inner.router is not None:
            self.inner.router.remove_hooks()

    @torch.no_grad()
    def _to_muon(self, *, transfer):
        old = self.inner
        if transfer and (old.completed_steps != C.SWITCH_UPDATE or old._clipping_recorded):
            raise RuntimeError("the switch requires the exact completed-update-100 boundary")
        named = [(n, p) for n, p in self.model.named_parameters() if p.requires_grad]
        structural = [(n, p) for n, p in named
                      if p.ndim == 2 and n != "embed_tokens.weight" and ".rlb_activation." not in n]
        muon = Muon([p for _, p in structural], lr=self.lr, weight_decay=0.1, momentum=0.95, ns_steps=5,
                    adjust_lr_fn="match_rms_adamw")
        if transfer:
            buffers = {}
            for child in (old.router, old.attention):
                for g in child.param_groups:
                    for p in g["params"]:
                        buf = child.state[p]["momentum_buffer"]
                        if buf.shape != p.shape or not torch.isfinite(buf).all():
                            raise RuntimeError("invalid handoff momentum")
                        bundle = next((b for b in old.bundles if b.logical is p), None)
                        owners = bundle.parameters if bundle else (p,)
                        parts = buf.split(bundle.layout.widths, dim=0) if bundle else (buf,)
                        for o, value in zip(owners, parts):
                            if id(o) in buffers:
                                raise RuntimeError("duplicate handoff owner")
                            buffers[id(o)] = value
            if set(buffers) != {id(p) for _, p in structural}:
                raise RuntimeError("incomplete handoff momentum coverage")
            for _, p in structural:
                muon.state[p]["momentum_buffer"] = buffers[id(p)].clone()
        aux = old.children[-1]
        if old.roles[-1] != "adamw":
            raise RuntimeError("unexpected auxiliary child")
        ids = {id(p) for _, p in structural}
        aux_ids = {id(p) for g in aux.param_groups for p in g["params"]}
        if ids & aux_ids or ids | aux_ids != {id(p) for _, p in named}:
            raise RuntimeError("switch ownership mismatch")
        self._remove_hooks()
        inventory = [dict(name=n, shape=list(p.shape), role="muon" if id(p) in ids else "adamw",
                          weight_decay=0.1 if id(p) in ids else 0.0) for n, p in named]
        self.inner = CampaignOptimizer(self.model, self.condition, self.accumulation, (muon, aux),
                                       ("muon", "adamw"), inventory)
        self.inner.completed_steps = old.completed_steps
        self.inner.last_clipping = old.last_clipping
        self.phase = "muon"
        if transfer:
            self.handoff = dict(completed_update=C.SWITCH_UPDATE, next_update=C.SWITCH_UPDATE + 1,
                                structural_matrices=len(structural), auxiliary_preserved=True,
                                momentum_transferred=True, tiller_hooks_removed=True, policy=POLICY)

    def zero_grad(self, set_to_none=True):
        if self.phase == "tiller" and self.completed_steps == C.SWITCH_UPDATE:
            self._to_muon(transfer=True)
        self.inner.zero_grad(set_to_none=set_to_none)

    def step(self):
        if self.phase == "tiller" and self.completed_steps >= C.SWITCH_UPDATE:
            raise RuntimeError("the switch must occur before the forward pass of update 101")
        self.inner.step()

    def state_dict(self):
        return dict(schema=self.schema, condition=self.condition, policy=POLICY, phase=self.phase,
                    handoff=self.handoff, completed_steps=self.completed_steps, inner=self.inner.state_dict())

    def load_state_dict(self, state):
        if (state.get("schema") != self.schema or state.get("condition") != self.condition
                or state.get("policy") != POLICY):
            raise ValueError("switch checkpoint identity mismatch")
        phase, step = state.get("phase"), state["inner"]["completed_steps"]
        if state.get("completed_steps") != step:
            raise ValueError("switch/child counter mismatch")
        if (type(step) is not int or phase not in ("tiller", "muon")
                or (phase == "tiller" and not 1 <= step <= C.SWITCH_UPDATE)
                or (phase == "muon" and step < C.SWITCH_UPDATE)):
            raise ValueError("invalid switch checkpoint phase/counter")
        handoff = state.get("handoff")
        if phase == "tiller" and handoff is not None:
            raise ValueError("premature handoff receipt")
        if phase == "muon" and (not isinstance(handoff, dict) or handoff.get("policy") != POLICY
                                or handoff.get("completed_update") != C.SWITCH_UPDATE
                                or handoff.get("next_update") != C.SWITCH_UPDATE + 1
                                or handoff.get("momentum_transferred") is not True
                                or handoff.get("auxiliary_preserved") is not True
                                or handoff.get("tiller_hooks_removed") is not True):
            raise ValueError("missing verified handoff receipt")
        if self.phase != phase:
            if phase == "muon":
                self._to_muon(transfer=False)
            else:
                self._remove_hooks()
                self.inner = build_optimizer(self.model, MHA_TILLER, self.lr, self.accumulation)
                self.phase = "tiller"
        self.inner.load_state_dict(state["inner"])
        self.handoff = copy.deepcopy(handoff)
