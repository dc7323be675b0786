"""Two-stage schedule: TILLER for the first 1,000 updates, ordinary Muon after.

Behaviour matches optimizer_design/tiller_then_muon.py:59-328 (candidate id
``tiller_then_muon_v1``); the structure here is a generic two-stage switch:

* stage ``"tiller"`` is the TILLER composite of this package
  (:class:`~.composite.TILLERCompositeOptimizer`: router with its ledger on a
  side stream, attention optimizer, AdamW);
* stage ``"muon"`` is a plain :class:`~.composite.CompositeOptimizer` of
  ordinary Muon on the four structural matrices of every layer (q/k/v,
  attention output, GRAIN in/out projections) and the *same* AdamW object,
  so the AdamW state simply continues;
* the hand-off, run once after update number ``switch_after_step``, gives
  Muon the router's current LR and weight decay, and seeds each Muon matrix's
  ``momentum_buffer`` with a copy of the buffer that whichever TILLER child
  owns the matrix kept; TILLER's probe hooks and captured records are dropped.

Checkpoint schema ``tiller_then_muon_composite_v1`` (children
``tiller_router``, ``tiller_attention``, ``ordinary_muon``, ``adamw``); the
stage is re-derived from ``completed_steps`` on load.
"""
from __future__ import annotations

import torch

from .adamw import FusedAdamW
from .composite import CompositeOptimizer, TILLERCompositeOptimizer
from .muon import Muon
from .tiller import TILLERAttentionOptimizer, TILLERRouter, configure_microbatch_count

OPTIMIZER_ID = "tiller_then_muon_v1"
FAMILY_ID = OPTIMIZER_ID
PREFIX = "tiller_then_muon_"
SWITCH_AFTER_STEP = 1000
SCHEMA = "tiller_then_muon_composite_v1"
TRANSITION = "preserve_compatible_state"

# (parameter-name suffix, block key) of the matrices ordinary Muon takes over
_STRUCTURAL = (("attn.qkv.weight", "qkv_weight"), ("attn.out.weight", "attn_out_weight"),
               ("mlp.in_proj.weight", "in_weight"), ("mlp.out_proj.weight", "out_weight"))


def _layer_ordered(blocks):
    by_layer = {}
    for b in blocks:
        by_layer.setdefault(int(b["layer_index"]), []).append(dict(b))
    if sorted(by_layer) != list(range(len(by_layer))) or any(len(v) != 1 for v in by_layer.values()):
        raise ValueError(f"two-stage optimizer needs exactly one block per layer 0..L-1, got "
                         f"layers {sorted(by_layer)}")
    return [by_layer[i][0] for i in range(len(by_layer))]


def _structural_matrices(blocks):
    """[(name, parameter)] for Muon, in layer order; rejects shared or non-matrix entries."""
    out = {}
    for b in blocks:
        for suffix, key in _STRUCTURAL:
            name, p = f"layers.{int(b['layer_index'])}.{suffix}", b[key]
            if p.ndim != 2:
                raise ValueError(f"ordinary Muon needs 2-D matrices; {name} has shape {tuple(p.shape)}")
            if id(p) in out:
                raise ValueError(f"{name} is the same tensor as {out[id(p)][0]}")
            out[id(p)] = (name, p)
    return list(out.values())


class TillerThenMuonOptimizer:
    """TILLER until ``switch_after_step`` updates are done, then Muon + the same AdamW."""

    _SCHEMA = SCHEMA

    def __init__(self, blocks, *, adam_groups, lr, weight_decay, momentum, ns_steps, beta1, beta2,
                 eps, adjust_lr_fn, switch_after_step: int = SWITCH_AFTER_STEP):
        self.blocks = _layer_ordered(blocks)
        if not self.blocks:
            raise ValueError("two-stage optimizer built without GRAIN layers")
        if not adam_groups:
            raise ValueError("two-stage optimizer needs AdamW groups for the non-matrix parameters")
        self._switch = int(switch_after_step)
        shared = dict(weight_decay=weight_decay, momentum=momentum, ns_steps=ns_steps)
        router = TILLERRouter(self.blocks, lr=lr, beta2=beta2, eps=eps, **shared)
        attention = TILLERAttentionOptimizer(self.blocks, router, lr=lr, beta2=beta2, eps=eps,
                                             adjust_lr_fn=adjust_lr_fn, **shared)
        adamw = FusedAdamW(adam_groups, lr=lr, betas=(beta1, beta2), eps=eps)
        muon = Muon(_structural_matrices(self.blocks), lr=lr, adjust_lr_fn=adjust_lr_fn, **shared)
        self._stages = {"tiller": TILLERCompositeOptimizer((router, attention, adamw)),
                        "muon": CompositeOptimizer((muon, adamw))}
        self._completed_steps = 0
        self._stage = "tiller"
        self._capture_telemetry_next_step = False
        self._last_telemetry = {}

    # -- children ------------------------------------------------------------
    @property
    def tiller_router(self):
        return self._stages["tiller"].optimizers[0]

    @property
    def tiller_attention(self):
        return self._stages["tiller"].optimizers[1]

    @property
    def ordinary_muon(self):
        return self._stages["muon"].optimizers[0]

    @property
    def adamw(self):
        return self._stages["muon"].optimizers[1]

    @property
    def optimizers(self):
        """The children stepped in the current stage."""
        return self._stages[self._stage].optimizers

    @property
    def param_groups(self):
        """Groups of the current stage's children, rebuilt on each access (a child's
        ``load_state_dict`` replaces its group dicts)."""
        return self._stages[self._stage].param_groups

    @property
    def completed_steps(self):
        return self._completed_steps

    @property
    def switch_after_step(self):
        return self._switch

    @property
    def stage(self):
        return self._stage

    # -- trainer contract ------------------------------------------------------
    def lr_wd_fairness_audit(self):
        audit = dict.fromkeys(("formal_candidate_lr_scale", "stage1_full_tiller_lr_scale",
                               "stage2_ordinary_muon_lr_scale", "state_preserving_switch_lr_scale",
                               "shared_schedule_lr_scale", "weight_decay_scale"), 1.0)
        for prefix, child in (("stage1_router_", self.tiller_router),
                              ("stage1_attention_", self.tiller_attention)):
            audit.update({prefix + k: v for k, v in child.lr_wd_fairness_audit().items()})
        return audit

    def set_telemetry_capture(self, enabled=True):
        self._capture_telemetry_next_step = bool(enabled)

    def telemetry(self):
        return dict(self._last_telemetry)

    def method_specific_sync_active(self):
        return self._stage == "tiller"

    def eager_step_required(self):
        """True when this step's forward/backward must run eagerly (TILLER response-probe refresh)."""
        return self._stage == "tiller" and self._stages["tiller"].eager_step_required()

    def probe_recorder(self):
        """The TILLER router while it records probes, else None (Muon stage)."""
        return self.tiller_router if self._stage == "tiller" else None

    def zero_grad(self, set_to_none=True):
        self._stages[self._stage].zero_grad(set_to_none=set_to_none)

    def record_realized_clipping(self, preclip_norm, max_norm):
        if self._stage != "tiller":
            return  # Muon does not observe clipping
        if preclip_norm is None:
            raise RuntimeError("the TILLER stage needs the pre-clip gradient norm of every step")
        self.tiller_router.record_realized_clipping(preclip_norm, max_norm)

    # -- switch ----------------------------------------------------------------
    def _hand_off(self):
        """Carry LR, weight decay and momentum from the TILLER children into Muon."""
        if self._completed_steps != self._switch:
            raise RuntimeError(f"stage switch at update {self._completed_steps}, expected "
                               f"{self._switch}")
        router_group = self.tiller_router.param_groups[0]
        muon = self.ordinary_muon
        for group in muon.param_groups:
            group["lr"] = float(router_group["lr"])
            group["weight_decay"] = float(router_group["weight_decay"])
        holders = (self.tiller_router.state, self.tiller_attention.state)
        absent = []
        for group in muon.param_groups:
            for p in group["params"]:
                buf = next((st[p]["momentum_buffer"] for st in holders
                            if p in st and torch.is_tensor(st[p].get("momentum_buffer"))), None)
                if buf is None:
                    absent.append(tuple(p.shape))
                else:
                    muon.state[p]["momentum_buffer"] = buf.detach().clone(
                        memory_format=torch.preserve_format)
        if absent:
            raise RuntimeError(f"no TILLER momentum to hand to Muon for {len(absent)} matrices "
                               f"(first shapes {absent[:4]})")
        self._enter_muon_stage()

    def _enter_muon_stage(self):
        self._stage = "muon"
        self.tiller_router.remove_hooks()

    @torch.no_grad()
    def step(self):
        before = self._stage
        self._stages[before].step()
        self._completed_steps += 1
        record = self._capture_telemetry_next_step
        children = {}
        if record and before == "tiller":
            for child in (self.tiller_router, self.tiller_attention):
                children.update(child.telemetry())
        switched = before == "tiller" and self._completed_steps == self._switch
        if switched:
            self._hand_off()
        self._last_telemetry = {}
        if record:
            self._last_telemetry = {PREFIX + k: v for k, v in (
                ("family_id", FAMILY_ID), ("formal_candidate", 1),
                ("switch_after_step", self._switch), ("completed_steps", self._completed_steps),
                ("stage_before_step", before), ("stage_after_step", self._stage),
                ("switched_to_muon", int(switched)), ("state_transition", TRANSITION))}
            if switched:
                self._last_telemetry.update(children)
        self._capture_telemetry_next_step = False

    # -- checkpoints -----------------------------------------------------------
    def state_dict(self):
        return {"schema": SCHEMA, "optimizer_id": OPTIMIZER_ID, "switch_after_step": self._switch,
                "completed_steps": self._completed_steps, "stage": self._stage,
                "state_transition": TRANSITION,
                "children": {"tiller_router": self.tiller_router.state_dict(),
                             "tiller_attention": self.tiller_attention.state_dict(),
                             "ordinary_muon": self.ordinary_muon.state_dict(),
                             "adamw": self.adamw.state_dict()}}

    def load_state_dict(self, state_dict):
        expected = {"schema": SCHEMA, "optimizer_id": OPTIMIZER_ID, "state_transition": TRANSITION}
        if not isinstance(state_dict, dict) or not isinstance(state_dict.get("children"), dict):
            raise RuntimeError(f"not a {SCHEMA} state dict")
        wrong = {k: state_dict.get(k) for k, v in expected.items() if state_dict.get(k) != v}
        if int(state_dict.get("switch_after_step", -1)) != self._switch:
            wrong["switch_after_step"] = state_dict.get("switch_after_step")
        if wrong:
            raise RuntimeError(f"{SCHEMA} checkpoint does not match this optimizer: {wrong}")
        completed = int(state_dict["completed_steps"])
        if completed < 0:
            raise RuntimeError(f"negative completed_steps {completed} in checkpoint")
        children = state_dict["children"]
        if completed > 0:  # a step-0 checkpoint carries no TILLER state yet
            self.tiller_router.load_state_dict(children["tiller_router"])
            self.tiller_attention.load_state_dict(children["tiller_attention"])
        self.ordinary_muon.load_state_dict(children["ordinary_muon"])
        self.adamw.load_state_dict(children["adamw"])
        self._completed_steps = completed
        self._stage = "tiller"
        if completed >= self._switch:
            self._enter_muon_stage()
        self._last_telemetry = {}
        self._capture_telemetry_next_step = False


__all__ = ("FAMILY_ID", "OPTIMIZER_ID", "PREFIX", "SWITCH_AFTER_STEP", "TillerThenMuonOptimizer",
           "configure_microbatch_count")
