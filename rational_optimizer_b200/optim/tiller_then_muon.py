"""TILLER for the first 1,000 updates, then ordinary Muon (reference:
optimizer_design/tiller_then_muon.py:59-328).

At the switch the LR/weight decay of the router are copied to the Muon child,
each structural matrix's ``momentum_buffer`` is cloned from TILLER into
Muon's state, TILLER's capture hooks and probe storage are removed, and the
active children become ``[muon, adamw]`` (the AdamW child is kept).  The
checkpoint schema is ``tiller_then_muon_composite_v1`` with children
``tiller_router``, ``tiller_attention``, ``ordinary_muon`` and ``adamw``; the
stage is re-derived from ``completed_steps`` on load.
"""
from __future__ import annotations

import torch

from .adamw import FusedAdamW
from .muon import Muon
from .tiller import TILLERAttentionOptimizer, TILLERRouter, configure_microbatch_count

OPTIMIZER_ID = "tiller_then_muon_v1"
FAMILY_ID = OPTIMIZER_ID
PREFIX = "tiller_then_muon_"
SWITCH_AFTER_STEP = 1000


def _sorted_blocks(blocks):
    ordered = sorted((dict(b) for b in blocks), key=lambda b: int(b["layer_index"]))
    if [int(b["layer_index"]) for b in ordered] != list(range(len(ordered))):
        raise ValueError("TILLER-then-Muon layer inventory must be contiguous")
    return ordered


def _muon_named_parameters(blocks):
    named, seen = [], set()
    for b in blocks:
        i = int(b["layer_index"])
        for name, p in ((f"layers.{i}.attn.qkv.weight", b["qkv_weight"]),
                        (f"layers.{i}.attn.out.weight", b["attn_out_weight"]),
                        (f"layers.{i}.mlp.in_proj.weight", b["in_weight"]),
                        (f"layers.{i}.mlp.out_proj.weight", b["out_weight"])):
            if p.ndim != 2:
                raise ValueError(f"{name} is not a Muon matrix parameter")
            if id(p) in seen:
                raise ValueError("TILLER-then-Muon structural parameter ownership overlaps")
            seen.add(id(p))
            named.append((name, p))
    return named


def _groups(optimizers):
    out = []
    for opt in optimizers:
        out.extend(opt.param_groups)
    return out


class TillerThenMuonOptimizer:
    _SCHEMA = "tiller_then_muon_composite_v1"

    def __init__(self, blocks, *, adam_groups, lr, weight_decay, momentum, ns_steps, beta1, beta2,
                 eps, adjust_lr_fn, switch_after_step: int = SWITCH_AFTER_STEP):
        self.blocks = _sorted_blocks(blocks)
        if not self.blocks:
            raise ValueError("TILLER-then-Muon requires GRAIN blocks")
        self._switch = int(switch_after_step)
        self.tiller_router = TILLERRouter(self.blocks, lr=lr, weight_decay=weight_decay,
                                          momentum=momentum, ns_steps=ns_steps, beta2=beta2, eps=eps)
        self.tiller_attention = TILLERAttentionOptimizer(
            self.blocks, self.tiller_router, lr=lr, weight_decay=weight_decay, momentum=momentum,
            ns_steps=ns_steps, beta2=beta2, eps=eps, adjust_lr_fn=adjust_lr_fn)
        self._ordinary_muon = Muon(_muon_named_parameters(self.blocks), lr=lr,
                                   weight_decay=weight_decay, momentum=momentum, ns_steps=ns_steps,
                                   adjust_lr_fn=adjust_lr_fn)
        if not adam_groups:
            raise ValueError("TILLER-then-Muon requires an AdamW child for non-structural parameters")
        self._adamw = FusedAdamW(adam_groups, lr=lr, betas=(beta1, beta2), eps=eps)
        self._momentum_sources = []
        for b in self.blocks:
            self._momentum_sources.extend(((b["in_weight"], self.tiller_router),
                                           (b["out_weight"], self.tiller_router),
                                           (b["qkv_weight"], self.tiller_attention),
                                           (b["attn_out_weight"], self.tiller_attention)))
        self._completed_steps = 0
        self._transitioned = False
        self._capture_telemetry_next_step = False
        self._last_telemetry = {}
        self.optimizers = [self.tiller_router, self.tiller_attention, self._adamw]

    @property
    def param_groups(self):
        """The active children's current groups (rebuilt per access: loading a
        child's state replaces its group dicts)."""
        return _groups(self.optimizers)

    @property
    def completed_steps(self):
        return self._completed_steps

    @property
    def switch_after_step(self):
        return self._switch

    @property
    def stage(self):
        return "muon" if self._transitioned else "tiller"

    @property
    def ordinary_muon(self):
        return self._ordinary_muon

    @property
    def adamw(self):
        return self._adamw

    def lr_wd_fairness_audit(self):
        out = {"formal_candidate_lr_scale": 1.0, "stage1_full_tiller_lr_scale": 1.0,
               "stage2_ordinary_muon_lr_scale": 1.0, "state_preserving_switch_lr_scale": 1.0,
               "shared_schedule_lr_scale": 1.0, "weight_decay_scale": 1.0}
        for prefix, child in (("stage1_router_", self.tiller_router),
                              ("stage1_attention_", self.tiller_attention)):
            for k, v in child.lr_wd_fairness_audit().items():
                out[prefix + k] = v
        return out

    def set_telemetry_capture(self, enabled=True):
        self._capture_telemetry_next_step = bool(enabled)

    def telemetry(self):
        return dict(self._last_telemetry)

    def method_specific_sync_active(self):
        return not self._transitioned

    def zero_grad(self, set_to_none=True):
        for opt in self.optimizers:
            opt.zero_grad(set_to_none=set_to_none)

    def record_realized_clipping(self, preclip_norm, max_norm):
        if self._transitioned:
            return
        if preclip_norm is None:
            raise RuntimeError("TILLER-then-Muon requires the realized gradient norm before the switch")
        self.tiller_router.record_realized_clipping(preclip_norm, max_norm)

    def _transition_to_muon(self):
        if self._transitioned:
            return
        if self._completed_steps != self._switch:
            raise RuntimeError("TILLER-then-Muon transition attempted at the wrong step")
        ref = self.tiller_router.param_groups[0]
        for g in self._ordinary_muon.param_groups:
            g["lr"] = float(ref["lr"])
            g["weight_decay"] = float(ref["weight_decay"])
        missing = []
        for p, src in self._momentum_sources:
            buf = src.state.get(p, {}).get("momentum_buffer")
            if not torch.is_tensor(buf):
                missing.append(tuple(p.shape))
                continue
            self._ordinary_muon.state[p]["momentum_buffer"] = buf.detach().clone(
                memory_format=torch.preserve_format)
        if missing:
            raise RuntimeError(f"TILLER-then-Muon missing compatible momentum buffers: {missing[:4]}")
        self._activate_muon_stage()

    def eager_step_required(self):
        """True when this step's forward/backward must run eagerly (TILLER response-probe refresh)."""
        return not self._transitioned and bool(self.tiller_router._capture_response_this_transition)

    def _activate_muon_stage(self):
        self._transitioned = True
        self.tiller_router.remove_hooks()
        self.optimizers = [self._ordinary_muon, self._adamw]

    @torch.no_grad()
    def step(self):
        self._last_telemetry = {}
        prior = self.stage
        switched = False
        child = {}
        try:
            for opt in list(self.optimizers):
                if opt is self.tiller_router:
                    # ledger kernel beside the attention and AdamW updates
                    opt.step(defer_apply=True)
                else:
                    opt.step()
        finally:
            if prior == "tiller":
                self.tiller_router.finish_step()
        self._completed_steps += 1
        if prior == "tiller" and self._capture_telemetry_next_step:
            for c in (self.tiller_router, self.tiller_attention):
                child.update(c.telemetry())
        if prior == "tiller" and self._completed_steps == self._switch:
            self._transition_to_muon()
            switched = True
        if self._capture_telemetry_next_step:
            self._last_telemetry = {
                PREFIX + "family_id": FAMILY_ID, PREFIX + "formal_candidate": 1,
                PREFIX + "switch_after_step": self._switch,
                PREFIX + "completed_steps": self._completed_steps,
                PREFIX + "stage_before_step": prior, PREFIX + "stage_after_step": self.stage,
                PREFIX + "switched_to_muon": int(switched),
                PREFIX + "state_transition": "preserve_compatible_state",
            }
            if switched:
                self._last_telemetry.update(child)
        self._capture_telemetry_next_step = False

    def state_dict(self):
        return {
            "schema": self._SCHEMA, "optimizer_id": OPTIMIZER_ID,
            "switch_after_step": self._switch, "completed_steps": self._completed_steps,
            "stage": self.stage, "state_transition": "preserve_compatible_state",
            "children": {"tiller_router": self.tiller_router.state_dict(),
                         "tiller_attention": self.tiller_attention.state_dict(),
                         "ordinary_muon": self._ordinary_muon.state_dict(),
                         "adamw": self._adamw.state_dict()},
        }

    def load_state_dict(self, state_dict):
        if (not isinstance(state_dict, dict) or state_dict.get("schema") != self._SCHEMA
                or state_dict.get("optimizer_id") != OPTIMIZER_ID
                or int(state_dict.get("switch_after_step", -1)) != self._switch
                or state_dict.get("state_transition") != "preserve_compatible_state"
                or not isinstance(state_dict.get("children"), dict)):
            raise RuntimeError("TILLER-then-Muon checkpoint schema changed")
        ch = state_dict["children"]
        completed = int(state_dict["completed_steps"])
        if completed < 0:
            raise RuntimeError("TILLER-then-Muon checkpoint step is invalid")
        if completed > 0:
            self.tiller_router.load_state_dict(ch["tiller_router"])
            self.tiller_attention.load_state_dict(ch["tiller_attention"])
        self._ordinary_muon.load_state_dict(ch["ordinary_muon"])
        self._adamw.load_state_dict(ch["adamw"])
        self._completed_steps = completed
        self._transitioned = completed >= self._switch
        if self._transitioned:
            self._activate_muon_stage()
        else:
            self.optimizers = [self.tiller_router, self.tiller_attention, self._adamw]
        self._last_telemetry = {}
        self._capture_telemetry_next_step = False


__all__ = ("FAMILY_ID", "OPTIMIZER_ID", "PREFIX", "SWITCH_AFTER_STEP", "TillerThenMuonOptimizer",
           "configure_microbatch_count")
