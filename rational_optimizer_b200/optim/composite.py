"""Optimizer assembly for the trainer (reference training/train.py:1346-1885 and
experiments/protocol/method_entrypoint.py:24-171).

* ``collect_rlb_optimizer_groups`` / ``collect_blocks``: the per-layer GRAIN
  and attention matrix inventory TILLER consumes;
* ``CompositeOptimizer`` (list state dict) and ``TILLERCompositeOptimizer``
  (``tiller_composite_v1`` schema, roles router/attention/adamw);
* ``configure_optimizer(model, args)``: AdamW, Muon(+AdamW), Lion, AdEMAMix,
  Schedule-Free AdamW, CAME-style, SOAP-style, TILLER (``tiller_v1``) and
  ``tiller_then_muon_v1``.
"""
from __future__ import annotations

import os
import re

import torch
import torch.nn as nn

from .adamw import FusedAdamW
from .tiller import FAMILY_ID as TILLER_ID
from .tiller import TILLERAttentionOptimizer, TILLERRouter, configure_microbatch_count

TILLER_THEN_MUON_OPTIMIZER = "tiller_then_muon_v1"
BASELINE_OPTIMIZERS = {"adamw", "muon", "lion", "ademamix", "schedule_free_adamw",
                       "adafactor_came", "soap_adamw"}
RATIONAL_SPECIFIC_OPTIMIZERS = {TILLER_THEN_MUON_OPTIMIZER, TILLER_ID}
ACTIVE_OPTIMIZERS = sorted(BASELINE_OPTIMIZERS | RATIONAL_SPECIFIC_OPTIMIZERS)


def unwrap_model(model):
    return model.module if hasattr(model, "module") and isinstance(model.module, nn.Module) else model


def is_no_decay_parameter(name, param):
    return param.dim() < 2 or ".rlb_activation." in name


def is_tied_embedding_parameter_name(name):
    return name.removeprefix("module.") in {"token_embedding.weight", "lm_head.weight"}


def split_decay_parameters(model):
    decay, no_decay = [], []
    for name, param in model.named_parameters():
        if not param.requires_grad:
            continue
        (no_decay if is_no_decay_parameter(name, param) else decay).append(param)
    return decay, no_decay


def rational_optimizer_layer_index(name):
    match = re.search(r"(?:^|\.)layers\.(\d+)\.", name)
    return int(match.group(1)) if match else -1


def collect_rlb_optimizer_groups(model, args=None):
    """Per-layer GRAIN inventory (mlp, activation, in/out matrices, coefficients)."""
    groups = []
    num_layers = getattr(args, "layers", None)
    for module_name, module in model.named_modules():
        act = getattr(module, "rlb_activation", None)
        inp = getattr(module, "in_proj", None)
        out = getattr(module, "out_proj", None)
        if act is None or inp is None or out is None:
            continue
        if not isinstance(inp, nn.Linear) or not isinstance(out, nn.Linear):
            continue
        if not all(hasattr(act, a) for a in ("groups", "hidden_dim", "numerator", "denominator")):
            continue
        hidden = int(act.hidden_dim)
        if inp.weight.shape[0] != hidden or out.weight.shape[1] != hidden:
            continue
        groups.append({
            "mlp": module, "module": act, "in_weight": inp.weight, "out_weight": out.weight,
            "numerator": act.numerator, "denominator": act.denominator, "coeff_logits": None,
            "centers": getattr(act, "centers", None), "beta": getattr(act, "beta", None),
            "coeff_limit": float(getattr(act, "coeff_limit", 0.0)), "groups": int(act.groups),
            "hidden_dim": hidden, "eps": float(getattr(act, "eps", 0.0)),
            "layer_index": rational_optimizer_layer_index(module_name + "."),
            "num_layers": num_layers,
        })
    return groups


def collect_blocks(model, args=None):
    """GRAIN pairs extended with the layer's attention matrices."""
    raw = unwrap_model(model)
    by_layer = {int(g["layer_index"]): dict(g) for g in collect_rlb_optimizer_groups(model, args)}
    if len(by_layer) != len(raw.layers):
        raise RuntimeError("TILLER requires one rational block per Transformer layer")
    blocks = []
    for index, block in enumerate(raw.layers):
        g = by_layer.get(index)
        if g is None or g["mlp"] is not block.mlp:
            raise RuntimeError("rational block inventory does not match model depth")
        g.update({"block": block, "qkv_weight": block.attn.qkv.weight,
                  "attn_out_weight": block.attn.out.weight})
        blocks.append(g)
    return blocks


def partition_parameters(model, blocks, *, decay_tied_embedding=False):
    structural = {id(p) for b in blocks for p in (b["in_weight"], b["out_weight"], b["qkv_weight"],
                                                  b["attn_out_weight"])}
    if len(structural) != 4 * len(blocks):
        raise RuntimeError("TILLER structural parameter ownership overlaps")
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad or id(p) in structural:
            continue
        tied = is_tied_embedding_parameter_name(name)
        if is_no_decay_parameter(name, p) or (tied and not decay_tied_embedding):
            no_decay.append(p)
        else:
            decay.append(p)
    return structural, decay, no_decay


class CompositeOptimizer:
    """Steps several optimizers in order; state dict is their list."""

    def __init__(self, optimizers):
        self.optimizers = list(optimizers)

    @property
    def param_groups(self):
        """The children's current groups.  Built on every access because a
        child's ``load_state_dict`` replaces its group dicts; a list cached at
        construction would keep receiving scheduled LRs the children no longer
        read (the reference's composite caches it, so its resumed composite
        runs step at the checkpointed LR)."""
        return [g for opt in self.optimizers for g in opt.param_groups]

    def zero_grad(self, set_to_none=True):
        for opt in self.optimizers:
            opt.zero_grad(set_to_none=set_to_none)

    def step(self):
        for opt in self.optimizers:
            opt.step()

    def eager_step_required(self):
        """No step records forward/backward probes, so every step's
        forward/backward may replay a captured graph."""
        return False

    def state_dict(self):
        return [opt.state_dict() for opt in self.optimizers]

    def load_state_dict(self, state_dict):
        for opt, st in zip(self.optimizers, state_dict):
            opt.load_state_dict(st)


class TILLERCompositeOptimizer(CompositeOptimizer):
    _ROLES = ("tiller_router", "tiller_attention", "adamw")
    _SCHEMA = "tiller_composite_v1"

    def __init__(self, optimizers):
        super().__init__(optimizers)
        if len(self.optimizers) != len(self._ROLES):
            raise RuntimeError("TILLER composite requires three optimizer children")

    @property
    def router(self):
        return self.optimizers[0]

    def step(self):
        """Router, attention, AdamW.  The router's single-CTA ledger kernel runs
        on a side stream beside the attention and AdamW updates (they touch
        disjoint parameters); the router's weight update is applied after."""
        router = self.router
        router.step(defer_apply=True)
        try:
            for opt in self.optimizers[1:]:
                opt.step()
        finally:
            router.finish_step()

    def eager_step_required(self):
        """True when this step's forward/backward records response probes (refresh step)."""
        return bool(self.router._capture_response_this_transition)

    def probe_recorder(self):
        """The child whose forward/backward hooks record probes (see ``train.graphs``)."""
        return self.router

    def record_realized_clipping(self, preclip_norm, max_norm):
        self.optimizers[0].record_realized_clipping(preclip_norm, max_norm)

    def set_telemetry_capture(self, enabled=True):
        for opt in self.optimizers[:2]:
            opt.set_telemetry_capture(enabled)

    def telemetry(self):
        out = {}
        for opt in self.optimizers[:2]:
            out.update(opt.telemetry())
        return out

    def state_dict(self):
        return {"schema": self._SCHEMA, "roles": self._ROLES,
                "children": [opt.state_dict() for opt in self.optimizers]}

    def load_state_dict(self, state_dict):
        if (not isinstance(state_dict, dict) or state_dict.get("schema") != self._SCHEMA
                or tuple(state_dict.get("roles", ())) != self._ROLES
                or len(state_dict.get("children", ())) != len(self.optimizers)):
            raise RuntimeError("TILLER composite checkpoint schema changed")
        for opt, st in zip(self.optimizers, state_dict["children"]):
            opt.load_state_dict(st)


def owner_layers(optimizer):
    """(per-layer matrices, layer -> owner rank) when ``optimizer`` updates each
    layer's structural matrices on one rank only (the layer-sharded TILLER
    composite, or a Muon composite whose Muon is layer-sharded), else
    (None, None).  This is what the reduce-to-owner gradient
    transport needs (``parallel.grad_sync``)."""
    if not isinstance(optimizer, TILLERCompositeOptimizer):
        shard = getattr(optimizer.optimizers[0], "shard", None) if isinstance(optimizer, CompositeOptimizer) \
            and optimizer.optimizers else None
        if shard is None:
            return None, None
        return shard.per_layer, shard.owner
    router, attention = optimizer.optimizers[0], optimizer.optimizers[1]
    if not router._shard()[2]:
        return None, None
    from .tiller import layer_owner
    L, world = len(router.pairs), router.world_size
    layers = [[router.pairs[l]["in_weight"], router.pairs[l]["out_weight"],
               attention.role_parameters["qkv"][l], attention.role_parameters["attn_out"][l]]
              for l in range(L)]
    return layers, (lambda layer: layer_owner(layer, L, world))


def _adam_groups(decay, no_decay, weight_decay):
    groups = []
    if decay:
        groups.append({"params": decay, "weight_decay": weight_decay})
    if no_decay:
        groups.append({"params": no_decay, "weight_decay": 0.0})
    return groups


def build_tiller(model, args, *, decay_tied_embedding=False, microbatches=None,
                 loss_probe_group=None):
    """Router + attention + AdamW for the ``tiller_v1`` optimizer id."""
    if microbatches is not None:
        configure_microbatch_count(int(microbatches))
    blocks = collect_blocks(model, args)
    structural, decay, no_decay = partition_parameters(model, blocks,
                                                       decay_tied_embedding=decay_tied_embedding)
    covered = structural | {id(p) for p in decay + no_decay}
    if covered != {id(p) for p in model.parameters() if p.requires_grad}:
        raise RuntimeError("TILLER parameter partition is incomplete")
    router = TILLERRouter(blocks, lr=args.lr, weight_decay=args.weight_decay,
                          momentum=args.muon_momentum, ns_steps=args.muon_ns_steps,
                          beta2=args.beta2, eps=args.eps, loss_probe_group=loss_probe_group)
    attention = TILLERAttentionOptimizer(blocks, router, lr=args.lr, weight_decay=args.weight_decay,
                                         momentum=args.muon_momentum, ns_steps=args.muon_ns_steps,
                                         beta2=args.beta2, eps=args.eps,
                                         adjust_lr_fn=args.muon_adjust_lr_fn)
    groups = _adam_groups(decay, no_decay, args.weight_decay)
    if not groups:
        raise RuntimeError("TILLER found no parameters for its AdamW child")
    adamw = FusedAdamW(groups, lr=args.lr, betas=(args.beta1, args.beta2), eps=args.eps)
    if router._shard()[2] and os.environ.get("RO_TILLER_PACK", "1") != "0":
        # layer-sharded across ranks: one contiguous buffer per owner so the
        # updated weights travel in one broadcast per owner
        from .tiller import OwnerPacking
        router.packing = OwnerPacking.for_tiller(router, attention)
    return TILLERCompositeOptimizer((router, attention, adamw))


def configure_optimizer(model, args):
    """Build the optimizer named by ``args.optimizer`` (reference train.py:1726-1887)."""
    name = args.optimizer
    if name not in ACTIVE_OPTIMIZERS:
        raise ValueError(f"Accepted optimizer choices: {', '.join(ACTIVE_OPTIMIZERS)}")
    decay, no_decay = split_decay_parameters(model)
    groups = [{"params": decay, "weight_decay": args.weight_decay},
              {"params": no_decay, "weight_decay": 0.0}]
    if name == "adamw":
        return FusedAdamW(groups, lr=args.lr, betas=(args.beta1, args.beta2), eps=args.eps)
    if name in {"lion", "ademamix", "schedule_free_adamw", "adafactor_came", "soap_adamw"}:
        from . import baselines
        return baselines.build(name, groups, args)
    if name == "muon":
        from .muon import Muon
        muon_named, adam_decay, adam_no_decay = [], [], []
        for pname, p in model.named_parameters():
            if not p.requires_grad:
                continue
            nd = is_no_decay_parameter(pname, p)
            tied = is_tied_embedding_parameter_name(pname)
            if p.dim() == 2 and not nd and not tied:
                muon_named.append((pname, p))
            elif nd or tied:
                adam_no_decay.append(p)
            else:
                adam_decay.append(p)
        opts = []
        if muon_named:
            from .muon import shard_muon
            muon = Muon(muon_named, lr=args.lr, weight_decay=args.weight_decay,
                        momentum=args.muon_momentum, ns_steps=args.muon_ns_steps,
                        adjust_lr_fn=args.muon_adjust_lr_fn)
            shard_muon(muon)
            opts.append(muon)
        ag = _adam_groups(adam_decay, adam_no_decay, args.weight_decay)
        if ag:
            opts.append(FusedAdamW(ag, lr=args.lr, betas=(args.beta1, args.beta2), eps=args.eps))
        return CompositeOptimizer(opts)
    if name == TILLER_ID:
        return build_tiller(model, args, microbatches=int(args.grad_accum),
                            decay_tied_embedding=bool(getattr(args, "decay_tied_embedding", False)))
    if name == TILLER_THEN_MUON_OPTIMIZER:
        from .tiller_then_muon import TillerThenMuonOptimizer
        configure_microbatch_count(int(args.grad_accum))
        blocks = collect_blocks(model, args)
        structural, decay, no_decay = partition_parameters(model, blocks, decay_tied_embedding=False)
        return TillerThenMuonOptimizer(blocks, adam_groups=_adam_groups(decay, no_decay, args.weight_decay),
                                       lr=args.lr, weight_decay=args.weight_decay,
                                       momentum=args.muon_momentum, ns_steps=args.muon_ns_steps,
                                       beta1=args.beta1, beta2=args.beta2, eps=args.eps,
                                       adjust_lr_fn=args.muon_adjust_lr_fn)
    raise ValueError(f"Accepted optimizer choices: {', '.join(ACTIVE_OPTIMIZERS)}")
