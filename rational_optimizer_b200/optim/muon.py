"""Muon with batched Newton-Schulz (reference baseline: ``torch.optim.Muon``,
training/train.py:1808-1850).

Same constructor, defaults, parameter-group keys and ``momentum_buffer``
state as ``torch.optim.Muon``; the step groups parameters of equal shape and
runs one batched NS5 per shape
(:func:`~rational_optimizer_b200.optim.newton_schulz.batched_zero_power`)
instead of one small NS5 per matrix.

Layer-sharded across data-parallel ranks (:func:`shard_muon`, on by default
at world size > 1): the reference replicates Muon on every rank; here rank r
updates only the matrices of its contiguous block of layers (the same
ownership as the layer-sharded TILLER), receives only those layers' reduced
gradients (reduce-to-owner transport) and publishes the updated weights,
which the other ranks pull over peer memory before their next forward
(:class:`~rational_optimizer_b200.optim.tiller.OwnerPacking`).  Momentum
buffers live on the owner only; ``state_dict`` first replicates them, so a
checkpoint is the replicated optimizer's.
"""
from __future__ import annotations

import os
import re

import torch
import torch.distributed as dist

from .newton_schulz import batched_zero_power


def adjust_lr(lr, adjust_lr_fn, shape):
    a, b = shape[:2]
    if adjust_lr_fn is None or adjust_lr_fn == "original":
        return lr * max(1.0, a / b) ** 0.5
    if adjust_lr_fn == "match_rms_adamw":
        return lr * 0.2 * max(a, b) ** 0.5
    return lr


class Muon(torch.optim.Muon):
    shard = None  # MuonShard when layer-sharded across ranks

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        owned = self.shard.owned if self.shard is not None else None
        for group in self.param_groups:
            lr = float(group["lr"])
            wd = float(group["weight_decay"])
            mu = float(group["momentum"])
            by_shape = {}
            for p in group["params"]:
                if p.grad is None or (owned is not None and id(p) not in owned):
                    continue
                if p.grad.ndim != 2:
                    raise ValueError("Param gradient must be a 2D matrix")
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p.grad, memory_format=torch.preserve_format)
                by_shape.setdefault(tuple(p.shape), []).append(p)
            for shape, ps in by_shape.items():
                grads = [p.grad for p in ps]
                bufs = [self.state[p]["momentum_buffer"] for p in ps]
                torch._foreach_lerp_(bufs, grads, 1.0 - mu)
                upd = torch._foreach_lerp(grads, bufs, mu) if group["nesterov"] else bufs
                polar = batched_zero_power(torch.stack(upd), int(group["ns_steps"]))
                alr = adjust_lr(lr, group["adjust_lr_fn"], shape)
                torch._foreach_mul_(ps, 1.0 - lr * wd)
                torch._foreach_add_(ps, list(polar.to(ps[0].dtype).unbind(0)), alpha=-alr)
        if self.shard is not None:
            self.shard.packing.broadcast()
        return loss

    def state_dict(self):
        if self.shard is not None:
            self.shard.replicate_state(self)
        return super().state_dict()


_LAYER = re.compile(r"(?:^|\.)layers\.(\d+)\.")


class MuonShard:
    """Which rank updates which layers' matrices, and the packed weight buffer
    that replicates them."""

    def __init__(self, per_layer, world, rank, group=None):
        from .tiller import OwnerPacking, shard_bounds
        self.per_layer = per_layer
        self.world, self.rank, self.group = int(world), int(rank), group
        lo, hi = shard_bounds(len(per_layer), self.rank, self.world)
        self.owned = {id(p) for l in range(lo, hi) for p in per_layer[l]}
        self.packing = OwnerPacking(per_layer, self.world, group)

    def owner(self, layer):
        from .tiller import layer_owner
        return layer_owner(layer, len(self.per_layer), self.world)

    @torch.no_grad()
    def replicate_state(self, muon):
        """Give every rank every layer's momentum buffer (one broadcast per
        matrix from its owner); a no-op before the first step."""
        state = muon.state
        started = torch.tensor([float(any("momentum_buffer" in state[p] for ps in self.per_layer
                                          for p in ps if id(p) in self.owned))],
                               device=self.per_layer[0][0].device)
        dist.all_reduce(started, op=dist.ReduceOp.MAX, group=self.group)
        if started.item() == 0.0:
            return
        for layer, ps in enumerate(self.per_layer):
            src = self.owner(layer)
            src = dist.get_global_rank(self.group, src) if self.group is not None else src
            for p in ps:
                st = state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                dist.broadcast(st["momentum_buffer"], src=src, group=self.group)


def shard_muon(muon: Muon, group=None):
    """Layer-shard ``muon`` across the ranks of ``group`` when every matrix
    belongs to a transformer layer (``layers.<i>.`` in its name); returns the
    shard or None (replicated)."""
    if not dist.is_available() or not dist.is_initialized():
        return None
    world = dist.get_world_size(group)
    if world <= 1 or os.environ.get("RO_MUON_SHARD", "1") == "0":
        return None
    per_layer = {}
    for g in muon.param_groups:
        names = g.get("param_names") or [None] * len(g["params"])
        for name, p in zip(names, g["params"]):
            m = _LAYER.search(name or "")
            if m is None or not p.is_cuda:
                return None
            per_layer.setdefault(int(m.group(1)), []).append(p)
    if not per_layer or sorted(per_layer) != list(range(len(per_layer))):
        return None
    muon.shard = MuonShard([per_layer[l] for l in range(len(per_layer))], world, dist.get_rank(group), group)
    return muon.shard
