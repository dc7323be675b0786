"""Protocol audits: the exact LR/WD fairness contract, the registered
experiment identity, and data-parallel replica equality
(reference training/train.py:969-1026, 1369-1567).

* :func:`audit_optimizer_lr_wd_fairness` proves that every trainable
  parameter sits in exactly one optimizer group at the base LR with the
  weight decay its name requires, and that no optimizer in the tree hides an
  LR or WD multiplier other than 1.0 (non-standard optimizers must declare
  theirs through ``lr_wd_fairness_audit()``).
* :func:`assert_optimizer_realized_lr` checks every group's LR against the
  schedule after it is set and after the step.
* :func:`assert_rlb_matrix_parameters_synced` /
  :func:`assert_rlb_coefficient_parameters_synced` all-gather the GRAIN
  matrices / coefficients and require bitwise equality across ranks.
"""
from __future__ import annotations

import hashlib

import torch
import torch.distributed as dist

from ..optim import baselines
from ..optim.adamw import FusedAdamW
from ..optim.composite import (TILLER_THEN_MUON_OPTIMIZER, CompositeOptimizer,
                               collect_rlb_optimizer_groups, is_no_decay_parameter,
                               is_tied_embedding_parameter_name, unwrap_model)

EXACT_LR_WD_CONTRACT = "exact_lr_wd_v1"
TILLER_LR_WD_CONTRACT = EXACT_LR_WD_CONTRACT
TILLER_EXPERIMENT_IDENTITY = "tiller_matrix_v1"
TILLER_THEN_MUON_EXPERIMENT_IDENTITY = "tiller_then_muon_matrix_v1"
TILLER_EXPERIMENT_IDENTITIES = (TILLER_EXPERIMENT_IDENTITY, TILLER_THEN_MUON_EXPERIMENT_IDENTITY)

_IDENTITY_AUDITOR = None


def install_tiller_identity_auditor(auditor):
    """Install the suite's model/data/schedule identity check (a callable)."""
    global _IDENTITY_AUDITOR
    if not callable(auditor):
        raise TypeError("TILLER identity auditor must be callable")
    _IDENTITY_AUDITOR = auditor


def audit_tiller_experiment_identity(args, *, world_size, global_tokens, train_token_count,
                                     val_token_count, parameter_count):
    if args.experiment_identity not in TILLER_EXPERIMENT_IDENTITIES:
        return None
    if _IDENTITY_AUDITOR is None:
        raise RuntimeError("the TILLER suite has not installed its identity auditor")
    return _IDENTITY_AUDITOR(args, world_size=world_size, global_tokens=global_tokens,
                             train_token_count=train_token_count, val_token_count=val_token_count,
                             parameter_count=parameter_count)


def optimizer_tree(optimizer):
    """Each optimizer object once, composite children included."""
    pending, seen = [optimizer], set()
    while pending:
        cur = pending.pop()
        if id(cur) in seen:
            continue
        seen.add(id(cur))
        yield cur
        pending.extend(getattr(cur, "optimizers", ()))


def _unit(value, *, label):
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise RuntimeError(f"{label} must be the literal scalar 1.0, got {value!r}")
    if float(value) != 1.0:
        raise RuntimeError(f"{label} must be 1.0, got {value!r}")


_STANDARD = (torch.optim.AdamW, torch.optim.Muon, FusedAdamW, CompositeOptimizer, baselines.Lion,
             baselines.AdEMAMix, baselines.ScheduleFreeAdamW, baselines.CAMEStyleAdamW,
             baselines.SOAPStyleAdamW)


def audit_optimizer_lr_wd_fairness(model, optimizer, args):
    if args.fairness_contract != EXACT_LR_WD_CONTRACT:
        return None
    raw = unwrap_model(model)
    named = {id(p): (n, p) for n, p in raw.named_parameters() if p.requires_grad}
    owner, records = {}, []
    for gi, group in enumerate(optimizer.param_groups):
        _unit(group.get("lr_scale", 1.0), label=f"param_groups[{gi}].lr_scale")
        if float(group.get("lr", args.lr)) != float(args.lr):
            raise RuntimeError(f"param_groups[{gi}].lr must equal base LR {args.lr}, got {group.get('lr')!r}")
        wd = float(group.get("weight_decay", 0.0))
        names, count = [], 0
        for p in group["params"]:
            if id(p) not in named:
                raise RuntimeError("optimizer contains an unknown or frozen parameter")
            name, original = named[id(p)]
            if id(p) in owner:
                raise RuntimeError(f"parameter {name} occurs in optimizer groups {owner[id(p)]} and {gi}")
            owner[id(p)] = gi
            tied_no_decay = is_tied_embedding_parameter_name(name) and args.optimizer in {
                "muon", "tiller_v1", TILLER_THEN_MUON_OPTIMIZER}
            required = 0.0 if is_no_decay_parameter(name, original) or tied_no_decay else float(args.weight_decay)
            if wd != required:
                raise RuntimeError(f"weight decay mismatch for {name}: {wd} != {required}")
            names.append(name)
            count += int(p.numel())
        records.append({"group_index": gi, "lr_scale": 1.0, "weight_decay": wd,
                        "parameter_tensor_count": len(names), "parameter_element_count": count,
                        "parameter_name_sha256": hashlib.sha256("\n".join(sorted(names)).encode("utf-8")).hexdigest()})
    missing = sorted(n for pid, (n, _) in named.items() if pid not in owner)
    if missing:
        raise RuntimeError(f"trainable parameters missing from optimizer: {missing[:8]}")
    internal = {}
    for oi, cur in enumerate(optimizer_tree(optimizer)):
        for attr, value in vars(cur).items():
            if attr.endswith(("_lr_scale", "_lr_scale_final", "_weight_decay_scale")):
                _unit(value, label=f"{type(cur).__name__}.{attr}")
                internal[f"{oi}:{type(cur).__name__}.{attr}"] = 1.0
        if isinstance(cur, _STANDARD):
            continue
        provider = getattr(cur, "lr_wd_fairness_audit", None)
        if provider is None:
            raise RuntimeError(f"nonstandard optimizer {type(cur).__name__} does not expose "
                               "lr_wd_fairness_audit(); campaign execution is refused")
        declared = provider()
        if not isinstance(declared, dict) or not declared:
            raise RuntimeError(f"{type(cur).__name__}.lr_wd_fairness_audit() must return a nonempty dict")
        for label, value in declared.items():
            _unit(value, label=f"{type(cur).__name__}.{label}")
            internal[f"{oi}:{type(cur).__name__}.{label}"] = 1.0
    return {
        "contract": EXACT_LR_WD_CONTRACT, "passed": True, "base_lr": float(args.lr),
        "minimum_lr": float(args.min_lr), "base_weight_decay": float(args.weight_decay),
        "group_count": len(records),
        "trainable_parameter_elements": sum(int(p.numel()) for _, p in named.values()),
        "covered_parameter_elements": sum(r["parameter_element_count"] for r in records),
        "groups": records, "internal_lr_wd_scalars": internal,
    }


def assert_optimizer_realized_lr(optimizer, scheduled_lr, args):
    if args.fairness_contract != EXACT_LR_WD_CONTRACT:
        return
    for gi, group in enumerate(optimizer.param_groups):
        _unit(group.get("lr_scale", 1.0), label=f"param_groups[{gi}].lr_scale")
        if float(group["lr"]) != float(scheduled_lr):
            raise RuntimeError(f"realized LR mismatch in param group {gi}: {float(group['lr'])} != {scheduled_lr}")


@torch.no_grad()
def assert_rlb_matrix_parameters_synced(model, args, device, is_distributed):
    params = []
    for g in collect_rlb_optimizer_groups(unwrap_model(model), args):
        params.extend((g["in_weight"], g["out_weight"]))
    if not params:
        raise RuntimeError("DDP parameter synchronization check found no GRAIN matrix pair")
    if not is_distributed:
        return 0.0
    world = dist.get_world_size()
    chunk = 1 << 20
    for p in params:
        flat = p.detach().float().reshape(-1)
        for start in range(0, flat.numel(), chunk):
            local = flat[start:start + chunk].to(device=device)
            gathered = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(gathered, local)
            for peer in gathered[1:]:
                diff = float((peer - gathered[0]).abs().max().item())
                if diff != 0.0:
                    raise RuntimeError("DDP GRAIN matrix replicas diverged after optimizer step; "
                                       f"max absolute difference={diff}")
    return 0.0


@torch.no_grad()
def assert_rlb_coefficient_parameters_synced(model, args, device, is_distributed):
    values = []
    for g in collect_rlb_optimizer_groups(unwrap_model(model), args):
        values.extend((g["numerator"].detach().float().reshape(-1), g["denominator"].detach().float().reshape(-1)))
    if not values:
        raise RuntimeError("DDP coefficient synchronization check found no GRAIN coefficients")
    if not is_distributed:
        return 0.0
    local = torch.cat(values).to(device=device)
    gathered = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(gathered, local)
    worst = max(float((peer - gathered[0]).abs().max().item()) for peer in gathered[1:])
    if worst != 0.0:
        raise RuntimeError(f"DDP GRAIN coefficient replicas diverged after optimizer step; max absolute difference={worst}")
    return worst
