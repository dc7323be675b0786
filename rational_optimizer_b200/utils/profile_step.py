"""Kernel-time breakdown of one training step (diagnostics, not a benchmark).

    python -m rational_optimizer_b200.utils.profile_step [--layers 18] [--batch 32]

Runs a few warm-up steps of the GRAIN model with the chosen optimizer, then
profiles ``--steps`` steps with torch.profiler and prints the kernels sorted
by total device time, the share of this package's kernels and the number of
launches per step.  Numbers taken under a profiler are for attribution only.
"""
from __future__ import annotations

import argparse
import collections

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=18)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--optimizer", default="tiller_v1")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--top", type=int, default=30)
    a = ap.parse_args()
    from torch.profiler import ProfilerActivity, profile
    from ..models.transformer import CausalTransformer, model_args
    from ..optim import composite
    from ..train.engine import TrainEngine

    args = model_args(layers=a.layers, d_model=1024, heads=16, ffn_dim=3072, seq_len=a.seq,
                      activation="grain", optimizer=a.optimizer, lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(0)
    model = CausalTransformer(args, 50304).cuda()
    opt = composite.configure_optimizer(model, args)
    eng = TrainEngine(model, opt)
    toks = torch.randint(0, 50304, (a.batch, a.seq + 1), device="cuda")
    batch = [(toks[:, :-1], toks[:, 1:])]
    for _ in range(a.warmup):
        eng.step(batch, lr=3e-4)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        for _ in range(a.steps):
            eng.step(batch, lr=3e-4)
        torch.cuda.synchronize()
    totals = collections.Counter()
    counts = collections.Counter()
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            totals[e.name] += e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total
            counts[e.name] += 1
    all_us = sum(totals.values())
    own_us = sum(v for k, v in totals.items() if "ro::" in k)
    print(f"device time per step: {all_us / a.steps / 1000:.2f} ms; this package's kernels: "
          f"{own_us / max(all_us, 1) * 100:.1f}%; launches per step: {sum(counts.values()) // a.steps}")
    for name, us in totals.most_common(a.top):
        print(f"{us / a.steps / 1000:9.3f} ms  {counts[name] // a.steps:5d}x  {name[:150]}")


if __name__ == "__main__":
    main()
