#!/usr/bin/env python3
"""Headline benchmark: training tokens/s of the 18-layer, 1024-wide GRAIN
Transformer (296.9M parameters at vocab 50,304) with the TILLER optimizer,
seq 1024, global batch 32 sequences, data-parallel over N GPUs (one process
per GPU).  Synthetic Zipf(1.1) token ids from seed 0, random-init weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torchrun (RANK/LOCAL_RANK/WORLD_SIZE from the env).
``value`` is device-timed (CUDA events around exactly K steps, barrier +
synchronize on both sides, max over ranks) with inputs already on the device;
``e2e`` re-times K steps through the public ``TrainEngine`` API including the
pinned host->device copy of each step's tokens and the device->host read of
the step's loss.  ``--impl reference`` runs the unmodified reference trainer
code path (installed under baseline/_ref) on the same model, data and timing.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
METRIC = "train tokens/sec at 18L/1024d GRAIN+TILLER (1/2/4/8 B200, max over ranks)"
BASELINE_TOKENS_PER_S = 38528.0  # published 18L GRAIN+TILLER (4x A6000, seq 256)
MODEL_CFG = dict(layers=18, d_model=1024, heads=16, ffn_dim=3072, seq_len=1024,
                 activation="grain", rational_init="silu", rational_group_size=256,
                 rational_max_groups=32, rational_basis_eps=1e-6, init_std=0.02)
VOCAB = 50304
GLOBAL_BATCH = 32
SEQ = 1024
ZIPF_TOKENS = 8_000_000


# where the reference's unmodified source tree is read from when baseline/_ref
# has to be installed on this machine (RO_REFERENCE_SRC overrides it)
REF_SRC = os.environ.get("RO_REFERENCE_SRC", "/root/reference")


def ensure_reference() -> str | None:
    """Install the unmodified reference into baseline/_ref when it is missing.

    The install is the same one recorded for this arm: ``pip install --no-index
    --no-build-isolation --find-links /opt/wheelhouse --target baseline/_ref``
    of a copy of the reference tree (its build writes into the source tree),
    with its CUDA extension compiled for sm_100; the reference's unpackaged
    study directories are copied beside it unmodified.  Ranks of one node
    serialise on a lock file, so one of them installs and the rest reuse it.
    Returns None when the package is present afterwards, else the reason.
    """
    import fcntl
    import shutil
    import tempfile
    if os.path.isdir(os.path.join(REF_DIR, "training")):
        return None
    if not os.path.isdir(REF_SRC):
        return "reference package not installed in baseline/_ref and no reference source to build it from"
    os.makedirs(os.path.dirname(REF_DIR), exist_ok=True)
    with open(os.path.join(os.path.dirname(REF_DIR), ".install.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if os.path.isdir(os.path.join(REF_DIR, "training")):
            return None
        with tempfile.TemporaryDirectory() as tmp:
            src = os.path.join(tmp, "reference")
            shutil.copytree(REF_SRC, src, ignore=shutil.ignore_patterns(".git"))
            env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0")
            done = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index",
                                   "--no-build-isolation", "--no-deps", "--find-links", "/opt/wheelhouse",
                                   "--target", REF_DIR, src], env=env, capture_output=True, text=True)
            if done.returncode != 0:
                tail = (done.stderr or done.stdout).strip().splitlines()[-1:] or [""]
                return f"reference install failed: {tail[0][:200]}"
        # the protocol's data files (manifest, matrix, source freeze) sit beside
        # its installed modules; the studies and results are not packaged
        for sub in ("protocol", "mha_1b_tokens", "swiglu_tiller", "results"):
            there = os.path.join(REF_SRC, "experiments", sub)
            if os.path.isdir(there):
                shutil.copytree(there, os.path.join(REF_DIR, "experiments", sub), dirs_exist_ok=True,
                                ignore=shutil.ignore_patterns("__pycache__"))
    return None if os.path.isdir(os.path.join(REF_DIR, "training")) else "reference install left no package"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--optimizer", default="tiller_v1")
    ap.add_argument("--global-batch", type=int, default=GLOBAL_BATCH)
    ap.add_argument("--layers", type=int, default=MODEL_CFG["layers"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-count-launches", action="store_true")
    return ap.parse_args()


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region.

    nvidia-smi writes straight into a temporary file and is parsed after the
    region, so no thread of the benchmark process wakes up while it is timed.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None

    def start(self):
        import tempfile
        self.file = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        samples = []
        if self.file is not None:
            self.file.seek(0)
            for line in self.file:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    samples.append(parts)
            self.file.close()
        mhz, maxes, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for s in samples:
            try:
                mhz.append(float(s[1]))
                maxes.append(float(s[2]))
            except ValueError:
                continue
            for name, val in zip(names, s[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None,
                "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


def count_own_launches(step_fn):
    """Run one step under the profiler and count launches of this package's kernels."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    own = total = 0
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA:
            total += 1
            if "ro::" in evt.name or "(anonymous namespace)::" in evt.name and "ro" in evt.name:
                own += 1
    return own, total


def timed(step_fn, steps, device, dist_on, flush=None, kind=None):
    """Mean device ms per step over exactly ``steps`` steps, MAX over ranks.

    An event is also recorded after every step (no synchronisation), so the
    per-step device times can be split by ``kind()`` (called before each
    step, e.g. ``"plain"`` / ``"refresh"``); returns (ms, {kind: [median ms,
    count, max ms]}) with each median and maximum also reduced with MAX over
    ranks (the maximum shows a slow outlier step that the median hides).
    """
    import torch
    import torch.distributed as dist
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize(device)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    end = torch.cuda.Event(enable_timing=True)
    kinds = []
    marks[0].record()
    for i in range(steps):
        kinds.append(kind() if kind is not None else "step")
        step_fn()
        marks[i + 1].record()
    if flush is not None:
        flush()  # side-stream work of the last step (deferred weight broadcasts) inside the region
    end.record()
    torch.cuda.synchronize(device)
    if dist_on:
        dist.barrier()
    ms = marks[0].elapsed_time(end) / steps
    per = {}
    for i, k in enumerate(kinds):
        per.setdefault(k, []).append(marks[i].elapsed_time(marks[i + 1]))
    names = sorted(per)
    med = [sorted(per[k])[len(per[k]) // 2] for k in names]
    top = [max(per[k]) for k in names]
    global LAST_RANK_MS, LAST_STEP_MS
    steps_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
    LAST_RANK_MS = [round(ms, 3)]
    if dist_on:
        every = torch.zeros(dist.get_world_size(), device=device)
        dist.all_gather_into_tensor(every, torch.tensor([ms], device=device))
        LAST_RANK_MS = [round(v, 3) for v in every.tolist()]
        t = torch.tensor([ms] + med + top + steps_ms, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = len(names)
        vals = t.tolist()
        ms, med, top, steps_ms = vals[0], vals[1:1 + n], vals[1 + n:1 + 2 * n], vals[1 + 2 * n:]
    LAST_STEP_MS = [round(v, 2) for v in steps_ms]
    return ms, {k: [round(m, 3), len(per[k]), round(x, 3)] for k, m, x in zip(names, med, top)}


# device ms per step of every rank in the last timed() window (which rank sets the MAX),
# and each step's device ms in that window (MAX over ranks), in order
LAST_RANK_MS = []
LAST_STEP_MS = []


def run_ours(a, info):
    import torch
    sys.path.insert(0, ROOT)
    from rational_optimizer_b200.models.transformer import model_args, CausalTransformer
    from rational_optimizer_b200.optim import composite
    from rational_optimizer_b200.parallel import param_ready
    from rational_optimizer_b200.parallel.grad_sync import GradientSynchronizer
    from rational_optimizer_b200.train.data import PinnedBatcher, zipf_tokens
    from rational_optimizer_b200.train.engine import TrainEngine

    device = info.device
    world = info.world_size
    local_batch = a.global_batch // world
    cfg = dict(MODEL_CFG, layers=a.layers)
    args = model_args(**cfg, optimizer=a.optimizer, lr=3e-4, weight_decay=0.1, muon_momentum=0.95,
                      muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(1337)
    model = CausalTransformer(args, VOCAB).to(device)
    if info.is_distributed:
        import torch.distributed as dist
        for p in model.parameters():
            dist.broadcast(p.data, 0)
    optimizer = composite.configure_optimizer(model, args)
    layers, owner_of = composite.owner_layers(optimizer)
    sync = GradientSynchronizer(model, owner_layers=layers, layer_owner=owner_of)
    engine = TrainEngine(model, optimizer, grad_clip=1.0, grad_accum=1, synchronizer=sync)
    tokens = zipf_tokens(ZIPF_TOKENS, VOCAB, alpha=1.1, seed=0)
    batcher = PinnedBatcher(tokens, local_batch, SEQ, seed=0, rank=info.rank)
    # device-resident inputs for the kernel-timed loop
    staged = [batcher.to_device(device, batcher.next_host().clone()) for _ in range(4)]
    counter = {"i": 0}

    def device_step():
        x, y = staged[counter["i"] % len(staged)]
        counter["i"] += 1
        engine.step([(x, y)], lr=3e-4)

    def e2e_step():
        host = batcher.next_host()
        x, y = batcher.to_device(device, host)
        loss = engine.step([(x, y)], lr=3e-4)
        return float(loss.item())

    from rational_optimizer_b200.utils.step_phases import step_kind

    def kind():
        return step_kind(engine)

    for _ in range(a.warmup):
        device_step()
    sampler = ClockSampler(device.index or 0) if info.rank == 0 else None
    if sampler:
        sampler.start()
    start_step = counter["i"]
    ms, split = timed(device_step, a.steps, device, info.is_distributed, flush=param_ready.wait_all,
                      kind=kind)
    split = dict(split, ms_per_rank=list(LAST_RANK_MS), steps_ms=list(LAST_STEP_MS))
    clocks = sampler.stop() if sampler else None
    e2e_ms = e2e_split = None
    if not a.no_e2e:
        # start the end-to-end window at the same phase of the optimizer's
        # 8-step refresh cadence as the device-timed window, so both hold the
        # same number of refresh steps
        done = a.warmup + a.steps
        extra = 2 + (start_step - (done + 2)) % 8
        for _ in range(extra):
            e2e_step()
        e2e_ms, e2e_split = timed(e2e_step, a.steps, device, info.is_distributed,
                                  flush=param_ready.wait_all, kind=kind)
    launches = None
    if not a.no_count_launches:  # every rank profiles one step (same collective sequence)
        own, total = count_own_launches(device_step)
        launches = {"own_per_step": own, "all_per_step": total}
    loss = float(engine.step([staged[0]], lr=3e-4).item())
    if sync.communicator is not None:
        sync.communicator.check()
    return (ms, e2e_ms, clocks, launches, loss, batcher.bytes_per_batch, sync.transport,
            {"device": split, "e2e": e2e_split})


def run_reference(a, info):
    """The reference trainer's own objects and step sequence (training/train.py:2814-2950)."""
    import torch
    import torch.nn.functional as F
    if not os.path.isdir(os.path.join(REF_DIR, "training")):
        return None
    sys.path.insert(0, REF_DIR)
    os.environ.pop("RATIONAL_OPT_TORCH_FALLBACK", None)
    from training import train as T
    from experiments.protocol import method_entrypoint as M
    import types
    device = info.device
    world = info.world_size
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    torch.set_float32_matmul_precision("high")
    args = types.SimpleNamespace(**MODEL_CFG)
    args.layers = a.layers
    args.optimizer = "tiller_v1"
    args.lr, args.min_lr, args.warmup_steps, args.weight_decay = 3e-4, 3e-5, 200, 0.1
    args.beta1, args.beta2, args.eps = 0.9, 0.95, 1e-8
    args.muon_momentum, args.muon_ns_steps, args.muon_adjust_lr_fn = 0.95, 5, "match_rms_adamw"
    args.grad_clip, args.grad_accum, args.batch_size = 1.0, 1, a.global_batch // world
    args.steps = a.warmup + 2 * a.steps + 4
    T.RATIONAL_SPECIFIC_OPTIMIZERS.add(M.OPTIMIZER_ID)
    T.ACTIVE_OPTIMIZERS = sorted(set(T.ACTIVE_OPTIMIZERS) | {M.OPTIMIZER_ID})
    T.configure_optimizer = M.configure_candidate_optimizer
    T.clip_or_measure_gradients = M.clip_candidate_gradients
    torch.manual_seed(1337)
    torch.cuda.manual_seed_all(1337)
    model = T.CausalTransformer(args, VOCAB).to(device)
    if info.is_distributed:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[info.local_rank],
                                                          output_device=info.local_rank)
    M.set_experiment_layout(microbatches=1, decay_tied_embedding=False)
    optimizer = M.configure_candidate_optimizer(model, args)
    from rational_optimizer_b200.train.data import zipf_tokens
    tokens = zipf_tokens(ZIPF_TOKENS, VOCAB, alpha=1.1, seed=0).pin_memory()
    offsets = torch.arange(SEQ + 1)
    gen = torch.Generator(device="cpu")
    gen.manual_seed(1337 + 997 * info.rank)
    state = {"step": 0}

    def one_step(read_loss):
        step = state["step"]
        state["step"] += 1
        lr = T.learning_rate(step, args)
        for group in optimizer.param_groups:
            group["lr"] = lr * float(group.get("lr_scale", 1.0))
        optimizer.zero_grad(set_to_none=True)
        x, y = T.sample_batch(tokens, args.batch_size, SEQ, offsets, gen, device)
        logits = model(x)
        loss = F.cross_entropy(logits.view(-1, logits.size(-1)), y.reshape(-1))
        loss.backward()
        T.clip_or_measure_gradients(model, args.grad_clip, False)
        optimizer.step()
        return float(loss.item()) if read_loss else loss

    for _ in range(a.warmup):
        one_step(True)
    sampler = ClockSampler(device.index or 0) if info.rank == 0 else None
    if sampler:
        sampler.start()
    ms, split = timed(lambda: one_step(True), a.steps, device, info.is_distributed)
    clocks = sampler.stop() if sampler else None
    # the timed loop is already end to end: each step copies its batch from
    # pinned host memory (sample_batch) and reads the loss back (loss.item())
    h2d = 2 * args.batch_size * SEQ * tokens.element_size()
    return ms, clocks, h2d


def main():
    a = parse()
    sys.path.insert(0, ROOT)
    missing = ensure_reference() if a.impl == "reference" else None
    import torch
    from rational_optimizer_b200.parallel.dist import cleanup_distributed, setup_distributed
    info = setup_distributed()
    if a.gpus != info.world_size:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={info.world_size}")
    tokens_per_step = a.global_batch * SEQ
    cfg = {"model": "18L/1024d/16h GRAIN (H=4608, G=18), vocab 50304, 296.92M params",
           "global_batch": a.global_batch, "seq_len": SEQ, "parallelism": f"dp{a.gpus}",
           "optimizer": a.optimizer, "grad_accum": 1,
           "l2": "inputs and working set larger than L2 (no flush needed)"}
    if a.layers != MODEL_CFG["layers"]:
        cfg["model"] = f"{a.layers}L/1024d GRAIN (reduced depth)"
    if a.impl == "reference":
        try:
            res = run_reference(a, info)
        except Exception as exc:  # report, do not crash the driver
            res = None
            reason = f"reference run failed: {type(exc).__name__}: {str(exc)[:200]}"
        else:
            reason = missing or "reference package not installed in baseline/_ref"
        if res is None:
            if info.rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
            cleanup_distributed(info)
            return
        ms, clocks, h2d = res
        value = tokens_per_step / (ms / 1000.0)
        if info.rank == 0:
            print(json.dumps({
                "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
                "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong",
                "vs_baseline": value / BASELINE_TOKENS_PER_S, "dtype": "fp32+tf32",
                "data": "synthetic Zipf(1.1) token ids, seed 0; random-init weights",
                "config": cfg, "clocks": clocks,
                "e2e": {"value": value, "unit": "tokens/s", "ms_per_step": ms,
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                        "note": "the reference's own step loop: sample_batch H2D copy and "
                                "loss.item() inside every timed step"}}), flush=True)
        cleanup_distributed(info)
        return
    ms, e2e_ms, clocks, launches, loss, h2d, transport, split = run_ours(a, info)
    value = tokens_per_step / (ms / 1000.0)
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": value / BASELINE_TOKENS_PER_S, "dtype": "bf16",
        "data": "synthetic Zipf(1.1) token ids, seed 0; random-init weights",
        "config": cfg, "clocks": clocks, "final_loss": loss,
    }
    out["config"]["grad_transport"] = transport
    # per-step device time by step kind: {kind: [median ms, steps, max ms]}; "refresh"
    # steps run the optimizer's response-probe refresh (one in eight)
    out["step_ms_by_kind"] = split
    if e2e_ms is not None:
        out["e2e"] = {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
                      "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4}
    if launches is not None:
        out["gpu_launches"] = launches["own_per_step"] * a.steps
        out["gpu_launches_detail"] = {"own_per_step": launches["own_per_step"],
                                      "all_kernels_per_step": launches["all_per_step"]}
    if info.rank == 0:
        print(json.dumps(out), flush=True)
    cleanup_distributed(info)


if __name__ == "__main__":
    main()
