"""Portable torchrun trainer of the MHA study (reference experiments/mha_1b_tokens/train.py:1-278).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rational_optimizer_b200.mha.train \\
        --condition grain_tiller --data caches/manifest.json --output runs/grain_tiller \\
        [--config config.json] [--resume latest] [--microbatch M --accumulation A] \\
        [--max-hours H] [--stop-after U] [--device cpu]

Every update reads disjoint packed windows (:class:`PackedBatches`), the LR
follows warm-up + cosine to ``min_lr_ratio`` at the schedule horizon, the
gradient norm is clipped once at 1.0, validation runs every
``validation_every`` updates on a fixed prefix of the validation cache, and
checkpoints are atomic and checksum-verified at update boundaries
(periodic / switch / final / continuation).  A resumed run verifies the
run identity (config, data manifest, world size, condition) and that the
next batch is the one the interrupted run would have read; metric records
past the durable checkpoint are archived, never silently kept.  Each rank
runs on its own GPU with gradients averaged by the package's synchroniser.
"""
from __future__ import annotations

import argparse
import fcntl
import hashlib
import json
import math
import os
import random
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from ..parallel.grad_sync import GradientSynchronizer
from . import checkpoint
from . import config as C
from .config import GRAIN_CONDITIONS, MHA_SWITCH, default_config, schedule, validate_config
from .data import PackedBatches, atomic_json, digest, object_digest
from .model import ModernMHADecoder, copy_shared
from .optim import build_optimizer


def initial_model(cfg, condition):
    """Seeded SwiGLU model; GRAIN conditions copy its shared tensors so every condition starts alike."""
    random.seed(cfg["seed"])
    np.random.seed(cfg["seed"])
    torch.manual_seed(cfg["seed"])
    base = ModernMHADecoder(cfg["model"])
    if condition in GRAIN_CONDITIONS:
        model = ModernMHADecoder(cfg["model"], grain=True, groups=cfg["grain"]["groups"])
        copied = copy_shared(base, model)
    else:
        model = base
        copied = [n for n, _ in model.named_parameters() if ".mlp." not in n]
    h = hashlib.sha256()
    for name, p in model.named_parameters():
        if name in copied:
            h.update(name.encode())
            h.update(p.detach().contiguous().numpy().tobytes())
    return model, h.hexdigest()


def batch_hash(data, update, rank):
    try:
        x, y, mask = data.batch(update, 0, rank)
    except IndexError:
        return "END"
    return hashlib.sha256(x.tobytes() + y.tobytes() + mask.tobytes()).hexdigest()


def train_step(model, optimizer, sync, data, completed, cfg, device, rank, world):
    optimizer.zero_grad()
    sync.zero_grad()
    if optimizer.router is not None and (completed + 1) % 100 == 0:
        optimizer.router.set_telemetry_capture(True)
        optimizer.attention.set_telemetry_capture(True)
    lr = schedule(completed, cfg, cfg["conditions"][optimizer.condition]["lr"])
    for g in optimizer.param_groups:
        g["lr"] = lr
    count = 0
    summed = torch.zeros((), device=device)
    for micro in range(cfg["accumulation"]):
        x, y, mask = data.batch(completed, micro, rank)
        if not mask.all():
            raise RuntimeError("the packing protocol requires every target to be loss-bearing")
        count += int(mask.sum())
        value = model.forward_loss(torch.from_numpy(x).to(device), torch.from_numpy(y).to(device))
        if micro == cfg["accumulation"] - 1:
            sync.begin_backward()
        (value / cfg["accumulation"]).backward()
        summed += value.detach().float() / cfg["accumulation"]
    sync.synchronize()
    total = torch.tensor([count], device=device, dtype=torch.int64)
    if dist.is_initialized():
        dist.all_reduce(total)
    if int(total.item()) != cfg["loss_tokens_per_update"]:
        raise RuntimeError("actual mask count differs")
    norm = optimizer.clip_grad_norm()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    optimizer.step()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    opt_seconds = time.perf_counter() - t0
    if dist.is_initialized():
        dist.all_reduce(summed)
    value = float(summed / world)
    if not math.isfinite(value):
        raise RuntimeError("nonfinite training loss")
    return dict(loss=value, lr=lr, loss_tokens_this_update=int(total.item()), gradient_norm=float(norm),
                optimizer_seconds=opt_seconds,
                phase=getattr(optimizer, "phase", "tiller" if optimizer.router is not None else "baseline"),
                optimizer_child_lrs={role: [g["lr"] for g in child.param_groups]
                                     for role, child in zip(optimizer.roles, optimizer.children)})


@torch.no_grad()
def validation(model, path, cfg, device, rank, world):
    ids = np.memmap(path, dtype="<u4", mode="r")
    context, tokens = cfg["context"], cfg["small_validation_tokens"]
    if tokens % context or len(ids) <= tokens:
        raise ValueError("validation cache too short or unaligned")
    total = torch.zeros(2, device=device, dtype=torch.float64)
    was_training = model.training
    model.eval()
    try:
        for index in range(rank, tokens // context, world):
            block = torch.from_numpy(np.array(ids[index * context:(index + 1) * context + 1], dtype=np.int64)).to(device)[None]
            value = model.forward_loss(block[:, :-1], block[:, 1:])
            total += torch.stack((value.double() * context, value.new_tensor(context).double()))
    finally:
        model.train(was_training)
    if dist.is_initialized():
        dist.all_reduce(total)
    if int(total[1]) != tokens:
        raise RuntimeError("validation token count differs")
    value = float(total[0] / total[1])
    if not math.isfinite(value):
        raise RuntimeError("nonfinite validation loss")
    return value


def reconcile_metrics(path: Path, completed: int):
    """Keep records up to the durable checkpoint; archive the rest."""
    if not path.exists():
        return
    lines = path.read_text().splitlines(True)
    kept, abandoned = [], []
    for i, line in enumerate(lines):
        try:
            rec = json.loads(line)
        except json.JSONDecodeError:
            if i != len(lines) - 1:
                raise RuntimeError("corrupt metrics before the final line")
            abandoned.append(line)
            continue
        (kept if rec["step"] <= completed else abandoned).append(line)
    if abandoned:
        with path.with_name(f"metrics-abandoned-{time.time_ns()}.jsonl").open("x") as fh:
            fh.writelines(abandoned)
            fh.flush()
            os.fsync(fh.fileno())
        tmp = path.with_name(f".metrics-{time.time_ns()}.partial")
        with tmp.open("x") as fh:
            fh.writelines(kept)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)


def main(argv=None):
    launch_started = time.monotonic()
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--condition", required=True, choices=("swiglu_muon", "swiglu_adamw", "grain_tiller", MHA_SWITCH))
    p.add_argument("--data", type=Path, required=True, help="local uint32 cache manifest")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--config", type=Path, default=None)
    p.add_argument("--resume", help="verified manifest path, or 'latest' under --output")
    p.add_argument("--microbatch", type=int)
    p.add_argument("--accumulation", type=int)
    p.add_argument("--max-hours", type=float)
    p.add_argument("--checkpoint-margin-seconds", type=float, default=900)
    p.add_argument("--stop-after", type=int)
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    a = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    device = torch.device("cuda", local) if a.device == "cuda" else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl" if device.type == "cuda" else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    cfg = json.loads(a.config.read_text()) if a.config else default_config()
    cfg["world_size"] = world
    if a.microbatch is not None:
        cfg["microbatch"] = a.microbatch
    if a.accumulation is not None:
        cfg["accumulation"] = a.accumulation
    validate_config(cfg)
    if a.max_hours is not None and a.max_hours * 3600 <= a.checkpoint_margin_seconds:
        raise ValueError("walltime is shorter than the checkpoint margin")
    if a.stop_after is not None and not 1 <= a.stop_after <= cfg["updates"]:
        raise ValueError("invalid stop boundary")
    manifest = json.loads(a.data.read_text())
    if manifest["dtype"] != "<u4":
        raise ValueError("cache dtype differs")
    paths = {}
    for split in ("train", "validation"):
        item = manifest["splits"][split]
        path = Path(item["path"])
        paths[split] = path if path.is_absolute() else a.data.parent / path
        if rank == 0 and (digest(paths[split]) != item["sha256"] or paths[split].stat().st_size != 4 * item["tokens"]):
            raise RuntimeError("cache checksum/size mismatch")
    checkpoint.barrier()
    data = PackedBatches(paths["train"], world_size=world, microbatch=cfg["microbatch"],
                         accumulation=cfg["accumulation"], context=cfg["context"])
    data.batch(cfg["updates"] - 1, cfg["accumulation"] - 1, world - 1)  # the whole horizon must be local
    identity = dict(schema=1, condition=a.condition, config=object_digest(cfg), data=digest(a.data),
                    world_size=world, precision="bf16_gemm_fp32_master" if device.type == "cuda" else "cpu_fp32")
    a.output.mkdir(parents=True, exist_ok=True)
    lock = None
    if rank == 0:
        lock = (a.output / "trainer.lock").open("a")
        fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
        old = a.output / "identity.json"
        if old.exists():
            if not a.resume or json.loads(old.read_text()) != identity:
                raise RuntimeError("existing output requires explicit resume with a matching identity")
        elif a.resume:
            raise RuntimeError("resume requires the original output directory")
        else:
            atomic_json(old, identity)
            atomic_json(a.output / "resolved_config.json", cfg)
    checkpoint.barrier()
    model, shared_hash = initial_model(cfg, a.condition)
    count = sum(p.numel() for p in model.parameters())
    model = model.to(device)
    if device.type == "cpu":
        for m in model.modules():
            if hasattr(m, "out_dtype"):
                m.out_dtype = None
    sync = GradientSynchronizer(model)
    optimizer = build_optimizer(model, a.condition, cfg["conditions"][a.condition]["lr"], cfg["accumulation"])
    completed = 0
    if a.resume:
        saved = json.loads((a.output / "latest.json").read_text())["manifest"] if a.resume == "latest" else a.resume
        completed = checkpoint.load(saved, model, optimizer, identity, lambda u: batch_hash(data, u, rank))
        if rank == 0:
            reconcile_metrics(a.output / "metrics.jsonl", completed)
        checkpoint.barrier()
    if rank == 0:
        atomic_json(a.output / "startup.json", dict(parameter_count=count, shared_initial_sha256=shared_hash,
                                                    resumed_update=completed, identity=identity))
    saved_update = completed if a.resume else -1

    def save(kind):
        nonlocal saved_update
        mp = checkpoint.save(a.output / f"checkpoint-{completed:06d}-{kind}", model, optimizer, completed, identity,
                             batch_hash(data, completed, rank))
        if rank == 0:
            atomic_json(a.output / "latest.json", dict(manifest=str(mp.resolve()), update=completed,
                                                       tokens=completed * cfg["loss_tokens_per_update"]))
            checkpoint.prune_periodic(a.output, identity, cfg["checkpoint_keep_recent"])
        checkpoint.barrier()
        saved_update = completed

    while completed < cfg["updates"]:
        tick = time.perf_counter()
        metrics = train_step(model, optimizer, sync, data, completed, cfg, device, rank, world)
        completed += 1
        metrics.update(step=completed, loss_tokens=completed * cfg["loss_tokens_per_update"],
                       seconds=time.perf_counter() - tick,
                       peak_memory_bytes=torch.cuda.max_memory_allocated(device) if device.type == "cuda" else 0)
        if completed % cfg["validation_every"] == 0 or completed == cfg["updates"]:
            metrics["validation_loss"] = validation(model, paths["validation"], cfg, device, rank, world)
        if optimizer.router is not None and completed % 100 == 0:
            metrics["tiller_telemetry"] = optimizer.router.telemetry()
            metrics["attention_telemetry"] = optimizer.attention.telemetry()
        if rank == 0:
            with (a.output / "metrics.jsonl").open("a") as fh:
                fh.write(json.dumps(metrics, allow_nan=False, default=float) + "\n")
            print(json.dumps(metrics, allow_nan=False, default=float), flush=True)
        boundary = a.condition == MHA_SWITCH and completed in (C.SWITCH_UPDATE, C.SWITCH_UPDATE + 1)
        final = completed == cfg["updates"]
        if boundary or final or completed % cfg["checkpoint_every"] == 0:
            save("final" if final else "switch" if boundary else "periodic")
        stop = torch.tensor(int((a.stop_after is not None and completed >= a.stop_after) or
                                (a.max_hours is not None and
                                 time.monotonic() - launch_started >= a.max_hours * 3600 - a.checkpoint_margin_seconds)),
                            device=device)
        if dist.is_initialized():
            dist.all_reduce(stop, op=dist.ReduceOp.MAX)
        if stop.item():
            break
    if completed > 0 and completed != saved_update and completed != cfg["updates"]:
        save("continuation")
    if rank == 0:
        atomic_json(a.output / "result.json", dict(completed=completed == cfg["updates"], update=completed,
                                                   loss_tokens=completed * cfg["loss_tokens_per_update"],
                                                   identity=identity))
    checkpoint.barrier()
    if getattr(sync, "communicator", None) is not None:
        sync.communicator.close()
    if dist.is_initialized():
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
