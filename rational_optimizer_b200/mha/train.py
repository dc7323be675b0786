"""Portable torchrun trainer of the MHA study (behaviour of
experiments/mha_1b_tokens/train.py:1-278; same CLI, outputs and checkpoints).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rational_optimizer_b200.mha.train \\
        --condition grain_tiller --data caches/manifest.json --output runs/grain_tiller \\
        [--config config.json] [--resume latest] [--microbatch M --accumulation A] \\
        [--max-hours H] [--stop-after U] [--device cpu]

:class:`StudyRun` owns one run: it verifies the token caches, fixes the run
identity (condition, config digest, data-manifest digest, world size,
precision) and the output directory, builds the seeded model and the
condition's optimizer, and optionally resumes from a verified checkpoint.
``StudyRun.update`` performs one optimizer update over ``accumulation``
disjoint packed micro-batches (gradients averaged by the package's
synchroniser, clip at 1.0, warm-up + cosine LR); validation runs every
``validation_every`` updates on a fixed prefix of the validation cache;
checkpoints (periodic / switch / final / continuation) go through
:class:`~.checkpoint.CheckpointStore`.  On resume, metric records past the
durable checkpoint are archived to ``metrics-abandoned-*.jsonl``, never kept.
"""
from __future__ import annotations

import argparse
import datetime
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

TELEMETRY_EVERY = 100


def _shared_digest(model, names):
    """SHA-256 over (name, raw bytes) of the named parameters, in model order."""
    h = hashlib.sha256()
    wanted = set(names)
    for name, p in model.named_parameters():
        if name in wanted:
            h.update(name.encode())
            h.update(p.detach().contiguous().numpy().tobytes())
    return h.hexdigest()


def initial_model(cfg, condition):
    """(model, digest of its shared initial tensors).

    Every condition starts from the same seeded SwiGLU decoder; GRAIN
    conditions take over its attention, norm and embedding tensors, so the
    digest of the tensors the conditions share is equal across conditions.
    """
    seed = cfg["seed"]
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    swiglu = ModernMHADecoder(cfg["model"])
    if condition not in GRAIN_CONDITIONS:
        return swiglu, _shared_digest(swiglu, [n for n, _ in swiglu.named_parameters() if ".mlp." not in n])
    grain = ModernMHADecoder(cfg["model"], grain=True, groups=cfg["grain"]["groups"])
    return grain, _shared_digest(grain, copy_shared(swiglu, grain))


def batch_hash(data, update, rank):
    """Digest of this rank's first micro-batch of ``update`` ("END" past the cache)."""
    try:
        arrays = data.batch(update, 0, rank)
    except IndexError:
        return "END"
    return hashlib.sha256(b"".join(a.tobytes() for a in arrays)).hexdigest()


def reconcile_metrics(path: Path, completed: int):
    """Keep the records up to the durable checkpoint; archive the others (a torn
    last line included) to ``metrics-abandoned-<ns>.jsonl``."""
    if not path.exists():
        return
    lines = path.read_text().splitlines(True)
    keep, drop = [], []
    for i, line in enumerate(lines):
        try:
            step = json.loads(line)["step"]
        except json.JSONDecodeError:
            if i + 1 != len(lines):
                raise RuntimeError(f"{path}: unreadable record on line {i + 1} of {len(lines)}")
            drop.append(line)
            continue
        (keep if step <= completed else drop).append(line)
    if not drop:
        return

    def durable(target, records):
        with target.open("x") as fh:
            fh.writelines(records)
            fh.flush()
            os.fsync(fh.fileno())

    stamp = time.time_ns()
    durable(path.with_name(f"metrics-abandoned-{stamp}.jsonl"), drop)
    staged = path.with_name(f".metrics-{stamp}.partial")
    durable(staged, keep)
    os.replace(staged, path)


class StudyRun:
    """One condition's training run on this rank."""

    def __init__(self, a):
        self.started = time.monotonic()
        self.args = a
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.rank = int(os.environ.get("RANK", 0))
        local = int(os.environ.get("LOCAL_RANK", 0))
        self.device = torch.device("cuda", local) if a.device == "cuda" else torch.device("cpu")
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        if self.world > 1 and not dist.is_initialized():
            dist.init_process_group("nccl" if self.device.type == "cuda" else "gloo",
                                    timeout=datetime.timedelta(seconds=600))
        self.cfg = self._config()
        self.paths = self._verified_caches()
        cfg = self.cfg
        self.data = PackedBatches(self.paths["train"], world_size=self.world, microbatch=cfg["microbatch"],
                                  accumulation=cfg["accumulation"], context=cfg["context"])
        # the whole schedule must be readable before the first update
        self.data.batch(cfg["updates"] - 1, cfg["accumulation"] - 1, self.world - 1)
        precision = "bf16_gemm_fp32_master" if self.device.type == "cuda" else "cpu_fp32"
        self.identity = {"schema": 1, "condition": a.condition, "config": object_digest(cfg),
                         "data": digest(a.data), "world_size": self.world, "precision": precision}
        self.output = a.output
        self._lock = self._claim_output()
        model, self.shared_digest = initial_model(cfg, a.condition)
        self.parameter_count = sum(p.numel() for p in model.parameters())
        self.model = model.to(self.device)
        if self.device.type == "cpu":  # fp32 GEMM outputs on the CPU oracle path
            for m in self.model.modules():
                if hasattr(m, "out_dtype"):
                    m.out_dtype = None
        self.sync = GradientSynchronizer(self.model)
        self.optimizer = build_optimizer(self.model, a.condition, cfg["conditions"][a.condition]["lr"],
                                         cfg["accumulation"])
        self.store = checkpoint.CheckpointStore(self.output, self.identity)
        self.completed = 0
        self.last_saved = -1

    # -- set-up -------------------------------------------------------------
    def _config(self):
        a = self.args
        cfg = json.loads(a.config.read_text()) if a.config else default_config()
        cfg["world_size"] = self.world
        for key in ("microbatch", "accumulation"):
            if getattr(a, key) is not None:
                cfg[key] = getattr(a, key)
        validate_config(cfg)
        if a.max_hours is not None and a.max_hours * 3600 <= a.checkpoint_margin_seconds:
            raise ValueError("--max-hours leaves no time beyond the checkpoint margin")
        if a.stop_after is not None and not 1 <= a.stop_after <= cfg["updates"]:
            raise ValueError(f"--stop-after must be within 1..{cfg['updates']}")
        return cfg

    def _verified_caches(self):
        manifest = json.loads(self.args.data.read_text())
        if manifest["dtype"] != "<u4":
            raise ValueError(f"token caches must be little-endian uint32, manifest says {manifest['dtype']}")
        paths = {}
        for split in ("train", "validation"):
            entry = manifest["splits"][split]
            p = Path(entry["path"])
            p = p if p.is_absolute() else self.args.data.parent / p
            if self.rank == 0 and (p.stat().st_size != 4 * entry["tokens"] or digest(p) != entry["sha256"]):
                raise RuntimeError(f"{split} cache {p} does not match its manifest entry")
            paths[split] = p
        checkpoint.barrier()
        return paths

    def _claim_output(self):
        """Lock the output directory (rank 0) and record or check the run identity."""
        self.output.mkdir(parents=True, exist_ok=True)
        lock = None
        if self.rank == 0:
            lock = (self.output / "trainer.lock").open("a")
            fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
            recorded = self.output / "identity.json"
            if recorded.exists():
                if not self.args.resume or json.loads(recorded.read_text()) != self.identity:
                    raise RuntimeError(f"{self.output} holds another run; resume it with a matching "
                                       "identity or choose a new output")
            elif self.args.resume:
                raise RuntimeError(f"nothing to resume in {self.output}")
            else:
                atomic_json(recorded, self.identity)
                atomic_json(self.output / "resolved_config.json", self.cfg)
        checkpoint.barrier()
        return lock

    def resume(self):
        spec = self.args.resume
        if not spec:
            return
        manifest = (json.loads((self.output / "latest.json").read_text())["manifest"] if spec == "latest"
                    else spec)
        self.completed = self.store.load(manifest, self.model, self.optimizer,
                                         lambda u: batch_hash(self.data, u, self.rank))
        self.last_saved = self.completed
        if self.rank == 0:
            reconcile_metrics(self.output / "metrics.jsonl", self.completed)
        checkpoint.barrier()

    # -- one update ------------------------------------------------------------
    def update(self):
        cfg, opt, device = self.cfg, self.optimizer, self.device
        accum = cfg["accumulation"]
        opt.zero_grad()
        self.sync.zero_grad()
        if opt.router is not None and (self.completed + 1) % TELEMETRY_EVERY == 0:
            opt.router.set_telemetry_capture(True)
            opt.attention.set_telemetry_capture(True)
        lr = schedule(self.completed, cfg, cfg["conditions"][opt.condition]["lr"])
        for g in opt.param_groups:
            g["lr"] = lr
        tokens = 0
        loss_sum = torch.zeros((), device=device)
        for micro in range(accum):
            x, y, mask = self.data.batch(self.completed, micro, self.rank)
            if not mask.all():
                raise RuntimeError("packed batches must have every target loss-bearing")
            tokens += int(mask.sum())
            loss = self.model.forward_loss(torch.from_numpy(x).to(device), torch.from_numpy(y).to(device))
            if micro + 1 == accum:
                self.sync.begin_backward()  # the last backward's gradients are final
            (loss / accum).backward()
            loss_sum += loss.detach().float() / accum
        self.sync.synchronize()
        counts = torch.tensor([tokens], device=device, dtype=torch.int64)
        if dist.is_initialized():
            dist.all_reduce(counts)
        if int(counts.item()) != cfg["loss_tokens_per_update"]:
            raise RuntimeError(f"{int(counts.item())} loss tokens this update, the config says "
                               f"{cfg['loss_tokens_per_update']}")
        norm = opt.clip_grad_norm()
        seconds = self._timed(opt.step)
        if dist.is_initialized():
            dist.all_reduce(loss_sum)
        loss = float(loss_sum / self.world)
        if not math.isfinite(loss):
            raise RuntimeError(f"training loss became {loss} at update {self.completed + 1}")
        self.completed += 1
        phase = getattr(opt, "phase", "tiller" if opt.router is not None else "baseline")
        return {"loss": loss, "lr": lr, "loss_tokens_this_update": int(counts.item()),
                "gradient_norm": float(norm), "optimizer_seconds": seconds, "phase": phase,
                "optimizer_child_lrs": {role: [g["lr"] for g in child.param_groups]
                                        for role, child in zip(opt.roles, opt.children)}}

    def _timed(self, fn):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        fn()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return time.perf_counter() - t0

    @torch.no_grad()
    def validate(self):
        cfg = self.cfg
        ids = np.memmap(self.paths["validation"], dtype="<u4", mode="r")
        ctx, want = cfg["context"], cfg["small_validation_tokens"]
        if want % ctx or len(ids) <= want:
            raise ValueError(f"validation cache of {len(ids)} tokens cannot give {want} in windows of {ctx}")
        acc = torch.zeros(2, device=self.device, dtype=torch.float64)
        training = self.model.training
        self.model.eval()
        try:
            for w in range(self.rank, want // ctx, self.world):
                window = np.array(ids[w * ctx:(w + 1) * ctx + 1], dtype=np.int64)
                block = torch.from_numpy(window).to(self.device)[None]
                loss = self.model.forward_loss(block[:, :-1], block[:, 1:])
                acc += torch.stack((loss.double() * ctx, loss.new_tensor(ctx).double()))
        finally:
            self.model.train(training)
        if dist.is_initialized():
            dist.all_reduce(acc)
        if int(acc[1]) != want:
            raise RuntimeError(f"validated {int(acc[1])} tokens, expected {want}")
        value = float(acc[0] / acc[1])
        if not math.isfinite(value):
            raise RuntimeError(f"validation loss became {value}")
        return value

    # -- checkpoints -------------------------------------------------------------
    def save(self, kind):
        cfg = self.cfg
        manifest = self.store.save(self.completed, kind, self.model, self.optimizer,
                                   batch_hash(self.data, self.completed, self.rank))
        if self.rank == 0:
            atomic_json(self.output / "latest.json",
                        {"manifest": str(manifest.resolve()), "update": self.completed,
                         "tokens": self.completed * cfg["loss_tokens_per_update"]})
            self.store.prune(cfg["checkpoint_keep_recent"])
        checkpoint.barrier()
        self.last_saved = self.completed

    def _checkpoint_kind(self):
        if self.completed == self.cfg["updates"]:
            return "final"
        if self.args.condition == MHA_SWITCH and self.completed in (C.SWITCH_UPDATE, C.SWITCH_UPDATE + 1):
            return "switch"  # both sides of the TILLER -> Muon hand-off
        if self.completed % self.cfg["checkpoint_every"] == 0:
            return "periodic"
        return None

    def _should_stop(self):
        a = self.args
        by_count = a.stop_after is not None and self.completed >= a.stop_after
        by_time = (a.max_hours is not None and time.monotonic() - self.started
                   >= a.max_hours * 3600 - a.checkpoint_margin_seconds)
        flag = torch.tensor(int(by_count or by_time), device=self.device)
        if dist.is_initialized():
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)  # every rank stops at the same update
        return bool(flag.item())

    def _log(self, record):
        if self.rank != 0:
            return
        line = json.dumps(record, allow_nan=False, default=float)
        with (self.output / "metrics.jsonl").open("a") as fh:
            fh.write(line + "\n")
        print(line, flush=True)

    # -- driver ------------------------------------------------------------------
    def run(self):
        cfg = self.cfg
        if self.rank == 0:
            atomic_json(self.output / "startup.json",
                        {"parameter_count": self.parameter_count,
                         "shared_initial_sha256": self.shared_digest,
                         "resumed_update": self.completed, "identity": self.identity})
        while self.completed < cfg["updates"]:
            t0 = time.perf_counter()
            record = self.update()
            record.update(step=self.completed, loss_tokens=self.completed * cfg["loss_tokens_per_update"],
                          seconds=time.perf_counter() - t0,
                          peak_memory_bytes=(torch.cuda.max_memory_allocated(self.device)
                                             if self.device.type == "cuda" else 0))
            if self.completed % cfg["validation_every"] == 0 or self.completed == cfg["updates"]:
                record["validation_loss"] = self.validate()
            if self.optimizer.router is not None and self.completed % TELEMETRY_EVERY == 0:
                record["tiller_telemetry"] = self.optimizer.router.telemetry()
                record["attention_telemetry"] = self.optimizer.attention.telemetry()
            self._log(record)
            kind = self._checkpoint_kind()
            if kind is not None:
                self.save(kind)
            if self._should_stop():
                break
        if 0 < self.completed != self.last_saved and self.completed != cfg["updates"]:
            self.save("continuation")
        if self.rank == 0:
            atomic_json(self.output / "result.json",
                        {"completed": self.completed == cfg["updates"], "update": self.completed,
                         "loss_tokens": self.completed * cfg["loss_tokens_per_update"],
                         "identity": self.identity})
        checkpoint.barrier()

    def close(self):
        if getattr(self.sync, "communicator", None) is not None:
            self.sync.communicator.close()
        if dist.is_initialized():
            dist.destroy_process_group()


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--condition", required=True, choices=C.CONDITIONS)
    p.add_argument("--data", type=Path, required=True, help="manifest of the local uint32 token caches")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--config", type=Path, default=None)
    p.add_argument("--resume", help="a checkpoint manifest path, or 'latest' under --output")
    p.add_argument("--microbatch", type=int)
    p.add_argument("--accumulation", type=int)
    p.add_argument("--max-hours", type=float, help="wall-time budget of this launch, margin included")
    p.add_argument("--checkpoint-margin-seconds", type=float, default=900)
    p.add_argument("--stop-after", type=int, help="stop (with a checkpoint) after this update")
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    return p.parse_args(argv)


def main(argv=None):
    run = StudyRun(parse_args(argv))
    run.resume()
    try:
        run.run()
    finally:
        run.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
