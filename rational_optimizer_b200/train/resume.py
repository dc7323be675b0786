"""Exact resume: bitwise-continuable checkpoints of a distributed run.

Format (kept identical to the reference so either framework can resume the
other's run; reference training/train.py:2131-2311 and
training/exact_resume.py:25-342):

* ``<path>`` (rank 0, schema ``transformer_lm_exact_resume_v1``): the resume
  contract (17 run-defining fields), completed step, model and optimizer
  state dicts, best validation loss, step/optimizer-step time lists, clipping
  counters, CUDA memory peaks, active seconds;
* ``<path>.rank{r}.pt`` (schema ``transformer_lm_exact_resume_rank_v1``): the
  rank's CPU sampling generator, torch and CUDA RNG states, probe logits.

Commit protocol: every rank writes ``*.tmp``; barrier; ranks rename their
payloads; barrier; rank 0 renames the main payload; barrier.  Strict mode
adds :func:`recover_interrupted_commit`, which promotes the newest
generation that is complete on every rank after a crash mid-commit, and
:func:`prepare_trajectory`, which trims JSONL records past that checkpoint
so replayed steps are not counted twice.

Beyond the reference, :func:`save` writes a SHA-256 manifest of the files of
each generation and :func:`load` verifies it, so a truncated or corrupted
checkpoint is rejected with a message naming the file instead of failing
inside ``torch.load`` or, worse, loading silently.
"""
from __future__ import annotations

import hashlib
import json
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel import param_ready
from ..utils import faults
from .integrity import Manifest

MAIN_SCHEMA = "transformer_lm_exact_resume_v1"
RANK_SCHEMA = "transformer_lm_exact_resume_rank_v1"
STRICT_SCHEMA = "fairness_internal_exact_resume_v1"
CHECKPOINT_BASENAME = "trainer_state.pt"


def rank_path(path: Path, rank: int) -> Path:
    return Path(f"{path}.rank{rank}.pt")


def resume_contract(args, world_size: int, *, strict: bool = False) -> dict:
    contract = {
        "schema": MAIN_SCHEMA, "activation": args.activation, "optimizer": args.optimizer,
        "seed": int(args.seed), "steps": int(args.steps), "world_size": int(world_size),
        "batch_size": int(args.batch_size), "grad_accum": int(args.grad_accum),
        "seq_len": int(args.seq_len), "lr": float(args.lr), "min_lr": float(args.min_lr),
        "warmup_steps": int(args.warmup_steps), "weight_decay": float(args.weight_decay),
        "beta1": float(args.beta1), "beta2": float(args.beta2), "eps": float(args.eps),
        "grad_clip": float(args.grad_clip),
    }
    if strict:
        contract.update({"internal_resume_schema": STRICT_SCHEMA,
                         "fairness_contract": args.fairness_contract,
                         "complete_argument_sha256": complete_argument_digest(args)})
    return contract


def _jsonable(value):
    if isinstance(value, Path):
        return str(value)
    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    if isinstance(value, (list, tuple)):
        return [_jsonable(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _jsonable(v) for k, v in sorted(value.items(), key=lambda kv: str(kv[0]))}
    raise TypeError(f"cannot record a {type(value)!r} in the resume contract")


def complete_argument_digest(args) -> str:
    """SHA-256 of the whole parsed argument namespace (sorted, compact JSON)."""
    payload = {k: _jsonable(v) for k, v in sorted(vars(args).items())}
    return hashlib.sha256(json.dumps(payload, sort_keys=True, separators=(",", ":"),
                                     allow_nan=False).encode("utf-8")).hexdigest()


def full_lr_trace_digest(args) -> str:
    """Digest of ``"{step}:{lr.hex()}\\n"`` over the whole scheduled run."""
    from .engine import learning_rate
    digest = hashlib.sha256()
    for s in range(int(args.steps)):
        lr = learning_rate(s, lr=float(args.lr), min_lr=float(args.min_lr),
                           warmup_steps=int(args.warmup_steps), total_steps=int(args.steps))
        digest.update(f"{s + 1}:{float(lr).hex()}\n".encode("ascii"))
    return digest.hexdigest()


def expected_checkpoint_path(args) -> Path:
    """The only checkpoint location strict mode accepts for ``args``."""
    return (Path(args.output_dir) / args.run_name / ".exact_resume" / CHECKPOINT_BASENAME).resolve()


def _barrier(is_distributed):
    if is_distributed:
        dist.barrier()


def save(path: Path, *, args, rank, world_size, is_distributed, device, model, optimizer,
         train_generator, probe_state, completed_step, best_val_loss, step_times,
         optimizer_step_times, grad_clip_observed_steps, grad_clip_triggered_steps,
         run_cuda_max_memory_allocated, run_cuda_max_memory_reserved, active_seconds,
         strict=False, cpu_probe_state=None):
    param_ready.wait_all()
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    rpath = rank_path(path, rank)
    rtmp = Path(f"{rpath}.tmp")
    if rtmp.exists():
        rtmp.unlink()
    cuda_state = torch.cuda.get_rng_state(device) if device.type == "cuda" else None
    torch.save({"schema": RANK_SCHEMA, "rank": int(rank), "completed_step": int(completed_step),
                "train_generator_state": train_generator.get_state(),
                "torch_rng_state": torch.get_rng_state(), "cuda_rng_state": cuda_state,
                "probe_state": cpu_probe_state(probe_state) if cpu_probe_state else None}, rtmp)
    mtmp = Path(f"{path}.tmp")
    # every rank takes part: a layer-sharded optimizer completes its state collectively
    optimizer_state = optimizer.state_dict()
    if rank == 0:
        if mtmp.exists():
            mtmp.unlink()
        raw = model.module if hasattr(model, "module") else model
        torch.save({
            "schema": MAIN_SCHEMA, "contract": resume_contract(args, world_size, strict=strict),
            "completed_step": int(completed_step), "model": raw.state_dict(),
            "optimizer": optimizer_state, "best_val_loss": float(best_val_loss),
            "step_times": list(step_times), "optimizer_step_times": list(optimizer_step_times),
            "grad_clip_observed_steps": int(grad_clip_observed_steps),
            "grad_clip_triggered_steps": int(grad_clip_triggered_steps),
            "run_cuda_max_memory_allocated": int(run_cuda_max_memory_allocated),
            "run_cuda_max_memory_reserved": int(run_cuda_max_memory_reserved),
            "active_seconds": float(active_seconds),
        }, mtmp)
    faults.maybe_inject("checkpoint_written", rank, completed_step)
    if rank == 0:
        # the manifest describes one generation: drop the old one before any of
        # its files is replaced, write the new one after the last promotion
        Manifest.path_for(path).unlink(missing_ok=True)
    _barrier(is_distributed)
    rtmp.replace(rpath)
    _barrier(is_distributed)
    if rank == 0:
        mtmp.replace(path)
    faults.maybe_inject("checkpoint_promoted", rank, completed_step)
    if rank == 0:
        Manifest.write(path, [path] + [rank_path(path, r) for r in range(int(world_size))])
    _barrier(is_distributed)


def load(path: Path, *, args, rank, world_size, is_distributed, device, model, optimizer,
         train_generator, probe_state, strict=False):
    """Restore everything :func:`save` wrote; None when no checkpoint exists yet."""
    param_ready.wait_all()
    path = Path(path).resolve()
    if strict:
        if int(rank) == 0:
            recover_interrupted_commit(path, int(world_size))
        _barrier(is_distributed)
    if not path.is_file():
        return None
    rpath = rank_path(path, rank)
    if not rpath.is_file():
        raise RuntimeError(f"missing exact-resume rank state: {rpath}")
    if Manifest.path_for(path).is_file():
        Manifest.verify(path, [path.name, rpath.name])
    payload = torch.load(path, map_location="cpu", weights_only=False)
    rpayload = torch.load(rpath, map_location="cpu", weights_only=False)
    if (payload.get("schema") != MAIN_SCHEMA
            or payload.get("contract") != resume_contract(args, world_size, strict=strict)
            or rpayload.get("schema") != RANK_SCHEMA or rpayload.get("rank") != rank
            or rpayload.get("completed_step") != payload.get("completed_step")):
        raise RuntimeError("checkpoint contract differs from this run (schema, rank or step)")
    raw = model.module if hasattr(model, "module") else model
    raw.load_state_dict(payload["model"])
    optimizer.load_state_dict(payload["optimizer"])
    train_generator.set_state(rpayload["train_generator_state"])
    torch.set_rng_state(rpayload["torch_rng_state"])
    if device.type == "cuda" and rpayload.get("cuda_rng_state") is not None:
        torch.cuda.set_rng_state(rpayload["cuda_rng_state"], device)
    stored = rpayload.get("probe_state")
    if probe_state is not None and stored is not None:
        for key in ("first_logits", "prev_logits"):
            v = stored.get(key)
            probe_state[key] = None if v is None else v.to(device=device)
    _barrier(is_distributed)
    return payload


def _stored_step(path: Path, schema: str):
    if not path.is_file():
        return None
    try:
        payload = torch.load(path, map_location="cpu", weights_only=False)
    except Exception:
        return None
    if not isinstance(payload, dict) or payload.get("schema") != schema:
        return None
    try:
        return int(payload["completed_step"])
    except (KeyError, TypeError, ValueError):
        return None


def recover_interrupted_commit(path: Path, world_size: int):
    """Promote the newest checkpoint generation complete on every rank.

    A crash during :func:`save` can leave any mix of stable and ``.tmp``
    files.  A generation (main payload, stable or temporary) counts only if
    every rank has a readable payload, stable or temporary, with the same
    completed step.  Returns that step, or None when no generation is complete.
    """
    path = Path(path).resolve()
    complete = []
    for main in (path, Path(f"{path}.tmp")):
        step = _stored_step(main, MAIN_SCHEMA)
        if step is None:
            continue
        choices = []
        for r in range(int(world_size)):
            stable = rank_path(path, r)
            pick = next((c for c in (stable, Path(f"{stable}.tmp"))
                         if _stored_step(c, RANK_SCHEMA) == step), None)
            if pick is None:
                choices = []
                break
            choices.append(pick)
        if len(choices) == int(world_size):
            complete.append((step, main, choices))
    if not complete:
        return None
    step, main, ranks = max(complete, key=lambda item: item[0])
    path.parent.mkdir(parents=True, exist_ok=True)
    for r, source in enumerate(ranks):
        if source != rank_path(path, r):
            os.replace(source, rank_path(path, r))
    if main != path:
        os.replace(main, path)
    if Manifest.path_for(path).is_file():
        # the manifest belongs to the generation it was written with; rewrite it
        Manifest.write(path, [path] + [rank_path(path, r) for r in range(int(world_size))])
    return int(step)


def prepare_trajectory(checkpoint_path: Path, trajectory_path: Path, world_size: int) -> dict:
    """Make an append-only JSONL trajectory consistent with its last durable checkpoint."""
    checkpoint_path = Path(checkpoint_path).resolve()
    trajectory_path = Path(trajectory_path).resolve()
    step = recover_interrupted_commit(checkpoint_path, int(world_size))
    if not trajectory_path.is_file() or trajectory_path.stat().st_size == 0:
        return {"schema": STRICT_SCHEMA, "mode": "fresh", "completed_step": step}
    lines = trajectory_path.read_text(encoding="utf-8").splitlines()
    if step is None:
        archive = trajectory_path.with_name(
            f"{trajectory_path.name}.orphaned-before-first-checkpoint-{time.time_ns()}")
        os.replace(trajectory_path, archive)
        return {"schema": STRICT_SCHEMA, "mode": "fresh_after_archiving_uncheckpointed_partial",
                "completed_step": None, "archive": str(archive)}
    kept, removed, configs = [], [], 0
    for line in lines:
        try:
            rec = json.loads(line)
        except json.JSONDecodeError as error:
            raise RuntimeError(f"unreadable line in the trajectory being trimmed for resume: {error}") from error
        event = rec.get("event")
        configs += event == "config"
        rs = rec.get("step")
        keep = event not in {"summary", "checkpoint", "stopped_early"} and (rs is None or int(rs) <= int(step))
        (kept if keep else removed).append(line)
    if configs != 1:
        raise RuntimeError(f"the trajectory holds {configs} config records; a resumable one holds one")
    if not any(int(json.loads(l).get("step", -1)) == int(step) for l in kept):
        raise RuntimeError(f"the trajectory has no record at the checkpoint's step {int(step)}")
    archive = None
    if removed:
        archive = trajectory_path.with_name(f"{trajectory_path.name}.tail-after-step-{step}-{time.time_ns()}")
        archive.write_text("\n".join(lines) + "\n", encoding="utf-8")
        tmp = Path(f"{trajectory_path}.resume.tmp")
        tmp.write_text("\n".join(kept) + "\n", encoding="utf-8")
        os.replace(tmp, trajectory_path)
    return {"schema": STRICT_SCHEMA, "mode": "resume", "completed_step": int(step),
            "removed_records": len(removed), "archive": None if archive is None else str(archive)}


def validate_strict(args):
    """Strict mode: the run-local checkpoint path and an interval equal to eval_interval."""
    if args.resume_checkpoint is None:
        return
    if Path(args.resume_checkpoint).resolve() != expected_checkpoint_path(args):
        raise ValueError(f"strict resume reads only the run-local checkpoint {expected_checkpoint_path(args)}")
    interval = int(args.resume_checkpoint_interval)
    if interval <= 0 or interval != int(args.eval_interval):
        raise ValueError("strict resume saves at the evaluation interval, which must be positive")


def audited_summary(record, args):
    """After a strict resume the summary's LR audit covers the whole run."""
    if not isinstance(record, dict) or record.get("event") != "summary" or args.resume_checkpoint is None:
        return record
    out = dict(record)
    out["realized_lr_audit_steps"] = int(args.steps)
    out["realized_lr_trace_sha256"] = full_lr_trace_digest(args)
    out["realized_lr_trace_reconstructed_after_exact_resume"] = True
    return out


def _main():
    import argparse
    parser = argparse.ArgumentParser(description="Trim a run's JSONL to its last durable checkpoint")
    parser.add_argument("--checkpoint", required=True, type=Path)
    parser.add_argument("--trajectory", required=True, type=Path)
    parser.add_argument("--world-size", required=True, type=int)
    a = parser.parse_args()
    print(json.dumps(prepare_trajectory(a.checkpoint, a.trajectory, a.world_size), sort_keys=True), flush=True)


if __name__ == "__main__":
    _main()
