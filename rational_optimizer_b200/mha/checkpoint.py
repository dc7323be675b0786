"""Atomic, checksum-verified checkpoints at completed update boundaries
(reference experiments/mha_1b_tokens/checkpoint.py:1-83).

Layout: ``checkpoint-{update:06d}-{kind}/`` with ``model.pt`` (rank 0),
``rank-{r}.pt`` (optimizer state, RNG states, data position, hash of the
next batch, run identity) and ``manifest.json`` (schema 1, update, identity,
SHA-256 of every artifact, world size).  The directory is written as
``*.partial`` and renamed only after every artifact is read back and
verified, so a crash leaves either a complete checkpoint or none.  Loading
re-verifies checksums, identity, world size, the optimizer's update counter
and that the next batch is the one the interrupted run would have read.
Periodic checkpoints beyond the most recent ``keep`` are pruned; milestone
and final checkpoints are never removed.
"""
from __future__ import annotations

import json
import os
import random
import re
import shutil
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from .data import atomic_json, digest


def rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def world() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def barrier():
    if dist.is_initialized():
        dist.barrier()


def capture_rng():
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state() if torch.cuda.is_available() else None}


def restore_rng(state):
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"])
    if state["cuda"] is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"])


def _write_torch(path: Path, value):
    with path.open("xb") as fh:
        torch.save(value, fh)
        fh.flush()
        os.fsync(fh.fileno())


def prune_periodic(directory, identity, keep=2):
    if type(keep) is not int or keep < 2:
        raise ValueError("retain at least two periodic checkpoints")
    found = []
    for path in Path(directory).glob("checkpoint-*-periodic"):
        m = re.fullmatch(r"checkpoint-(\d+)-periodic", path.name)
        if not m or path.is_symlink() or not path.is_dir() or not (path / "manifest.json").exists():
            continue
        if json.loads((path / "manifest.json").read_text()).get("identity") != identity:
            raise RuntimeError("refuse to prune another checkpoint identity")
        found.append((int(m[1]), path))
    for _, path in sorted(found)[:-keep]:
        shutil.rmtree(path)


def save(directory, model, optimizer, update, identity, next_batch_hash):
    directory = Path(directory)
    partial = directory.with_name(directory.name + ".partial")
    if rank() == 0:
        if directory.exists() or partial.exists():
            raise RuntimeError("checkpoint target already exists")
        partial.mkdir(parents=True)
    barrier()
    if rank() == 0:
        _write_torch(partial / "model.pt", model.state_dict())
    _write_torch(partial / f"rank-{rank()}.pt", {
        "optimizer": optimizer.state_dict(), "rng": capture_rng(), "update": update, "data_position": update,
        "next_batch_hash": next_batch_hash, "identity": identity})
    barrier()
    if rank() == 0:
        artifacts = {p.name: digest(p) for p in sorted(partial.glob("*.pt"))}
        atomic_json(partial / "manifest.json", {"schema": 1, "update": update, "identity": identity,
                                                "artifacts": artifacts, "world_size": world()})
        for name, expected in artifacts.items():
            if digest(partial / name) != expected:
                raise RuntimeError("checkpoint readback checksum failure")
        os.rename(partial, directory)
        fd = os.open(directory.parent, os.O_RDONLY)
        try:
            os.fsync(fd)
        finally:
            os.close(fd)
    barrier()
    return directory / "manifest.json"


def load(manifest_path, model, optimizer, identity, next_hash_fn):
    manifest_path = Path(manifest_path)
    meta = json.loads(manifest_path.read_text())
    directory = manifest_path.parent
    expected = {"model.pt"} | {f"rank-{i}.pt" for i in range(world())}
    if meta.get("schema") != 1 or set(meta.get("artifacts", {})) != expected:
        raise RuntimeError("checkpoint schema/artifact inventory mismatch")
    if meta["identity"] != identity:
        raise RuntimeError("checkpoint source/config/data/schedule identity differs")
    if meta["world_size"] != world():
        raise RuntimeError("checkpoint world size differs")
    if rank() == 0:
        for name, want in meta["artifacts"].items():
            if digest(directory / name) != want:
                raise RuntimeError("checkpoint artifact checksum mismatch")
    barrier()
    model.load_state_dict(torch.load(directory / "model.pt", map_location="cpu", weights_only=False))
    state = torch.load(directory / f"rank-{rank()}.pt", map_location="cpu", weights_only=False)
    if state["identity"] != identity or state["update"] != meta["update"] or state["data_position"] != meta["update"]:
        raise RuntimeError("rank checkpoint identity/position differs")
    if state["optimizer"]["completed_steps"] != meta["update"]:
        raise RuntimeError("optimizer/data update count mismatch")
    optimizer.load_state_dict(state["optimizer"])
    if state["next_batch_hash"] != next_hash_fn(meta["update"]):
        raise RuntimeError("next batch changed across resume")
    restore_rng(state["rng"])
    barrier()
    return meta["update"]
