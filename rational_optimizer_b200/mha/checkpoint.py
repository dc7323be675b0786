"""Checkpoint store of the MHA study: atomic, checksum-verified, one per completed update.

Same on-disk format as experiments/mha_1b_tokens/checkpoint.py:1-83, so
either implementation can resume the other's runs:

    <output>/checkpoint-{update:06d}-{kind}/
        model.pt          model state dict (written by rank 0)
        rank-{r}.pt       {"optimizer", "rng", "update", "data_position",
                           "next_batch_hash", "identity"} of rank r
        manifest.json     {"schema": 1, "update", "identity",
                           "artifacts": {file name: sha256}, "world_size"}

:class:`CheckpointStore` stages a checkpoint in ``<name>.partial``; every
artifact is hashed while it is written, read back and re-hashed before the
manifest is trusted, and the directory is renamed into place last (then the
parent directory is fsynced), so an interrupted save leaves either a complete
checkpoint or only a ``.partial`` directory.  Loading re-checks the
manifest's inventory, the run identity, the world size, every checksum, the
optimizer's update counter and that the next batch is the one the
interrupted run would have read.  ``prune`` keeps the newest ``keep``
periodic checkpoints; milestone (switch, continuation) and final
checkpoints are never removed.
"""
from __future__ import annotations

import hashlib
import json
import os
import random
import re
import shutil
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from .data import atomic_json, digest

SCHEMA = 1
_PERIODIC = re.compile(r"checkpoint-(\d+)-periodic")


def _dist():
    """(rank, world size) of the default process group, (0, 1) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


@dataclass
class RngState:
    """Host and device random-generator states of one process."""

    python: object
    numpy: object
    torch: torch.Tensor
    cuda: torch.Tensor | None

    @classmethod
    def capture(cls):
        return cls(random.getstate(), np.random.get_state(), torch.get_rng_state(),
                   torch.cuda.get_rng_state() if torch.cuda.is_available() else None)

    def as_dict(self):
        return {"python": self.python, "numpy": self.numpy, "torch": self.torch, "cuda": self.cuda}

    @staticmethod
    def restore(saved):
        random.setstate(saved["python"])
        np.random.set_state(saved["numpy"])
        torch.set_rng_state(saved["torch"])
        if saved["cuda"] is not None and torch.cuda.is_available():
            torch.cuda.set_rng_state(saved["cuda"])


# kept for callers of the functional interface
def capture_rng():
    return RngState.capture().as_dict()


def restore_rng(state):
    RngState.restore(state)


class _HashingWriter:
    """File object that fsyncs on close and hashes every byte written through it."""

    def __init__(self, path: Path):
        self._fh = path.open("xb")  # never overwrite an artifact
        self.sha = hashlib.sha256()

    def write(self, data):
        self.sha.update(data)
        return self._fh.write(data)

    def flush(self):
        self._fh.flush()

    def close(self):
        self._fh.flush()
        os.fsync(self._fh.fileno())
        self._fh.close()


def _fsync_dir(path: Path):
    fd = os.open(path, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


class CheckpointStore:
    """Checkpoints of one run (``identity``) under ``root``."""

    def __init__(self, root, identity):
        self.root = Path(root)
        self.identity = identity

    def path(self, update, kind):
        return self.root / f"checkpoint-{int(update):06d}-{kind}"

    # -- save ----------------------------------------------------------------
    def save(self, update, kind, model, optimizer, next_batch_hash):
        """Write the checkpoint of completed ``update`` on every rank; returns its manifest path."""
        rank, world = _dist()
        final = self.path(update, kind)
        staging = final.with_name(final.name + ".partial")
        if rank == 0:
            for p in (final, staging):
                if p.exists():
                    raise RuntimeError(f"{p} exists; checkpoints are never overwritten")
            staging.mkdir(parents=True)
        barrier()
        written = {}
        if rank == 0:
            written["model.pt"] = self._write(staging / "model.pt", model.state_dict())
        payload = {"optimizer": optimizer.state_dict(), "rng": RngState.capture().as_dict(),
                   "update": update, "data_position": update, "next_batch_hash": next_batch_hash,
                   "identity": self.identity}
        self._write(staging / f"rank-{rank}.pt", payload)
        barrier()
        if rank == 0:
            # the other ranks' files are hashed from disk, ours as they were written
            artifacts = {p.name: written.get(p.name) or digest(p) for p in sorted(staging.glob("*.pt"))}
            atomic_json(staging / "manifest.json", {"schema": SCHEMA, "update": update,
                                                    "identity": self.identity, "artifacts": artifacts,
                                                    "world_size": world})
            bad = [n for n, h in artifacts.items() if digest(staging / n) != h]
            if bad:
                raise RuntimeError(f"checkpoint read-back differs from what was written: {bad}")
            os.rename(staging, final)
            _fsync_dir(final.parent)
        barrier()
        return final / "manifest.json"

    @staticmethod
    def _write(path, value):
        out = _HashingWriter(path)
        try:
            torch.save(value, out)
        finally:
            out.close()
        return out.sha.hexdigest()

    # -- load ----------------------------------------------------------------
    def load(self, manifest_path, model, optimizer, next_hash_fn):
        """Restore model, optimizer and RNG from a verified checkpoint; returns its update."""
        rank, world = _dist()
        manifest_path = Path(manifest_path)
        folder = manifest_path.parent
        meta = json.loads(manifest_path.read_text())
        inventory = {"model.pt"} | {f"rank-{r}.pt" for r in range(world)}
        if meta.get("schema") != SCHEMA or set(meta.get("artifacts", {})) != inventory:
            raise RuntimeError(f"{folder}: not a schema-{SCHEMA} checkpoint for {world} ranks")
        if meta["identity"] != self.identity:
            raise RuntimeError(f"{folder} belongs to a run with another source/config/data/schedule")
        if meta["world_size"] != world:
            raise RuntimeError(f"{folder} was written by {meta['world_size']} ranks, not {world}")
        update = meta["update"]
        if rank == 0:
            bad = [n for n, h in meta["artifacts"].items() if digest(folder / n) != h]
            if bad:
                raise RuntimeError(f"{folder}: checksum mismatch in {bad}")
        barrier()
        model.load_state_dict(torch.load(folder / "model.pt", map_location="cpu", weights_only=False))
        mine = torch.load(folder / f"rank-{rank}.pt", map_location="cpu", weights_only=False)
        if (mine["identity"] != self.identity or mine["update"] != update
                or mine["data_position"] != update):
            raise RuntimeError(f"{folder}: rank {rank}'s payload is from another run or position")
        if mine["optimizer"]["completed_steps"] != update:
            raise RuntimeError(f"{folder}: optimizer counted {mine['optimizer']['completed_steps']} "
                               f"updates, the manifest {update}")
        optimizer.load_state_dict(mine["optimizer"])
        if mine["next_batch_hash"] != next_hash_fn(update):
            raise RuntimeError(f"{folder}: the data would not continue where the run stopped")
        RngState.restore(mine["rng"])
        barrier()
        return update

    # -- retention -------------------------------------------------------------
    def prune(self, keep=2):
        """Remove all but the newest ``keep`` (>= 2) periodic checkpoints of this run."""
        if type(keep) is not int or keep < 2:
            raise ValueError(f"keep must be an int >= 2, got {keep!r}")
        periodic = []
        for path in self.root.glob("checkpoint-*-periodic"):
            m = _PERIODIC.fullmatch(path.name)
            manifest = path / "manifest.json"
            if m is None or path.is_symlink() or not path.is_dir() or not manifest.exists():
                continue
            if json.loads(manifest.read_text()).get("identity") != self.identity:
                raise RuntimeError(f"{path} belongs to another run; not pruning")
            periodic.append((int(m.group(1)), path))
        periodic.sort()
        for _, path in periodic[: max(0, len(periodic) - keep)]:
            shutil.rmtree(path)


# functional interface (the trainer and tests use the store through these)
def save(directory, model, optimizer, update, identity, next_batch_hash):
    directory = Path(directory)
    m = re.fullmatch(r"checkpoint-(\d+)-(\w+)", directory.name)
    if m is None or int(m.group(1)) != int(update):
        raise ValueError(f"checkpoint directory name {directory.name!r} does not encode update {update}")
    return CheckpointStore(directory.parent, identity).save(update, m.group(2), model, optimizer,
                                                            next_batch_hash)


def load(manifest_path, model, optimizer, identity, next_hash_fn):
    return CheckpointStore(Path(manifest_path).parent.parent, identity).load(
        manifest_path, model, optimizer, next_hash_fn)


def prune_periodic(directory, identity, keep=2):
    CheckpointStore(directory, identity).prune(keep)


def rank() -> int:
    return _dist()[0]


def world() -> int:
    return _dist()[1]
