"""Content hashes that bind runs, caches and checkpoints to their inputs.

Digests are defined exactly as the reference trainer defines them
(training/train.py:794-842), so a run of either framework can be checked
against the other's records:

* :func:`tensor_content_sha256` - SHA-256 of a tensor's logical bytes,
  streamed in chunks (token caches);
* :func:`tensor_sample_sha256` - shape, dtype, count and the first/last
  ``sample_count`` values (cheap fingerprints of large arrays);
* :func:`model_state_sha256` - every state-dict entry's name, shape, dtype and
  bytes in order (initial-state identity);
* :func:`sampled_start_fingerprint` - the batch start indices a seed draws.

:func:`file_sha256` and :class:`Manifest` add what the reference lacks: a
per-file manifest written next to a checkpoint so a corrupted or truncated
file is detected before it is loaded.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import torch


def tensor_content_sha256(tensor, chunk_bytes: int = 64 * 1024 * 1024) -> str:
    if not torch.is_tensor(tensor):
        raise TypeError("tensor_content_sha256 expects a tensor")
    if int(chunk_bytes) <= 0:
        raise ValueError("chunk_bytes must be positive")
    raw = tensor.detach().cpu().contiguous().view(torch.uint8).reshape(-1).numpy()
    view = memoryview(raw)
    digest = hashlib.sha256()
    for start in range(0, view.nbytes, int(chunk_bytes)):
        digest.update(view[start:start + int(chunk_bytes)])
    return digest.hexdigest()


def tensor_sample_sha256(tensor, sample_count: int = 4096) -> str:
    flat = tensor.detach().reshape(-1).cpu()
    count = min(int(sample_count), int(flat.numel()))
    digest = hashlib.sha256()
    digest.update(str(tuple(flat.shape)).encode("ascii"))
    digest.update(str(flat.dtype).encode("ascii"))
    digest.update(str(int(flat.numel())).encode("ascii"))
    if count > 0:
        digest.update(flat[:count].contiguous().numpy().tobytes())
        digest.update(flat[-count:].contiguous().numpy().tobytes())
    return digest.hexdigest()


def model_state_sha256(model) -> str:
    digest = hashlib.sha256()
    for name, value in model.state_dict().items():
        t = value.detach().cpu().contiguous()
        digest.update(name.encode("utf-8"))
        digest.update(str(tuple(t.shape)).encode("ascii"))
        digest.update(str(t.dtype).encode("ascii"))
        digest.update(t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                      else t.numpy().tobytes())
    return digest.hexdigest()


def sampled_start_fingerprint(token_count, seq_len, batch_size, draws, seed) -> str:
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed))
    starts = torch.randint(int(token_count) - int(seq_len) - 1, (int(draws), int(batch_size)),
                           generator=gen)
    return tensor_sample_sha256(starts, sample_count=starts.numel())


def file_sha256(path, chunk_bytes: int = 16 * 1024 * 1024) -> str:
    digest = hashlib.sha256()
    with open(path, "rb") as fh:
        while True:
            block = fh.read(chunk_bytes)
            if not block:
                break
            digest.update(block)
    return digest.hexdigest()


class Manifest:
    """``{file name: {bytes, sha256}}`` for the files of one checkpoint generation."""

    SCHEMA = "rational_optimizer_b200_manifest_v1"

    @staticmethod
    def path_for(checkpoint: Path) -> Path:
        return Path(f"{checkpoint}.manifest.json")

    @classmethod
    def write(cls, checkpoint: Path, files) -> Path:
        entries = {}
        for f in files:
            f = Path(f)
            entries[f.name] = {"bytes": f.stat().st_size, "sha256": file_sha256(f)}
        target = cls.path_for(checkpoint)
        tmp = Path(f"{target}.tmp")
        with open(tmp, "w", encoding="utf-8") as fh:
            json.dump({"schema": cls.SCHEMA, "files": entries}, fh, sort_keys=True)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, target)
        return target

    @classmethod
    def verify(cls, checkpoint: Path, names=None) -> dict:
        """Raise ``RuntimeError`` naming the first missing, truncated or altered file."""
        target = cls.path_for(checkpoint)
        if not target.is_file():
            raise RuntimeError(f"checkpoint manifest missing: {target}")
        payload = json.loads(target.read_text(encoding="utf-8"))
        if payload.get("schema") != cls.SCHEMA:
            raise RuntimeError(f"unknown checkpoint manifest schema in {target}")
        files = payload["files"]
        for name in (names if names is not None else files):
            if name not in files:
                raise RuntimeError(f"{name} is not listed in {target}")
            f = Path(checkpoint).parent / name
            if not f.is_file():
                raise RuntimeError(f"checkpoint file missing: {f}")
            if f.stat().st_size != files[name]["bytes"]:
                raise RuntimeError(f"checkpoint file truncated or grown: {f}")
            if file_sha256(f) != files[name]["sha256"]:
                raise RuntimeError(f"checkpoint file content differs from its manifest: {f}")
        return files
