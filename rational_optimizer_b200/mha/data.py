"""Document splits and packed uint32 token caches (reference
experiments/mha_1b_tokens/data.py:1-73, io.py).

The formats are kept as published: documents are assigned to
train/validation/test by a SHA-256 bucket of their normalised text, caches
are little-endian uint32 arrays with a JSON manifest (dtype, tokens, sha256,
vocab_size), and :class:`PackedBatches` maps (update, micro-step, rank) to
disjoint consecutive context windows so every update reads fresh tokens and
a resumed run reads exactly what an uninterrupted run would.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import tempfile
import unicodedata
from pathlib import Path

import numpy as np

NORMALIZATION = "NFKC+casefold+unicode-whitespace-v1"


def atomic_json(path, value):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix="." + path.name, dir=path.parent)
    try:
        with os.fdopen(fd, "w") as fh:
            json.dump(value, fh, indent=2, sort_keys=True, allow_nan=False)
            fh.write("\n")
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)
        dfd = os.open(path.parent, os.O_RDONLY)
        try:
            os.fsync(dfd)
        finally:
            os.close(dfd)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def digest(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as fh:
        for chunk in iter(lambda: fh.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def object_digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"),
                                     allow_nan=False).encode()).hexdigest()


def normalized(text: str) -> str:
    return " ".join(unicodedata.normalize("NFKC", text).casefold().split())


def document_id(text: str) -> str:
    return hashlib.sha256(normalized(text).encode("utf-8")).hexdigest()


def split_for(text: str) -> str:
    bucket = int(document_id(text)[:16], 16) % 10000
    return "validation" if bucket < 20 else "test" if bucket < 70 else "train"


def word_ngrams(text: str, n: int = 13) -> set:
    words = re.findall(r"\w+", normalized(text))
    return {" ".join(words[i:i + n]) for i in range(max(0, len(words) - n + 1))}


def overlaps(text: str, benchmark_ngrams: set) -> bool:
    return bool(word_ngrams(text) & benchmark_ngrams)


def write_cache(path, ids, *, vocab_size: int) -> dict:
    """Write an immutable uint32 cache, verify the round trip, then its manifest."""
    path = Path(path)
    ids = np.asarray(ids)
    if ids.ndim != 1 or ids.dtype.kind not in "iu" or np.any(ids < 0) or np.any(ids >= vocab_size):
        raise ValueError("invalid integer token IDs")
    path.parent.mkdir(parents=True, exist_ok=True)
    partial = path.with_suffix(path.suffix + ".partial")
    with partial.open("xb") as fh:
        ids.astype("<u4").tofile(fh)
        fh.flush()
        os.fsync(fh.fileno())
    if not np.array_equal(ids, np.fromfile(partial, dtype="<u4")):
        raise RuntimeError("uint32 round trip failed")
    if path.exists():
        raise FileExistsError("immutable cache already exists")
    partial.rename(path)
    manifest = {"dtype": "<u4", "tokens": int(len(ids)), "sha256": digest(path), "vocab_size": int(vocab_size)}
    atomic_json(path.with_suffix(path.suffix + ".json"), manifest)
    return manifest


class PackedBatches:
    """Every update owns consecutive disjoint targets; windows overlap by one input token.

    Sequence i reads tokens [i*context, (i+1)*context] (context + 1 tokens)
    giving context input/target pairs; the first sequence of (update,
    micro-step, rank) is ((update * accum + micro) * world + rank) * micro.
    """

    def __init__(self, path, *, world_size=4, microbatch=8, accumulation=4, context=2048):
        if min(world_size, microbatch, accumulation, context) < 1:
            raise ValueError("invalid batch geometry")
        self.tokens = np.memmap(path, dtype="<u4", mode="r")
        self.world, self.micro, self.accum, self.context = world_size, microbatch, accumulation, context
        self.loss_tokens = world_size * microbatch * accumulation * context

    def batch(self, update, microstep, rank):
        if update < 0 or not 0 <= microstep < self.accum or not 0 <= rank < self.world:
            raise ValueError("invalid data position")
        first = ((update * self.accum + microstep) * self.world + rank) * self.micro
        starts = (first + np.arange(self.micro, dtype=np.int64)) * self.context
        if starts[-1] + self.context >= len(self.tokens):
            raise IndexError("cache exhausted; replay forbidden")
        block = np.asarray(self.tokens[starts[:, None] + np.arange(self.context + 1, dtype=np.int64)], dtype=np.int64)
        return block[:, :-1].copy(), block[:, 1:].copy(), np.ones((self.micro, self.context), dtype=bool)


def whole_updates(target=12_000_000_000, batch=262144):
    updates = (target + batch // 2) // batch
    return updates, updates * batch
