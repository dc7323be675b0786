"""Token sources for the trainer: the on-disk token cache, offline synthetic
corpora, and tokenization.

Cache format (kept identical to the reference so caches are shared; reference
training/train.py:355-394, 590-782): one ``torch.save`` payload per split with
``schema = "rationalopt_token_cache_v2"``, a contiguous int32 ``tokens`` tensor,
``token_count``, ``token_content_sha256`` and the metadata fields of
:func:`cache_metadata`.  :func:`load_cached_tokens` rejects a payload whose
metadata, dtype, count, hash format or length disagrees with the request.

Sources:

* ``synthetic/{arithmetic,code,symbolic,reasoning_mix}`` - deterministic
  procedurally generated text (the same strings the reference generates, so
  the token streams match for the same tokenizer);
* ``synthetic/zipf`` and ``synthetic/uniform`` - token ids drawn directly
  (benchmark data; no tokenizer involved);
* any other name - a Hugging Face dataset through ``datasets.load_dataset``
  (needs network access or a populated ``--hf-cache``).

Tokenizers: a Hugging Face tokenizer name (``gpt2`` by default), or
``bytes`` - UTF-8 bytes with id 256 as end-of-document, which needs no files.
"""
from __future__ import annotations

import fcntl
import os
import re
from array import array
from pathlib import Path

import numpy as np
import torch

from .data import uniform_tokens, zipf_tokens
from .integrity import tensor_content_sha256

CACHE_SCHEMA = "rationalopt_token_cache_v2"
SPLIT_OFFSETS = {"train": 0, "validation": 50_000_000, "test": 75_000_000}
DIRECT_SOURCES = {"synthetic/zipf", "synthetic/uniform"}


def sanitize_name(name) -> str:
    return "".join(ch if ch.isalnum() else "_" for ch in str(name))


def actual_dataset_split(args, split):
    return {"train": args.train_split, "validation": args.validation_split}.get(split, split)


def dataset_skip_documents(args, split):
    key = {"train": "train_skip_documents", "validation": "validation_skip_documents"}.get(split)
    return max(0, int(getattr(args, key))) if key else 0


def dataset_skip_tokens(args, split):
    key = {"train": "train_skip_tokens", "validation": "validation_skip_tokens"}.get(split)
    return max(0, int(getattr(args, key))) if key else 0


def token_cache_path(args, split, max_tokens) -> Path:
    """Cache file name; the short legacy form is used when every option is at its default."""
    cache_dir = Path(args.cache_dir)
    cache_dir.mkdir(parents=True, exist_ok=True)
    max_part = "all" if max_tokens is None else str(max_tokens)
    config = args.dataset_config if args.dataset_config else "none"
    actual = actual_dataset_split(args, split)
    skip_docs = dataset_skip_documents(args, split)
    skip_toks = dataset_skip_tokens(args, split)
    revision = ""
    if args.dataset_revision is not None or args.tokenizer_revision is not None:
        revision = (f"_dsrev{sanitize_name(args.dataset_revision or 'default')}"
                    f"_tokrev{sanitize_name(args.tokenizer_revision or 'default')}")
    stem = f"{sanitize_name(args.dataset_name)}_{sanitize_name(config)}_{sanitize_name(args.tokenizer)}"
    legacy = (not args.dataset_streaming and args.dataset_text_column == "text" and actual == split
              and skip_docs == 0 and skip_toks == 0 and args.train_split == "train"
              and args.validation_split == "validation" and not revision)
    if legacy:
        return cache_dir / f"{stem}_{split}_{max_part}.pt"
    mode = "stream" if args.dataset_streaming else "map"
    return cache_dir / (f"{stem}_{sanitize_name(actual)}_{split}_{mode}_"
                        f"{sanitize_name(args.dataset_text_column)}_skipdocs{skip_docs}_"
                        f"skiptoks{skip_toks}{revision}_{max_part}.pt")


def cache_metadata(args, split) -> dict:
    return {
        "dataset": args.dataset_name,
        "dataset_config": args.dataset_config,
        "dataset_revision": args.dataset_revision,
        "split": split,
        "actual_split": actual_dataset_split(args, split),
        "dataset_streaming": args.dataset_streaming,
        "dataset_text_column": args.dataset_text_column,
        "skip_documents": dataset_skip_documents(args, split),
        "skip_tokens": dataset_skip_tokens(args, split),
        "tokenizer": args.tokenizer,
        "tokenizer_revision": args.tokenizer_revision,
    }


def load_cached_tokens(cache_file, args, split, max_tokens) -> torch.Tensor:
    payload = torch.load(cache_file, map_location="cpu", weights_only=False)
    if not isinstance(payload, dict) or not torch.is_tensor(payload.get("tokens")):
        raise RuntimeError(f"invalid token cache payload: {cache_file}")
    tokens = payload["tokens"]
    bad = {k: {"observed": payload.get(k), "required": v}
           for k, v in cache_metadata(args, split).items() if payload.get(k) != v}
    checks = [
        ("schema", payload.get("schema"), CACHE_SCHEMA, payload.get("schema") == CACHE_SCHEMA),
        ("dtype", str(tokens.dtype), str(torch.int32), tokens.dtype == torch.int32),
        ("payload_token_count", payload.get("token_count"), int(tokens.numel()),
         payload.get("token_count") == int(tokens.numel())),
    ]
    for key, observed, required, ok in checks:
        if not ok:
            bad[key] = {"observed": observed, "required": required}
    digest = payload.get("token_content_sha256")
    if not isinstance(digest, str) or re.fullmatch(r"[0-9a-f]{64}", digest) is None:
        bad["token_content_sha256"] = {"observed": digest,
                                       "required": "64 lowercase hexadecimal characters"}
    if max_tokens is not None and int(tokens.numel()) != int(max_tokens):
        bad["token_count"] = {"observed": int(tokens.numel()), "required": int(max_tokens)}
    if int(tokens.numel()) < int(args.seq_len) + 2:
        bad["minimum_token_count"] = {"observed": int(tokens.numel()), "required": int(args.seq_len) + 2}
    if not tokens.is_contiguous():
        bad["contiguous"] = {"observed": False, "required": True}
    if bad:
        raise RuntimeError(f"token cache metadata mismatch for {cache_file}: {bad}")
    return tokens


def write_token_cache(cache_file: Path, tokens: torch.Tensor, args, split) -> None:
    """Atomic write (temporary file, fsync, rename, directory fsync)."""
    payload = {"schema": CACHE_SCHEMA, "tokens": tokens, "token_count": int(tokens.numel()),
               "token_content_sha256": tensor_content_sha256(tokens), **cache_metadata(args, split)}
    tmp = cache_file.with_name(f".{cache_file.name}.tmp-{os.getpid()}")
    try:
        with tmp.open("wb") as fh:
            torch.save(payload, fh)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, cache_file)
        fd = os.open(cache_file.parent, os.O_RDONLY | os.O_DIRECTORY)
        try:
            os.fsync(fd)
        finally:
            os.close(fd)
    finally:
        if tmp.exists():
            tmp.unlink()


# ---------------------------------------------------------------------------
# Procedural text corpora (document ``index`` -> one string).

def arithmetic_text(i: int) -> str:
    a, b = (i * 48271 + 17) % 10000, (i * 69621 + 23) % 10000
    step, first = i % 17 + 2, (i * 37 + 11) % 2000
    seq = [first + step * k for k in range(5)]
    kind = i % 4
    if kind == 0:
        return f"Task add: {a} plus {b} equals {a + b}. Check: {a + b} minus {b} equals {a}."
    if kind == 1:
        lo, hi = min(a, b), max(a, b)
        return f"Task compare: between {a} and {b}, smaller is {lo}, larger is {hi}. Difference is {hi - lo}."
    if kind == 2:
        return (f"Task sequence: {seq[0]}, {seq[1]}, {seq[2]}, {seq[3]}; next is {seq[4]}. "
                f"Step size is {step}.")
    x, y = a % 100, b % 100
    return f"Task multiply-small: {x} times {y} equals {x * y}. Inputs came from {a} and {b}."


def code_text(i: int) -> str:
    base = (i * 1103515245 + 12345) & 0x7FFFFFFF
    x, y = base % 97, (base // 97) % 89
    z = (3 * x + 2 * y + i) % 211
    name = f"v{i % 17}"
    kind = i % 5
    if kind == 0:
        k = y % 7 + 2
        return (f"def f({name}, y):\n    total = {name} + {x}\n    total = total * {k}\n    return total\n"
                f"# f({y}, {z % 11}) -> {(y + x) * k}")
    if kind == 1:
        vals = [(x + j * (y % 5 + 1)) % 100 for j in range(5)]
        return f"items = {vals}\nacc = 0\nfor item in items:\n    acc += item\nprint(acc)  # {sum(vals)}"
    if kind == 2:
        chosen = x if (x + y) % 2 == 0 else y
        return (f"left = {x}\nright = {y}\nanswer = left if (left + right) % 2 == 0 else right\n"
                f"answer == {chosen}")
    if kind == 3:
        keys = [f"k{(i + j) % 9}" for j in range(3)]
        vals = [(x + y + 13 * j) % 50 for j in range(3)]
        body = ", ".join(f"{keys[j]!r}: {vals[j]}" for j in range(3))
        return f"data = {{{body}}}\nlookup = {keys[1]!r}\nvalue = data[lookup]  # {vals[1]}"
    final = x + 6 if x % 2 == (x + 6) % 2 else x + 7
    return f"while {name} < {x + 6}:\n    {name} += 2\n# start {x}, stop {x + 6}, final {final}"


def symbolic_text(i: int) -> str:
    letter = lambda k: chr(ord("A") + k % 8)
    a, b, c = letter(i), letter(i * 3 + 1), letter(i * 5 + 2)
    n = i % 7 + 3
    kind = i % 5
    if kind == 0:
        return f"Rewrite rule: ({a} -> {b}) and ({b} -> {c}). Query {a}. Result {c}."
    if kind == 1:
        seq = [((i + 2) * (k + 1) + n) % 19 for k in range(6)][:4]
        return f"Map every token by +{n}: input {seq} output {[v + n for v in seq]}."
    if kind == 2:
        bits = [(i >> k) & 1 for k in range(6)]
        parity = sum(bits) % 2
        return f"Boolean trace: bits {bits}; xor parity is {parity}; not parity is {1 - parity}."
    if kind == 3:
        depth = i % 4 + 1
        return f"Bracket task: source {'(' * depth + a + ')' * depth}; depth {depth}; core token {a}."
    src = [a, b, c, a]
    return f"Reverse-copy task: source {' '.join(src)}; target {' '.join(reversed(src))}."


def reasoning_mix_text(i: int) -> str:
    return (arithmetic_text, code_text, symbolic_text)[i % 3](i)


TEXT_CORPORA = {
    "synthetic/arithmetic": arithmetic_text,
    "synthetic/code": code_text,
    "synthetic/symbolic": symbolic_text,
    "synthetic/reasoning_mix": reasoning_mix_text,
}


# ---------------------------------------------------------------------------
# Tokenizers

class ByteTokenizer:
    """UTF-8 bytes (ids 0-255) plus end-of-document id 256; needs no files."""

    eos_token_id = 256
    pad_token_id = 256

    def __len__(self):
        return 257

    def __call__(self, texts, add_special_tokens=False):
        return {"input_ids": [list(t.encode("utf-8")) for t in texts]}


def load_tokenizer(args):
    if args.tokenizer == "bytes":
        return ByteTokenizer()
    import transformers
    return transformers.AutoTokenizer.from_pretrained(args.tokenizer, cache_dir=args.hf_cache,
                                                      revision=args.tokenizer_revision)


def vocab_size_for(args) -> int:
    if args.dataset_name in DIRECT_SOURCES:
        return int(args.vocab_size)
    return len(load_tokenizer(args))


def _append_document(tokens, ids, eos, max_tokens, skip):
    if not ids:
        return skip, False
    doc = list(ids) + [eos]
    if skip > 0:
        if skip >= len(doc):
            return skip - len(doc), False
        doc, skip = doc[skip:], 0
    tokens.extend(doc)
    return skip, max_tokens is not None and len(tokens) >= max_tokens


def _texts_of(batch, column):
    if column != "auto" and column in batch:
        values = batch[column]
    else:
        values = next((batch[k] for k in ("text", "content", "document", "raw_content") if k in batch),
                      None)
    if values is None:
        raise KeyError(f"could not find text column {column!r}; available columns: "
                       f"{', '.join(sorted(batch.keys()))}")
    return [t for t in values if isinstance(t, str) and t.strip()]


def _record_text(record, column):
    if column == "auto":
        return next((record.get(k) for k in ("text", "content", "document", "raw_content")
                     if record.get(k)), None)
    value = record
    for part in column.split("."):
        if not isinstance(value, dict):
            return None
        value = value.get(part)
    return value


def _tokenize(args, split, max_tokens):
    if args.dataset_name in DIRECT_SOURCES:
        if max_tokens is None:
            raise ValueError(f"{args.dataset_name} requires a token count")
        seed = int(args.seed) + SPLIT_OFFSETS.get(split, 90_000_000)
        if args.dataset_name == "synthetic/zipf":
            return zipf_tokens(max_tokens, int(args.vocab_size), alpha=float(args.zipf_alpha), seed=seed)
        return uniform_tokens(max_tokens, int(args.vocab_size), seed=seed)
    tokenizer = load_tokenizer(args)
    eos = tokenizer.eos_token_id if tokenizer.eos_token_id is not None else tokenizer.pad_token_id
    if eos is None:
        raise ValueError("tokenizer must define eos_token_id or pad_token_id")
    tokens = array("I")
    if args.dataset_name in TEXT_CORPORA:
        if max_tokens is None:
            raise ValueError(f"{args.dataset_name} requires max_tokens")
        make = TEXT_CORPORA[args.dataset_name]
        index = SPLIT_OFFSETS.get(split, 90_000_000)
        bs = int(args.tokenize_batch_size)
        while len(tokens) < max_tokens:
            batch = tokenizer([make(index + k) for k in range(bs)], add_special_tokens=False)
            index += bs
            for ids in batch["input_ids"]:
                if ids:
                    tokens.extend(ids)
                    tokens.append(eos)
                if len(tokens) >= max_tokens:
                    break
    else:
        from datasets import load_dataset
        config = args.dataset_config
        if config is not None and str(config).lower() in {"", "none", "null"}:
            config = None
        kw = dict(split=actual_dataset_split(args, split), cache_dir=args.hf_cache,
                  streaming=args.dataset_streaming, revision=args.dataset_revision)
        if args.trust_remote_code:
            kw["trust_remote_code"] = True
        ds = load_dataset(args.dataset_name, config, **kw) if config else load_dataset(args.dataset_name, **kw)
        skip_docs = dataset_skip_documents(args, split)
        skip = dataset_skip_tokens(args, split)
        bs = int(args.tokenize_batch_size)
        done = False
        if args.dataset_streaming:
            texts, seen = [], 0
            for record in ds:
                if seen < skip_docs:
                    seen += 1
                    continue
                text = _record_text(record, args.dataset_text_column)
                if isinstance(text, str) and text.strip():
                    texts.append(text)
                if len(texts) < bs:
                    continue
                for ids in tokenizer(texts, add_special_tokens=False)["input_ids"]:
                    skip, done = _append_document(tokens, ids, eos, max_tokens, skip)
                    if done:
                        break
                texts = []
                if done:
                    break
            if texts and not done:
                for ids in tokenizer(texts, add_special_tokens=False)["input_ids"]:
                    skip, done = _append_document(tokens, ids, eos, max_tokens, skip)
                    if done:
                        break
        else:
            for start in range(skip_docs, len(ds), bs):
                texts = _texts_of(ds[start:min(start + bs, len(ds))], args.dataset_text_column)
                for ids in tokenizer(texts, add_special_tokens=False)["input_ids"] if texts else []:
                    skip, done = _append_document(tokens, ids, eos, max_tokens, skip)
                    if done:
                        break
                if done:
                    break
    arr = np.frombuffer(tokens, dtype=np.uint32)
    if max_tokens is not None:
        arr = arr[:max_tokens]
    if arr.size and int(arr.max()) > np.iinfo(np.int32).max:
        raise ValueError("token ids exceed int32 range")
    return torch.from_numpy(arr.astype(np.int32, copy=True))


def load_or_tokenize(args, split, max_tokens) -> torch.Tensor:
    """Cached tokens for ``split``, building the cache under an exclusive file lock if needed."""
    cache_file = token_cache_path(args, split, max_tokens)
    with Path(f"{cache_file}.lock").open("a+b") as lock:
        if not args.refresh_cache:
            fcntl.flock(lock.fileno(), fcntl.LOCK_SH)
            if cache_file.exists():
                return load_cached_tokens(cache_file, args, split, max_tokens)
            fcntl.flock(lock.fileno(), fcntl.LOCK_UN)
        fcntl.flock(lock.fileno(), fcntl.LOCK_EX)
        if cache_file.exists() and not args.refresh_cache:
            return load_cached_tokens(cache_file, args, split, max_tokens)
        tokens = _tokenize(args, split, max_tokens)
        if tokens.numel() < args.seq_len + 2:
            raise ValueError(f"{split} split produced too few tokens")
        write_token_cache(cache_file, tokens, args, split)
        return load_cached_tokens(cache_file, args, split, max_tokens)
