"""Token sources and batch sampling.

* :func:`zipf_tokens` - synthetic Zipf(alpha) token ids from a seed (the
  benchmark data: no dataset download is possible or needed).
* :func:`uniform_tokens` - uniform ids (the CPU plumbing configuration).
* :func:`sample_batch` - random contiguous windows, identical in semantics to
  the reference sampler (training/train.py:785-791): ``starts`` drawn from a
  CPU generator seeded ``seed + 997 * rank``, inputs/targets shifted by one.
* :class:`PinnedBatcher` - draws the next batch into a pinned host buffer
  and copies it to the device asynchronously (the end-to-end input path).
"""
from __future__ import annotations

import numpy as np
import torch


def zipf_tokens(count: int, vocab: int, *, alpha: float = 1.1, seed: int = 0) -> torch.Tensor:
    """``count`` int32 ids with P(id = k) proportional to (k + 1)^-alpha."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    pmf = ranks ** (-float(alpha))
    cdf = np.cumsum(pmf)
    cdf /= cdf[-1]
    rng = np.random.default_rng(int(seed))
    ids = np.searchsorted(cdf, rng.random(int(count)), side="right")
    np.minimum(ids, vocab - 1, out=ids)
    return torch.from_numpy(ids.astype(np.int32))


def uniform_tokens(count: int, vocab: int, *, seed: int = 0) -> torch.Tensor:
    gen = torch.Generator().manual_seed(int(seed))
    return torch.randint(0, int(vocab), (int(count),), generator=gen, dtype=torch.int64).to(torch.int32)


def sample_batch(tokens, batch_size, seq_len, offsets, generator, device):
    """Random contiguous windows -> (x, y) long tensors on ``device``."""
    max_start = tokens.numel() - seq_len - 1
    starts = torch.randint(max_start, (batch_size,), generator=generator)
    block = tokens[starts[:, None] + offsets[None, :]]
    x = block[:, :-1].to(device=device, dtype=torch.long, non_blocking=True)
    y = block[:, 1:].to(device=device, dtype=torch.long, non_blocking=True)
    return x, y


class PinnedBatcher:
    """Samples windows into a pinned host buffer; :meth:`to_device` copies them.

    Bytes moved host->device per batch: ``batch * (seq_len + 1) * 8``.
    """

    def __init__(self, tokens, batch_size, seq_len, *, seed, rank=0):
        self.tokens = tokens
        self.batch_size = int(batch_size)
        self.seq_len = int(seq_len)
        self.offsets = torch.arange(self.seq_len + 1)
        self.generator = torch.Generator(device="cpu")
        self.generator.manual_seed(int(seed) + 997 * int(rank))
        self.host = torch.empty((self.batch_size, self.seq_len + 1), dtype=torch.long,
                                pin_memory=torch.cuda.is_available())

    @property
    def bytes_per_batch(self) -> int:
        return self.host.numel() * self.host.element_size()

    def next_host(self):
        max_start = self.tokens.numel() - self.seq_len - 1
        starts = torch.randint(max_start, (self.batch_size,), generator=self.generator)
        self.host.copy_(self.tokens[starts[:, None] + self.offsets[None, :]])
        return self.host

    def to_device(self, device, host=None):
        h = self.host if host is None else host
        block = h.to(device=device, non_blocking=True)
        return block[:, :-1], block[:, 1:]
