"""All-gather of the owners' updated weights over NVLink peer memory (csrc/owner_comm.cu).

With layer-sharded optimizers every rank updates the weights of the layers it
owns; the others need those weights before their next forward.  Instead of
one NCCL broadcast per owner, every rank pulls:

* ``publish()`` (after this rank's optimizer step, current stream): bump this
  rank's ``published`` counter at system scope, and mark a pull pending;
* ``pull()``: on the parameter side stream, for every other owner: one
  single-thread kernel waits (bounded) until that owner's counter has reached
  this rank's own (every rank publishes once per step, so the owner has
  finished the same step), then a copy kernel reads the owner's weight range
  with 16-byte peer loads into the local buffer.  Each owner's parameters are
  marked pending on an event after its copy
  (:mod:`~rational_optimizer_b200.parallel.param_ready`), so a layer's
  forward waits only for its own owner.  Pulls are idempotent: pulling again
  before the next publish copies the same weights.
* the pull is lazy: the first reader of a parameter after a publish
  (``param_ready.wait``) enqueues it; a captured step graph pulls inside the
  graph instead (``train.graphs``), so the copies overlap the forward of the
  layers whose owners have already been copied.

The weight buffer (every TILLER-managed matrix, owner-ordered, identical
layout on every rank) is ``cudaMalloc``'d so its CUDA IPC handle covers it
from offset 0.  An owner overwrites its weights only after it has this rank's
next gradients, which this rank produces after the forward that waited for
the copy, so a copy never reads a half-written update.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch.autograd.graph import increment_version

from .. import _ext
from . import param_ready

# CTAs per owner copy (RO_PULL_CTAS): enough to keep NVLink busy without
# taking many SMs from the forward that the copies overlap
PULL_CTAS = int(os.environ.get("RO_PULL_CTAS", "24"))


def available() -> bool:
    return _ext.available() and hasattr(_ext.ext(), "owner_pull")


def shared_buffer(numel: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(raw uint8 allocation, fp32 view of ``numel`` elements) for IPC sharing."""
    raw = _ext.ext().comm_alloc(max(16, 4 * int(numel)), torch.device(device).index)
    return raw, raw.view(torch.float32)[: int(numel)]


class OwnerGather:
    def __init__(self, raw: torch.Tensor, flat: torch.Tensor, ranges, params_by_owner, *, group=None,
                 timeout_s=None):
        """``ranges[r]``: (lo, hi) element range of owner r's weights in ``flat``
        (empty when r owns nothing); ``params_by_owner[r]``: those parameters."""
        C = _ext.ext()
        self.flat = flat
        self.device = flat.device
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.ranges = [(int(lo), int(hi)) for lo, hi in ranges]
        self.params_by_owner = params_by_owner
        if timeout_s is None:
            timeout_s = float(os.environ.get("RO_COMM_TIMEOUT_S", "10"))
        self.timeout_ns = int(timeout_s * 1e9)
        self.published = C.comm_alloc(16, self.device.index)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.pending = False
        param_ready.register_puller(self, replace=True)
        local = (C.comm_handle(raw), C.comm_handle(self.published))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, local, group=group)
        self._opened = []
        self.peer_flat, self.peer_published = [], []
        for r, (hf, hp) in enumerate(gathered):
            if r == self.rank:
                self.peer_flat.append(raw.data_ptr())
                self.peer_published.append(self.published.data_ptr())
            else:
                pf = C.comm_open(hf, self.device.index)
                pp = C.comm_open(hp, self.device.index)
                self._opened += [pf, pp]
                self.peer_flat.append(pf)
                self.peer_published.append(pp)

    def publish(self):
        _ext.ext().owner_publish(self.published)
        self.pending = True
        for r in range(self.world):
            if r != self.rank:
                for p in self.params_by_owner[r]:
                    increment_version(p)

    def pull(self):
        """Enqueue the copies from every other owner (side stream); returns the last event."""
        C = _ext.ext()
        side = param_ready.side_stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        event = None
        for r in range(self.world):
            lo, hi = self.ranges[r]
            if r == self.rank or hi <= lo:
                continue
            with torch.cuda.stream(side):
                C.owner_pull(self.peer_flat[r] + 4 * lo, self.flat[lo:hi], self.peer_published[r],
                             self.published, self.err, self.timeout_ns, PULL_CTAS)
                event = torch.cuda.Event()
                event.record(side)
            param_ready.defer(self.params_by_owner[r], event)
        return event

    def check(self):
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"weight all-gather: an owner did not publish in time (code {code}) "
                               f"on rank {self.rank}")

    def close(self):
        C = _ext.ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            C.comm_close(p)
        self._opened = []
