"""Deferred parameter replication: CUDA events the next use of a parameter waits on.

With layer-sharded optimizers each rank updates the weights of the layers it
owns and the updated weights are broadcast from their owners on a side
stream, so the transfer overlaps whatever the default stream does next (the
next step's forward).  ``defer(params, event)`` marks parameters as pending
until ``event``; ``wait(param)`` (called by every ``ops.linear.Linear``
forward) makes the current stream wait for it first, so a layer's forward
starts as soon as its own weights have arrived.  ``wait_all()`` is for code
that reads every parameter (checkpoints, evaluation, state dicts).
"""
from __future__ import annotations

import torch

_PENDING: dict[int, torch.cuda.Event] = {}
_STREAMS: dict[int, torch.cuda.Stream] = {}
# objects with a ``pending`` flag and ``pull()``: replication that is enqueued
# lazily, by the first reader of a parameter (see ``parallel.owner_gather``)
_PULLERS: list = []


def register_puller(obj, *, replace=False) -> None:
    """Add ``obj``; ``replace=True`` first drops every other puller on the same device
    (a newly built model's replication supersedes the previous model's)."""
    if replace:
        _PULLERS[:] = [o for o in _PULLERS if getattr(o, "device", None) != getattr(obj, "device", None)]
    if obj not in _PULLERS:
        _PULLERS.append(obj)


def _flush_pullers() -> None:
    for obj in _PULLERS:
        if obj.pending:
            obj.pending = False
            obj.pull()


def claim_pullers() -> list:
    """Mark every pending lazy replication as taken by the caller (a captured
    step graph that performs the pulls itself) and return the claimed objects."""
    claimed = [obj for obj in _PULLERS if obj.pending]
    for obj in claimed:
        obj.pending = False
    return claimed


def side_stream(device: torch.device) -> torch.cuda.Stream:
    index = torch.device(device).index
    if index is None:
        index = torch.cuda.current_device()
    s = _STREAMS.get(index)
    if s is None:
        s = torch.cuda.Stream(device=index)
        _STREAMS[index] = s
    return s


def defer(params, event: torch.cuda.Event) -> None:
    for p in params:
        _PENDING[id(p)] = event


def pending() -> bool:
    """True while some parameter may still be waiting for its replication
    (an event to wait on, or a lazy pull not enqueued yet)."""
    return bool(_PENDING) or any(obj.pending for obj in _PULLERS)


def pullers() -> list:
    return list(_PULLERS)


def forget_events(events) -> None:
    """Drop pending entries whose events are in ``events`` (recorded inside a
    graph capture: the graph carries those dependencies itself)."""
    ids = {id(e) for e in events}
    for key in [k for k, ev in _PENDING.items() if id(ev) in ids]:
        del _PENDING[key]


def wait(param) -> None:
    if _PULLERS:
        _flush_pullers()
    if _PENDING:
        ev = _PENDING.pop(id(param), None)
        if ev is not None:
            torch.cuda.current_stream(param.device).wait_event(ev)


def wait_all() -> None:
    if _PULLERS:
        _flush_pullers()
    if not _PENDING:
        return
    for ev in set(_PENDING.values()):
        torch.cuda.current_stream().wait_event(ev)
    _PENDING.clear()
