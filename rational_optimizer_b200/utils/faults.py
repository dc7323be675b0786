"""Host-side fault injection for failure-detection tests.

Faults are injected on the host only (never on a GPU): a rank raises, exits
without cleanup, or stalls in Python at a named point of the trainer.  The
environment variable ``RO_INJECT_FAULT`` selects one fault as
``point:rank:step:mode`` (``mode`` is ``raise``, ``exit`` or ``stall``), e.g.
``train_step:1:3:raise`` makes rank 1 raise at the start of step 3.

Points: ``train_step`` (start of a training step, before any collective of
that step), ``checkpoint_written`` (after this rank's temporary checkpoint
files are written, before they are promoted) and ``checkpoint_promoted``
(after the files are promoted, before the new manifest is written).  Unset,
every call is a no-op.
"""
from __future__ import annotations

import os
import time

ENV = "RO_INJECT_FAULT"
EXIT_CODE = 71


class InjectedFault(RuntimeError):
    """Raised by ``mode == "raise"``."""


def _spec():
    raw = os.environ.get(ENV, "")
    if not raw:
        return None
    parts = raw.split(":")
    if len(parts) != 4 or parts[3] not in ("raise", "exit", "stall"):
        raise ValueError(f"{ENV} must be point:rank:step:mode, got {raw!r}")
    return parts[0], int(parts[1]), int(parts[2]), parts[3]


def maybe_inject(point: str, rank: int, step: int) -> None:
    spec = _spec()
    if spec is None:
        return
    p, r, s, mode = spec
    if p != point or r != int(rank) or s != int(step):
        return
    if mode == "raise":
        raise InjectedFault(f"injected fault at {point} on rank {rank}, step {step}")
    if mode == "exit":
        os._exit(EXIT_CODE)
    time.sleep(float(os.environ.get("RO_INJECT_STALL_S", "3600")))
