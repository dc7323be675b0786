"""Process-group bootstrap (one process per GPU) and small collective helpers.

``setup_distributed`` mirrors training/train.py:275-290 (``RANK``/
``LOCAL_RANK``/``WORLD_SIZE`` from the environment, NCCL on CUDA) but also
accepts gloo for CPU multi-process tests and always sets a finite
process-group timeout so ranks waiting on a dead peer fail instead of hanging.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    is_distributed: bool
    rank: int
    local_rank: int
    world_size: int
    device: torch.device


def setup_distributed(backend: str | None = None, timeout_s: float = 300.0) -> DistInfo:
    """Initialise the default process group when launched by torchrun."""
    if "RANK" not in os.environ:
        device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
        return DistInfo(False, 0, 0, 1, device)
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
    else:
        device = torch.device("cpu")
    if not dist.is_initialized():
        kwargs = {"backend": backend, "timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kwargs["device_id"] = device
        dist.init_process_group(**kwargs)
    return DistInfo(True, dist.get_rank(), local_rank, dist.get_world_size(), device)


def cleanup_distributed(info: DistInfo):
    if info.is_distributed and dist.is_initialized():
        # captured graphs holding NCCL calls must go before the process group
        from ..train.graphs import release_all
        release_all()
        dist.destroy_process_group()


def reduce_mean(value, device, is_distributed):
    t = torch.tensor(float(value), device=device)
    if is_distributed:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        t /= dist.get_world_size()
    return float(t.item())


def reduce_max(value, device, is_distributed):
    t = torch.tensor(float(value), device=device)
    if is_distributed:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
