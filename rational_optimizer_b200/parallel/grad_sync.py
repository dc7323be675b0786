"""Data-parallel gradient synchronisation over one flat gradient buffer.

Every trainable parameter's ``.grad`` is a view into a single fp32 buffer
(the reference's DDP runs with per-parameter grads in 25 MB buckets,
training/train.py:2366-2371).  After backward the whole buffer is averaged
across ranks in fixed-size buckets, by the in-kernel NVLink all-reduce of
``csrc/comm.cu`` when the communicator is available (one process per GPU,
peer memory mapped through CUDA IPC), otherwise by NCCL.  With one rank the
synchroniser only manages the buffer.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops.linear import ACCUMULATE_ATTR


class GradientSynchronizer:
    def __init__(self, model: torch.nn.Module, *, group=None, bucket_bytes: int = 256 << 20,
                 communicator=None, transport: str | None = None):
        seen, params = set(), []
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                params.append(p)
        self.params = params
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        dtype = params[0].dtype
        device = params[0].device
        total = sum(p.numel() for p in params)
        if transport is None:
            transport = os.environ.get("RO_GRAD_TRANSPORT", "p2p")
        if communicator is None and self.world > 1 and transport == "p2p" and device.type == "cuda":
            from .comm import maybe_communicator
            communicator = maybe_communicator(device, total, group=group)
        self.communicator = communicator
        self.transport = "p2p" if communicator is not None else ("nccl" if self.world > 1 else "none")
        if communicator is not None and dtype == torch.float32:
            self.flat = communicator.float_view(total)
            self.flat.zero_()
        else:
            self.flat = torch.zeros(total, dtype=dtype, device=device)
        self.views = []
        offset = 0
        accumulate = self.flat.is_cuda and self.flat.dtype == torch.float32
        for p in params:
            n = p.numel()
            view = self.flat[offset: offset + n].view_as(p)
            p.grad = view
            if accumulate:
                # the model's GEMMs may add weight gradients straight into the view
                setattr(p, ACCUMULATE_ATTR, True)
            self.views.append(view)
            offset += n
        self.bucket_elems = max(1, bucket_bytes // self.flat.element_size())

    def zero_grad(self):
        for p, v in zip(self.params, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                p.grad = v
        self.flat.zero_()

    def synchronize(self):
        """Average gradients across ranks (no-op for one rank)."""
        if self.world == 1:
            return
        if self.communicator is not None:
            self.communicator.all_reduce_mean_(self.flat)
            return
        for start in range(0, self.flat.numel(), self.bucket_elems):
            chunk = self.flat[start: start + self.bucket_elems]
            dist.all_reduce(chunk, op=dist.ReduceOp.SUM, group=self.group)
        self.flat.div_(self.world)
