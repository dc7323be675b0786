"""Peer-memory communicator for the in-kernel NVLink collectives (csrc/comm.cu).

Each rank ``cudaMalloc``s one communication buffer and a flag array, exports
their CUDA IPC handles, and opens every peer's handles once at construction
(exchange through the default process group).  Collectives are then single
kernels that read peer memory directly over NVLink/NVSwitch; flags at system
scope order the phases.  Every wait inside the kernels is bounded by
``timeout_s``; :meth:`check` raises if any kernel recorded a timeout.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import _ext

FLAG_SLOTS = 3 * 16  # [phase][rank] uint32


class P2PCommunicator:
    def __init__(self, device, rank, world, buffer_bytes, *, group=None, timeout_s=None, mode="f32"):
        C = _ext.ext()
        self.device = torch.device(device)
        self.rank = int(rank)
        self.world = int(world)
        self.group = group
        self.mode = mode
        if timeout_s is None:
            timeout_s = float(os.environ.get("RO_COMM_TIMEOUT_S", "10"))
        self.timeout_ns = int(timeout_s * 1e9)
        self.buffer = C.comm_alloc(int(buffer_bytes), self.device.index)
        self.flags = C.comm_alloc(FLAG_SLOTS * 4, self.device.index)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        local = (C.comm_handle(self.buffer), C.comm_handle(self.flags))
        if self.world > 1:
            gathered = [None] * self.world
            dist.all_gather_object(gathered, local, group=group)
        else:
            gathered = [local]
        self._opened = []
        self.data_ptrs, self.flag_ptrs = [], []
        for r, (hb, hf) in enumerate(gathered):
            if r == self.rank:
                self.data_ptrs.append(self.buffer.data_ptr())
                self.flag_ptrs.append(self.flags.data_ptr())
            else:
                pb = C.comm_open(hb, self.device.index)
                pf = C.comm_open(hf, self.device.index)
                self._opened += [pb, pf]
                self.data_ptrs.append(pb)
                self.flag_ptrs.append(pf)

    @classmethod
    def create(cls, device, numel=None, *, group=None, mode="f32"):
        """A communicator over ``group`` (2..16 ranks), or None when the process
        group, the peer-memory kernels of the extension, or enough ranks are missing
        (callers then use NCCL through torch.distributed)."""
        if not (dist.is_available() and dist.is_initialized()):
            return None
        if not _ext.available() or not hasattr(_ext.ext(), "comm_allreduce_f32"):
            return None
        world = dist.get_world_size(group)
        if world < 2 or world > 16:
            return None
        rank = dist.get_rank(group)
        return cls(device, rank, world, max(16, 4 * int(numel or 1)), group=group, mode=mode)

    def float_view(self, numel):
        """The first ``numel`` fp32 elements of the communication buffer."""
        if numel * 4 > self.buffer.numel():
            raise ValueError("communication buffer too small")
        return self.buffer[: numel * 4].view(torch.float32)

    def all_reduce_mean_(self, flat: torch.Tensor):
        """In-place mean over ranks of ``flat`` (must be :meth:`float_view` of this buffer)."""
        C = _ext.ext()
        if flat.data_ptr() != self.buffer.data_ptr():
            raise ValueError("all_reduce_mean_ operates on the registered buffer")
        self.epoch += 1
        C.comm_allreduce_f32(self.data_ptrs, self.flag_ptrs, self.rank, flat.numel(), 1.0 / self.world,
                             self.epoch, self.err, self.timeout_ns)

    def check(self):
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"peer collective timed out (phase code {code}) on rank {self.rank}")

    def close(self):
        C = _ext.ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            C.comm_close(p)
        self._opened = []


class Int8AllReduce:
    """Mean all-reduce of an fp32 tensor with int8 transport (256-element blocks, fp32 scales)."""

    def __init__(self, device, numel, *, group=None, timeout_s=None):
        C = _ext.ext()
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        self.numel = int(numel)
        self.comm = P2PCommunicator(device, rank, world, C.comm_i8_bytes(self.numel), group=group,
                                    timeout_s=timeout_s, mode="i8")

    def __call__(self, src: torch.Tensor, out: torch.Tensor):
        C = _ext.ext()
        c = self.comm
        c.epoch += 1
        C.comm_allreduce_i8(src, out, c.data_ptrs, c.flag_ptrs, c.rank, 1.0 / c.world, c.epoch, c.err,
                            c.timeout_ns)
