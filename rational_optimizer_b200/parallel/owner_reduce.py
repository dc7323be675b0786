"""Reduce-to-owner of layer gradients over NVLink peer memory (csrc/owner_comm.cu).

With the TILLER optimizers layer-sharded across data-parallel ranks, only a
layer's owner uses its averaged gradient.  :class:`OwnerReduce` replaces the
all-reduce of those gradients (the reference runs DDP's fp32 all-reduce,
training/train.py:2366-2371) by

* ``send(layer)``: as soon as backward has produced a layer's gradient, every
  other rank writes it (fp32; bf16 with ``transport="bf16"``; int8 with one
  fp32 scale per 256 elements with ``transport="int8"``) into its slot of the
  owner's receive buffer with peer stores, on a communication stream,
  overlapped with the rest of backward (fp32 with ``copy_engine=True``: one
  copy-engine copy per layer, so the sends occupy no SM);
* ``reduce()``: after backward the owner waits (bounded) for every sender,
  sums the slots in rank order together with its own gradient, scales by
  1/world, writes the result over its own gradient, and keeps the sum of
  squares of what it wrote for the global gradient norm.

Per rank and step that moves (world-1)/world of the managed gradient once
(an all-reduce moves it twice and also delivers it where it is not used).
Non-owners keep their local, un-averaged gradient of the layers they do not
own; nothing on the optimizer path reads it (the sharded optimizers work on
owned layers, the clip norm and TILLER's decay derivative take the owners'
partial sums).

Buffers are ``cudaMalloc``'d and shared through CUDA IPC; the receive layout
of every owner is a deterministic function of the layer sizes and the
ownership map (:func:`receive_layout`), so a sender computes the slot address
without any exchange beyond the handles.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import _ext

# CTAs per send (RO_SEND_CTAS): sends run beside the backward's kernels
SEND_CTAS = int(os.environ.get("RO_SEND_CTAS", "16"))
REDUCE_CTAS = 296
MODES = {"f32": 0, "bf16": 1, "int8": 2}
QBLOCK = 256  # int8: elements per fp32 scale


def slot_bytes(n: int, transport: str) -> int:
    """Bytes of one sender's slot of an ``n``-element layer (the kernels'
    layout: fp32 / bf16 values, or int8 values padded to 16 bytes followed by
    the per-256 fp32 scales padded to 16 bytes)."""
    n = int(n)
    if transport == "f32":
        return 4 * n
    if transport == "bf16":
        return 2 * n
    r16 = lambda b: (b + 15) // 16 * 16  # noqa: E731
    return r16(n) + r16(4 * ((n + QBLOCK - 1) // QBLOCK))


def receive_layout(sizes, owners, world, transport="f32"):
    """Per owner: {layer: byte offset of the layer's first slot} in its receive
    buffer (``world`` slots per layer back to back, layers in order), and the
    buffer's total bytes."""
    offsets, totals = {}, {}
    for layer, (n, owner) in enumerate(zip(sizes, owners)):
        table = offsets.setdefault(owner, {})
        table[layer] = totals.get(owner, 0)
        totals[owner] = totals.get(owner, 0) + world * slot_bytes(n, transport)
    return offsets, totals


def counter_index(layer, owners):
    """Index of ``layer`` among the layers its owner owns (the owner's counter slot)."""
    return sum(1 for l in range(layer) if owners[l] == owners[layer])


class OwnerReduce:
    def __init__(self, flat: torch.Tensor, segments, owners, *, group=None, transport="f32",
                 timeout_s=None, send_ctas=None, copy_engine=False):
        """``copy_engine`` (fp32 transport only): each send is one device-to-device
        copy into the owner's slot, done by a copy engine instead of send CTAs,
        followed by the same arrival; the backward's kernels keep every SM."""
        if transport not in MODES:
            raise ValueError(f"owner transport must be one of {sorted(MODES)}, got {transport!r}")
        if copy_engine and transport != "f32":
            raise ValueError("copy-engine sends carry the fp32 transport only")
        self.copy_engine = bool(copy_engine)
        C = _ext.ext()
        self.flat = flat
        self.device = flat.device
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.segments = [(int(o), int(n)) for o, n in segments]
        self.owners = [int(r) for r in owners]
        self.transport = transport
        self.mode = MODES[transport]
        # CTAs per send launch; the owner expects (world - 1) * send_ctas arrivals per layer,
        # so every rank must use the same value
        self.send_ctas = int(send_ctas or SEND_CTAS)
        for off, n in self.segments:
            if off % 8 or n % 8:
                raise ValueError("owner-reduce segments must start and end on 32-byte boundaries")
        if timeout_s is None:
            timeout_s = float(os.environ.get("RO_COMM_TIMEOUT_S", "10"))
        self.timeout_ns = int(timeout_s * 1e9)
        sizes = [n for _, n in self.segments]
        self.recv_offsets, totals = receive_layout(sizes, self.owners, self.world, transport)
        self.owned = [l for l, r in enumerate(self.owners) if r == self.rank]
        self.recv = C.comm_alloc(max(16, totals.get(self.rank, 0)), self.device.index)
        self.counters = C.comm_alloc(max(16, 4 * len(self.owned)), self.device.index)
        local = (C.comm_handle(self.recv), C.comm_handle(self.counters))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, local, group=group)
        self._opened = []
        self.peer_recv, self.peer_counters = [], []
        for r, (hr, hc) in enumerate(gathered):
            if r == self.rank:
                self.peer_recv.append(self.recv.data_ptr())
                self.peer_counters.append(self.counters.data_ptr())
            else:
                pr = C.comm_open(hr, self.device.index)
                pc = C.comm_open(hc, self.device.index)
                self._opened += [pr, pc]
                self.peer_recv.append(pr)
                self.peer_counters.append(pc)
        dev = self.device
        mine = self.recv_offsets.get(self.rank, {})
        self.dev_offsets = torch.tensor([self.segments[l][0] for l in self.owned], dtype=torch.int64, device=dev)
        self.dev_sizes = torch.tensor([self.segments[l][1] for l in self.owned], dtype=torch.int64, device=dev)
        self.dev_recv_offsets = torch.tensor([mine[l] for l in self.owned], dtype=torch.int64, device=dev)
        self.sumsq = torch.zeros(REDUCE_CTAS, dtype=torch.float32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self._sent = set()

    def slot_address(self, layer: int, element: int) -> int:
        """Device address (in the owner's memory) of element ``element`` of this
        rank's fp32 slot for ``layer`` - where a weight-gradient GEMM may store
        its tiles directly (fp32 transport only)."""
        if self.transport != "f32":
            raise RuntimeError("direct slot stores need the fp32 transport")
        owner = self.owners[layer]
        n = self.segments[layer][1]
        return (self.peer_recv[owner] + self.recv_offsets[owner][layer] + self.rank * slot_bytes(n, "f32")
                + 4 * int(element))

    # -- per step ---------------------------------------------------------------
    def begin(self):
        self._sent = set()

    def send(self, layer: int, delivered=()):
        """Ship this rank's gradient of ``layer`` to its owner (no-op for owned
        layers).  ``delivered``: (start, length) element ranges of the layer that
        already sit in the owner's slot (stored there by the weight-gradient
        GEMMs); the rest is sent, then the arrival is signalled once."""
        if layer in self._sent:
            return
        self._sent.add(layer)
        owner = self.owners[layer]
        if owner == self.rank:
            return
        off, n = self.segments[layer]
        dst = self.peer_recv[owner] + self.recv_offsets[owner][layer] + self.rank * slot_bytes(n, self.transport)
        counter = self.peer_counters[owner] + 4 * counter_index(layer, self.owners)
        current = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(current)
        C = _ext.ext()
        with torch.cuda.stream(self.stream):
            if not delivered:
                if self.copy_engine:
                    C.owner_copy(self.flat[off:off + n], dst)
                    C.owner_signal(counter, self.send_ctas)
                else:
                    C.owner_send(self.flat[off:off + n], dst, self.mode, counter, self.send_ctas)
                return
            cursor = 0
            for start, length in sorted(delivered) + [(n, 0)]:
                if start > cursor:  # a gap the GEMMs did not store: send it without an arrival
                    if self.copy_engine:
                        C.owner_copy(self.flat[off + cursor:off + start], dst + 4 * cursor)
                    else:
                        C.owner_send(self.flat[off + cursor:off + start], dst + 4 * cursor, self.mode, 0,
                                     self.send_ctas)
                cursor = max(cursor, start + length)
            # one arrival worth a full send, after everything this stream ordered before it
            C.owner_signal(counter, self.send_ctas)

    def reduce(self):
        """Send what backward did not report, then reduce the owned layers (current stream)."""
        for layer in range(len(self.segments)):
            if layer not in self._sent:
                self.send(layer)
        current = torch.cuda.current_stream(self.device)
        current.wait_stream(self.stream)  # local gradients stay untouched until the sends read them
        if self.owned:
            _ext.ext().owner_reduce(self.flat, self.recv.data_ptr(), self.counters, self.dev_offsets,
                                    self.dev_sizes, self.dev_recv_offsets, self.sumsq, self.rank,
                                    self.world, (self.world - 1) * self.send_ctas, 1.0 / self.world, self.mode,
                                    self.err, self.timeout_ns)
        else:
            self.sumsq.zero_()
        self._sent = set()

    def owned_sumsq(self) -> torch.Tensor:
        """Sum of squares of the reduced gradient of this rank's layers (device scalar)."""
        return self.sumsq.sum()

    def check(self):
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"reduce-to-owner: a sender did not arrive in time (code {code}) "
                               f"on rank {self.rank}")

    def close(self):
        C = _ext.ext()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            C.comm_close(p)
        self._opened = []
