"""Data-parallel gradient synchronisation over one flat gradient buffer.

Every trainable parameter's ``.grad`` is a view into a single fp32 buffer
(the reference's DDP runs with per-parameter grads in 25 MB buckets,
training/train.py:2366-2371).  Two ways to average it across ranks:

* overlapped (default with NCCL): one bucket per transformer layer.  A
  layer's bucket is all-reduced (NCCL, ``ReduceOp.AVG``) as soon as the
  backward pass has produced every gradient in it, so the collectives of
  layers L-1 .. 1 run under the backward of the layers below; only the
  embedding/final-norm bucket is reduced after backward.  Readiness is
  tracked per parameter: weights whose gradient the GEMM accumulates in
  place report through ``READY_ATTR`` (``ops.linear``), all others through
  post-accumulate-grad hooks.  Buckets are launched strictly in descending
  layer order, so every rank issues the same collectives in the same order.
* whole buffer after backward: the in-kernel NVLink all-reduce of
  ``csrc/comm.cu`` when the P2P communicator is available (one process per
  GPU, peer memory mapped through CUDA IPC), otherwise NCCL in fixed-size
  buckets.

* reduce-to-owner (``transport="owner"`` / ``"owner-bf16"`` /
  ``"owner-int8"`` (per-256 fp32 block scales; lossy) / ``"owner-ce"``
  (fp32 sent by copy engines, no SM taken from backward; the default with
  several ranks when ``owner_layers`` names the matrices of layer-sharded
  optimizers): those matrices are laid out first in the buffer, one
  contiguous segment per layer, and each segment goes only to the rank that
  owns the layer (:class:`~.owner_reduce.OwnerReduce`, own NVLink kernels,
  sent during backward); the remaining parameters (embeddings, norms, GRAIN
  coefficients - the replicated optimizer's) are one contiguous range
  averaged with a single NCCL all-reduce after backward.

With one rank the synchroniser only manages the buffer.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import _ext
from ..ops.linear import ACCUMULATE_ATTR, READY_ATTR, ROUTE_ATTR


class GradientSynchronizer:
    def __init__(self, model: torch.nn.Module, *, group=None, bucket_bytes: int = 256 << 20,
                 communicator=None, transport: str | None = None, overlap: bool | None = None,
                 owner_layers=None, layer_owner=None):
        """``owner_layers``: per layer, the parameters a layer-sharded optimizer updates
        on the layer's owner only; ``layer_owner(layer) -> rank``.  Both are required
        for the reduce-to-owner transport."""
        seen, params = set(), []
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                params.append(p)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        dtype = params[0].dtype
        device = params[0].device
        total = sum(p.numel() for p in params)
        if transport is None:
            # With layer-sharded optimizers on several GPUs: reduce-to-owner
            # with fp32 copy-engine sends (measured 18.41 against 19.37 ms per
            # step for the per-layer NCCL buckets on 8 B200s); otherwise the
            # NCCL buckets overlapped with backward.
            default = "nccl"
            if (owner_layers is not None and self.world > 1 and device.type == "cuda" and _ext.available()
                    and hasattr(_ext.ext(), "owner_copy")):
                default = "owner-ce"
            transport = os.environ.get("RO_GRAD_TRANSPORT", default)
            if transport.startswith("owner") and not (
                    _ext.available() and hasattr(_ext.ext(), "owner_send")):
                transport = "nccl"
        self.owner = None
        owned_matrices = []
        if transport.startswith("owner"):
            if owner_layers is None or layer_owner is None or self.world < 2 or device.type != "cuda":
                transport = "nccl"
            else:
                # managed matrices first, one contiguous segment per layer
                owned_matrices = [list(ps) for ps in owner_layers]
                managed = {id(p) for ps in owned_matrices for p in ps}
                params = [p for ps in owned_matrices for p in ps] + [p for p in params if id(p) not in managed]
        self.params = params
        if overlap is None:
            overlap = os.environ.get("RO_GRAD_OVERLAP", "1") == "1"
        self.overlap = bool(overlap and self.world > 1 and device.type == "cuda" and transport == "nccl")
        self.owner_mode = transport.startswith("owner")
        if (communicator is None and self.world > 1 and transport == "p2p" and device.type == "cuda"):
            from .p2p import P2PCommunicator
            communicator = P2PCommunicator.create(device, total, group=group)
        self.communicator = communicator
        if communicator is not None:
            self.transport = "p2p"
        elif self.owner_mode:
            self.transport = transport if transport in ("owner-bf16", "owner-int8", "owner-ce") else "owner-f32"
        elif self.world > 1:
            self.transport = "nccl-overlap" if self.overlap else "nccl"
        else:
            self.transport = "none"
        if communicator is not None and dtype == torch.float32:
            self.flat = communicator.float_view(total)
            self.flat.zero_()
        else:
            self.flat = torch.zeros(total, dtype=dtype, device=device)
        self.views = []
        self.offsets = []
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
            self.offsets.append(offset)
            offset += n
        self.bucket_elems = max(1, bucket_bytes // self.flat.element_size())
        self._armed = False
        self._works = []
        self._trace = None
        self._reported = set()
        if self.overlap:
            self._setup_buckets(model)
        if self.owner_mode:
            self._setup_owner(owned_matrices, layer_owner)

    # -- reduce-to-owner ---------------------------------------------------------
    def _setup_owner(self, layers, layer_owner):
        from .owner_reduce import OwnerReduce
        index = {id(p): i for i, p in enumerate(self.params)}
        segments, self._layer_of, self._layer_left = [], {}, []
        for layer, ps in enumerate(layers):
            lo = self.offsets[index[id(ps[0])]]
            n = sum(p.numel() for p in ps)
            segments.append((lo, n))
            for p in ps:
                self._layer_of[id(p)] = layer
                setattr(p, READY_ATTR, self._owner_ready)
                p.register_post_accumulate_grad_hook(self._owner_ready)
            self._layer_left.append(len(ps))
        self._layer_size = list(self._layer_left)
        self._tail = segments[-1][0] + segments[-1][1] if segments else 0
        owners = [int(layer_owner(l)) for l in range(len(layers))]
        copy_engine = self.transport == "owner-ce"  # fp32 payload, copy-engine sends
        self.owner = OwnerReduce(self.flat, segments, owners, group=self.group,
                                 transport="f32" if copy_engine else self.transport.split("-", 1)[1],
                                 copy_engine=copy_engine)
        self._reported = set()
        self._delivered = {}   # layer -> [(start, length)] stored in the owner's slot by GEMMs
        self._dirty = False    # a backward ran since zero_grad (gradient accumulation)
        self._route_ok = False
        self.fused_wgrad = (self.transport == "owner-f32"
                            and os.environ.get("RO_FUSED_WGRAD_SEND", "0") == "1"
                            and hasattr(_ext.ext(), "gemm_bf16_to"))
        if self.fused_wgrad:
            for layer, ps in enumerate(layers):
                if owners[layer] == self.owner.rank:
                    continue
                lo = segments[layer][0]
                for p in ps:
                    if p.dim() == 2:
                        start = self.offsets[index[id(p)]] - lo
                        setattr(p, ROUTE_ATTR, self._make_route(p, layer, start))

    def _make_route(self, p, layer, start):
        """dW of ``p`` computed by the package's GEMM straight into the owner's
        slot (fp32 tiles stored over NVLink from the epilogue) when this is the
        only backward of the step; False (compute locally) otherwise."""
        addr = self.owner.slot_address(layer, start)
        rows, cols, n = p.shape[0], p.shape[1], p.numel()
        C = _ext.ext()

        def route(gy2, x2):
            if not (self._armed and self._route_ok) or gy2.shape[-1] != rows or x2.shape[-1] != cols:
                return False
            if not C.gemm_bf16_to(gy2, x2, True, False, addr, cols):
                return False
            self._delivered.setdefault(layer, []).append((start, n))
            return True
        return route
    def _owner_ready(self, p):
        if not self._armed:
            self._dirty = True  # a gradient-accumulation micro-step: later GEMMs must add locally
            return
        layer = self._layer_of.get(id(p))
        if layer is None or id(p) in self._reported:
            return
        self._reported.add(id(p))
        self._layer_left[layer] -= 1
        if self._layer_left[layer] == 0:
            self.owner.send(layer, self._delivered.pop(layer, ()))

    def grad_sumsq(self):
        """Sum of squares of the averaged gradient (device scalar, identical on every
        rank) when gradients are not replicated everywhere; None otherwise."""
        if not self.owner_mode:
            return None
        from .. import _ext as ext
        tail = self.flat[self._tail:]
        owned = self.owner.owned_sumsq().reshape(1).clone()
        dist.all_reduce(owned, group=self.group)
        rest = ext.ext().multi_tensor_dot([tail], [tail], 1.0) if tail.numel() else owned.new_zeros(1)
        return (owned + rest.reshape(1)).reshape(())

    # -- overlapped buckets ----------------------------------------------------
    def _setup_buckets(self, model):
        """One bucket per ``layers.<i>.`` prefix (contiguous in the flat buffer)."""
        names = {}
        for n, p in model.named_parameters():
            names.setdefault(id(p), n)
        layer_of = []
        for p in self.params:
            parts = names.get(id(p), "").split(".")
            layer_of.append(int(parts[1]) if len(parts) > 2 and parts[0] == "layers" and parts[1].isdigit()
                            else None)
        self.bucket_ranges = []      # (lo, hi) element ranges, index = layer
        self.bucket_params = []      # parameter count per bucket
        self._bucket_of = {}
        layers = sorted({l for l in layer_of if l is not None})
        for layer in layers:
            idx = [i for i, l in enumerate(layer_of) if l == layer]
            lo = self.offsets[idx[0]]
            hi = self.offsets[idx[-1]] + self.params[idx[-1]].numel()
            if any(layer_of[i] != layer for i in range(idx[0], idx[-1] + 1)):
                raise RuntimeError("layer parameters are not contiguous in the gradient buffer")
            b = len(self.bucket_ranges)
            self.bucket_ranges.append((lo, hi))
            self.bucket_params.append(len(idx))
            for i in idx:
                self._bucket_of[id(self.params[i])] = b
        covered = set(self._bucket_of)
        self.rest = [(self.offsets[i], self.offsets[i] + p.numel()) for i, p in enumerate(self.params)
                     if id(p) not in covered]
        for p in self.params:
            if id(p) in covered:
                setattr(p, READY_ATTR, self._param_ready)
                p.register_post_accumulate_grad_hook(self._param_ready)
        self._pending = list(self.bucket_params)
        self._next = len(self.bucket_ranges) - 1
        # RO_GRAD_TRACE=1 records (bucket, parameter, next bucket to launch) per report
        self._trace = [] if os.environ.get("RO_GRAD_TRACE") == "1" else None
        self._names = {id(p): n for n, p in model.named_parameters()}

    def begin_backward(self):
        """Arm readiness tracking for the backward pass whose gradients are final."""
        if self.owner_mode:
            self._armed = True
            self._reported = set()
            self._layer_left = list(self._layer_size)
            self._delivered = {}
            self._route_ok = self.fused_wgrad and not self._dirty
            self.owner.begin()
            return
        if not self.overlap:
            return
        self._armed = True
        self._reported = set()
        if self._trace is not None:
            self._trace.clear()
        self._pending = list(self.bucket_params)
        self._next = len(self.bucket_ranges) - 1
        self._works = []

    def _param_ready(self, p):
        if not self._armed:
            return
        b = self._bucket_of.get(id(p))
        if b is None or id(p) in self._reported:
            # a weight whose gradient the GEMM accumulated also passes through
            # an AccumulateGrad node with no gradient, whose hook reports again
            return
        self._reported.add(id(p))
        if self._trace is not None:
            self._trace.append((b, self._names.get(id(p), "?"), self._next))
        self._pending[b] -= 1
        while self._next >= 0 and self._pending[self._next] <= 0:
            self._launch(self._next)
            self._next -= 1

    def _launch(self, b):
        lo, hi = self.bucket_ranges[b]
        self._works.append(dist.all_reduce(self.flat[lo:hi], op=dist.ReduceOp.AVG, group=self.group,
                                           async_op=True))

    # -- common ----------------------------------------------------------------
    def flat_covering(self):
        """The flat buffer when every managed gradient is still a view of it, else None."""
        for p, v in zip(self.params, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                return None
        return self.flat

    def zero_grad(self):
        for p, v in zip(self.params, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                p.grad = v
        self.flat.zero_()
        self._dirty = False

    def synchronize(self):
        """Average gradients across ranks (no-op for one rank)."""
        if self.world == 1:
            return
        if self.owner_mode:
            work = None
            if self._tail < self.flat.numel():
                work = dist.all_reduce(self.flat[self._tail:], op=dist.ReduceOp.AVG, group=self.group,
                                       async_op=True)
            self.owner.reduce()
            if work is not None:
                work.wait()
            self._armed = False
            self._reported = set()
            return
        if self.overlap:
            # buckets whose readiness was not reported (e.g. unused parameters)
            # are launched now, still in descending order
            while self._next >= 0:
                self._launch(self._next)
                self._next -= 1
            for lo, hi in _merge(self.rest):
                self._works.append(dist.all_reduce(self.flat[lo:hi], op=dist.ReduceOp.AVG,
                                                   group=self.group, async_op=True))
            for w in self._works:
                w.wait()
            self._works = []
            self._armed = False
            self._reported = set()
            self._pending = list(self.bucket_params)
            self._next = len(self.bucket_ranges) - 1
            return
        if self.communicator is not None:
            self.communicator.all_reduce_mean_(self.flat)
            return
        for start in range(0, self.flat.numel(), self.bucket_elems):
            chunk = self.flat[start: start + self.bucket_elems]
            dist.all_reduce(chunk, op=dist.ReduceOp.SUM, group=self.group)
        self.flat.div_(self.world)


def _merge(ranges):
    out = []
    for lo, hi in sorted(ranges):
        if out and out[-1][1] == lo:
            out[-1] = (out[-1][0], hi)
        else:
            out.append((lo, hi))
    return out
