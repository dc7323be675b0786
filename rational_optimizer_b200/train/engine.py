"""One optimizer step of the shared trainer, as a reusable engine.

``TrainEngine.step(batches, lr)`` performs what the reference trainer's hot
loop does per step (training/train.py:2814-2932): set the scheduled LR on
every group, zero gradients, forward + loss + backward for each micro-batch,
average gradients across data-parallel ranks, clip to ``grad_clip`` and report
the realised pre-clip norm to the clipping observer (TILLER), then step the
optimizer.  The returned loss stays on the device; callers decide when to
read it (the reference synchronises on ``loss.item()`` every micro-batch).
"""
from __future__ import annotations

import math
import os

import torch

from ..parallel.grad_sync import GradientSynchronizer
from .graphs import StepGraph, graphs_requested


def learning_rate(step, *, lr, min_lr, warmup_steps, total_steps):
    """Linear warm-up then cosine decay to ``min_lr`` (train.py:1889-1895)."""
    if warmup_steps > 0 and step < warmup_steps:
        return lr * float(step + 1) / float(warmup_steps)
    progress = (step - warmup_steps) / max(1, total_steps - warmup_steps)
    progress = min(1.0, max(0.0, progress))
    return min_lr + 0.5 * (1.0 + math.cos(math.pi * progress)) * (lr - min_lr)


def clip_grad_norm(params, max_norm, flat=None, sumsq=None):
    """Global L2 norm of all gradients (fp32) and in-place clipping; returns the device norm.

    ``flat``: the single fp32 buffer every gradient is a view of (the data-
    parallel synchroniser's); on CUDA the norm is then one fixed-order
    reduction kernel over the buffer and the clip one scaling pass, instead of
    per-tensor norms (torch.nn.utils.clip_grad_norm_, used by the reference
    trainer, training/train.py:957).  ``sumsq``: the squared norm when the
    caller has it already (reduce-to-owner: the buffer then holds averaged
    gradients only for this rank's layers, so the norm comes from the owners'
    partial sums).
    """
    if flat is not None and flat.is_cuda and flat.dtype == torch.float32 and _has_dot():
        from .. import _ext
        C = _ext.ext()
        if sumsq is None:
            sumsq = C.multi_tensor_dot([flat], [flat], 1.0)
        if max_norm > 0:
            C.clip_scale_(flat, sumsq.reshape(1), float(max_norm))
        return sumsq.sqrt()
    grads = [p.grad for p in params if p.grad is not None]
    norms = torch._foreach_norm(grads, 2.0)
    total = torch.linalg.vector_norm(torch.stack([n.float() for n in norms]), 2.0)
    if max_norm > 0:
        coef = (float(max_norm) / (total + 1e-6)).clamp(max=1.0)
        torch._foreach_mul_(grads, coef)
    return total


def _has_dot():
    from .. import _ext
    return _ext.available() and hasattr(_ext.ext(), "multi_tensor_dot")


class TrainEngine:
    def __init__(self, model, optimizer, *, grad_clip=1.0, grad_accum=1, synchronizer=None,
                 clip_observer=None):
        self.model = model
        self.optimizer = optimizer
        self.grad_clip = float(grad_clip)
        self.grad_accum = int(grad_accum)
        self.sync = synchronizer if synchronizer is not None else GradientSynchronizer(model)
        self.clip_observer = clip_observer
        if clip_observer is None and hasattr(optimizer, "record_realized_clipping"):
            self.clip_observer = optimizer
        self.last_grad_norm = None
        self._graphs = {}  # "plain" / "refresh" -> StepGraph
        self._graph_state = "off" if not graphs_requested() else "pending"
        self._eligible_steps = 0

    def _graph_kind(self, batches):
        """``"plain"`` or ``"refresh"`` when this step may replay a captured graph, else None."""
        if self._graph_state in ("off", "failed") or len(batches) != 1:
            return None
        if self.sync.world > 1 and os.environ.get("RO_CUDA_GRAPH_DIST", "1") != "1":
            return None
        x, y = batches[0]
        if not x.is_cuda:
            return None
        # only optimizers that say which steps record probes in the forward/backward
        probes = getattr(self.optimizer, "eager_step_required", None)
        if probes is None:
            return None
        kind = "plain"
        if probes():
            if os.environ.get("RO_REFRESH_GRAPH", "1") != "1" or self._recorder() is None:
                return None
            kind = "refresh"
        if any(getattr(m, "_rlb_optimizer_track_stats", False) for m in self.model.modules()):
            return None
        graph = self._graphs.get("plain")
        if graph is not None and not graph.matches(x, y):
            return None
        return kind

    def _recorder(self):
        get = getattr(self.optimizer, "probe_recorder", None)
        return get() if get is not None else None

    def _capture_graphs(self, x, y):
        recorder = self._recorder()
        graphs = {"plain": StepGraph(self.model, self.sync, x, y, recorder=recorder, probes=False)}
        if recorder is not None and os.environ.get("RO_REFRESH_GRAPH", "1") == "1":
            # the plain graph's capture warmed everything up; one warm-up
            # pass initialises the probe hooks' own work
            graphs["refresh"] = StepGraph(self.model, self.sync, x, y, warmup=1, recorder=recorder,
                                          probes=True)
        for g in graphs.values():
            g.capture()
        return graphs

    def _graphed_forward_backward(self, x, y, kind):
        """The loss via a captured graph, or None (eager path) when capture is not possible."""
        if any(g.graph is None for g in self._graphs.values()):
            self._graphs = {}  # released (process-group teardown): capture again if stepped
        if not self._graphs:
            self._eligible_steps += 1
            # one complete step first (lazily created optimizer state, weight
            # casts); capture on the second, so any run with three or more
            # warm-up steps has captured before it is timed
            if self._eligible_steps < 2:
                return None
            try:
                self._graphs = self._capture_graphs(x, y)
                self._graph_state = "on"
            except Exception as exc:  # an operation that cannot be captured
                for g in self._graphs.values():
                    g.release()
                self._graphs = {}
                self._graph_state = "failed"
                self.graph_error = f"{type(exc).__name__}: {exc}"
                recorder = self._recorder()
                if recorder is not None:
                    recorder.take_probe_records()
                self.sync.zero_grad()
                return None
        graph = self._graphs.get(kind)
        if graph is None:
            return None
        self.sync.zero_grad()
        return graph.replay(x, y)

    def set_lr(self, lr):
        for group in self.optimizer.param_groups:
            group["lr"] = lr * float(group.get("lr_scale", 1.0))

    def step(self, batches, lr=None):
        """``batches``: list of ``grad_accum`` (x, y) device tensors.  Returns the mean loss."""
        if len(batches) != self.grad_accum:
            raise ValueError("expected one batch per micro-step")
        if lr is not None:
            self.set_lr(lr)
        kind = self._graph_kind(batches)
        if kind is not None:
            loss = self._graphed_forward_backward(*batches[0], kind)
            if loss is not None:
                return self._finish(loss)
        self.sync.zero_grad()
        total = None
        for i, (x, y) in enumerate(batches):
            loss = self.model.forward_loss(x, y)
            if i == len(batches) - 1:
                self.sync.begin_backward()
            (loss / self.grad_accum).backward()
            total = loss.detach() if total is None else total + loss.detach()
        self.sync.synchronize()
        return self._finish(total / self.grad_accum)

    def _finish(self, loss):
        norm = clip_grad_norm(self.sync.params, self.grad_clip, self.sync.flat_covering(),
                              sumsq=self.sync.grad_sumsq())
        self.last_grad_norm = norm
        if self.clip_observer is not None:
            self.clip_observer.record_realized_clipping(norm, self.grad_clip)
        self.optimizer.step()
        return loss
