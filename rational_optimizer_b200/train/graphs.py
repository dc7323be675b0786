"""CUDA graph of one training micro-batch: forward, backward and gradient reduction.

With one process per GPU the host enqueues about a thousand kernels per step
for the 18-layer model (autograd bookkeeping, Python-level ops); at the
per-GPU batch of an 8-GPU run that host time exceeds the GPU time of the
forward and backward.  ``StepGraph`` captures ``forward_loss`` +
``backward`` + the data-parallel gradient reduction once (static input
buffers, weights cast to bf16 inside the graph because they change between
replays) and replays it on later steps; the optimizer step stays eager.

TILLER's response-probe refresh steps get a graph of their own: with a
``recorder`` (the optimizer child whose hooks record probe rows) and
``probes=True`` the capture runs with the hooks forced on, and the probe
records it made - index selects of fixed rows into tensors owned by the
graph - are handed back to the recorder after every replay; the plain
step's graph is captured with the hooks forced off.  Steps that still need host-side work
inside the forward or backward (telemetry statistics, a different
micro-batch shape) run eagerly; the graphs are kept for the next eligible
step.  Capture failures (an operation that cannot be recorded) disable
graphs for the run and the engine continues eagerly.
"""
from __future__ import annotations

import contextlib
import os
import weakref

import torch

from ..ops import linear as _linear
from ..parallel import param_ready


def graphs_requested() -> bool:
    return os.environ.get("RO_CUDA_GRAPH", "1") != "0"


_LIVE = weakref.WeakSet()


def release_all() -> None:
    """Free every captured step graph of this process.

    A graph that recorded NCCL collectives must be freed before the process
    group is destroyed; otherwise process exit waits on it indefinitely.
    ``parallel.dist.cleanup_distributed`` calls this first.
    """
    for g in list(_LIVE):
        g.release()


class StepGraph:
    def __init__(self, model, sync, x, y, *, warmup: int = 3, recorder=None, probes=False):
        self.model = model
        self.sync = sync
        self.x = x.detach().clone()
        self.y = y.detach().clone()
        self.warmup = int(warmup)
        self.recorder = recorder
        self.probes = bool(probes) and recorder is not None
        self.records = None
        self.graph = None
        self.loss = None
        self.replays = 0
        self._keep = []
        self._pullers = []
        self._captured_events = []
        _LIVE.add(self)

    def release(self):
        """Free the captured graph and its pinned tensors (replay needs a new capture)."""
        if self.graph is not None:
            torch.cuda.synchronize(self.x.device)
            self.graph.reset()
        self.graph = None
        self.loss = None
        self.records = None
        self._keep = []

    def matches(self, x, y) -> bool:
        return (x.shape == self.x.shape and y.shape == self.y.shape and x.dtype == self.x.dtype
                and y.dtype == self.y.dtype and x.device == self.x.device)

    def _one(self, pull=False):
        pulled = []
        if pull:
            # replicate the owners' weights inside the graph: each layer's
            # forward waits only for the copy from its own owner
            param_ready.claim_pullers()
            for obj in self._pullers:
                ev = obj.pull()
                if ev is not None:
                    pulled.append(ev)
        loss = self.model.forward_loss(self.x, self.y)
        self.sync.begin_backward()
        loss.backward()
        self.sync.synchronize()
        if pulled:
            torch.cuda.current_stream(self.x.device).wait_stream(param_ready.side_stream(self.x.device))
            self._captured_events = pulled
        return loss

    def capture(self):
        """Capture with the recorder's probe hooks forced on (``probes``) or off."""
        forced = (self.recorder.probes_forced(self.probes) if self.recorder is not None
                  else contextlib.nullcontext())
        with forced:
            self._capture()

    def _capture(self):
        self._pullers = param_ready.pullers()
        self._captured_events = []
        param_ready.wait_all()
        side = torch.cuda.Stream(device=self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self.sync.zero_grad()
                self._one()
                if self.probes:
                    self.recorder.take_probe_records()  # warm-up records are not used
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        self.sync.zero_grad()
        graph = torch.cuda.CUDAGraph()
        _linear.capture_casts(True, self._keep)
        # with several ranks the process group's watchdog thread keeps querying
        # its events while we capture: restrict capture checks to this thread
        mode = "thread_local" if self.sync.world > 1 else "global"
        try:
            with torch.cuda.graph(graph, capture_error_mode=mode):
                self.loss = self._one(pull=bool(self._pullers)).detach()
        finally:
            _linear.capture_casts(False)
            param_ready.forget_events(self._captured_events)
            if self.probes:
                self.records = self.recorder.take_probe_records()
        self.graph = graph

    def replay(self, x, y):
        if self._pullers:
            param_ready.claim_pullers()  # the graph pulls the owners' weights itself
        param_ready.wait_all()
        if x.data_ptr() != self.x.data_ptr():
            self.x.copy_(x, non_blocking=True)
        if y.data_ptr() != self.y.data_ptr():
            self.y.copy_(y, non_blocking=True)
        self.graph.replay()
        self.replays += 1
        if self.probes:
            self.recorder.restore_probe_records(self.records)
        return self.loss.clone()  # the graph's output tensor is overwritten by the next replay
