"""Per-phase device time of training steps (tracing without a profiler).

The reference times whole steps on the host and the optimizer step with CUDA
events on rank 0 only (training/train.py:2764-2773, 2816, 2929-2932).  Here
:class:`PhaseTimer` places markers on the launching stream around the parts
of a :class:`~rational_optimizer_b200.train.engine.TrainEngine` step - the
forward/backward (with the gradient reduction when it is not captured in the
step graph), the reduction wait, each optimizer child, and the TILLER
router's deferred apply - and reports the median time between consecutive
markers, reduced with MAX over ranks.  On CUDA the markers are events, so
the split is device time and the host may run ahead; on the CPU they are
host clock readings.

    timer = PhaseTimer.attach(engine)
    for batch in batches:
        timer.begin_step(); engine.step([batch]); timer.end_step()
    print(timer.summary())

``python -m rational_optimizer_b200.utils.step_phases`` runs the 18-layer
GRAIN + TILLER training step on synthetic tokens and prints one JSON line per
phase (``torchrun`` for several GPUs).
"""
from __future__ import annotations

import argparse
import json
import time

import torch
import torch.distributed as dist

# the 18-layer GRAIN model of the headline training benchmark
MODEL = dict(layers=18, d_model=1024, heads=16, ffn_dim=3072, seq_len=1024, activation="grain",
             rational_init="silu", rational_group_size=256, rational_max_groups=32,
             rational_basis_eps=1e-6, init_std=0.02)
VOCAB = 50304


class PhaseTimer:
    def __init__(self, device=None):
        self.device = torch.device(device) if device is not None else None
        self.cuda = self.device is not None and self.device.type == "cuda"
        self._kind = None
        self._host0 = 0.0
        self._marks = []
        self._samples = {}
        self._patched = []

    # -- markers ------------------------------------------------------------
    def mark(self, name):
        if self.cuda and torch.cuda.is_current_stream_capturing():
            return  # inside a step-graph capture: its replays carry no markers
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record(torch.cuda.current_stream(self.device))
            self._marks.append((name, e))
        else:
            self._marks.append((name, time.perf_counter()))

    def wrap(self, obj, attr, name):
        """Mark entry (``name>``) and exit (``name<``) of ``obj.attr`` (instance patch)."""
        original = getattr(obj, attr)

        def timed(*args, **kwargs):
            self.mark(name + ">")
            try:
                return original(*args, **kwargs)
            finally:
                self.mark(name + "<")

        setattr(obj, attr, timed)
        self._patched.append((obj, attr, original))

    @classmethod
    def attach(cls, engine):
        """Markers around the reduction wait and every optimizer (child) step."""
        first = next(iter(engine.model.parameters()))
        timer = cls(first.device)
        timer.wrap(engine.sync, "synchronize", "grad_sync")
        opt = engine.optimizer
        children = getattr(opt, "optimizers", None)
        if children:
            for i, child in enumerate(children):
                timer.wrap(child, "step", f"{type(child).__name__}[{i}]")
            router = getattr(opt, "router", None)
            if router is not None and hasattr(router, "finish_step"):
                timer.wrap(router, "finish_step", "router_apply")
        else:
            timer.wrap(opt, "step", "optimizer")
        return timer

    def detach(self):
        for obj, attr, original in reversed(self._patched):
            setattr(obj, attr, original)
        self._patched = []

    # -- steps --------------------------------------------------------------
    def begin_step(self, kind=None):
        """Open a step; ``kind`` (e.g. ``"plain"`` / ``"refresh"``) keys its samples separately."""
        self._marks = []
        self._kind = kind
        self._host0 = time.perf_counter()
        self.mark("step")

    def end_step(self, record=True):
        """Close the step; ``record=False`` discards it (warm-up)."""
        host_ms = (time.perf_counter() - self._host0) * 1000.0
        self.mark("end")
        if self.cuda:
            torch.cuda.synchronize(self.device)
        if not record:
            return
        prefix = f"{self._kind}:" if self._kind else ""
        for (a, ta), (b, tb) in zip(self._marks, self._marks[1:]):
            self._samples.setdefault(f"{prefix}{a}->{b}", []).append(self._elapsed_ms(ta, tb))
        self._samples.setdefault(f"{prefix}total", []).append(
            self._elapsed_ms(self._marks[0][1], self._marks[-1][1]))
        # host time to enqueue the step (no synchronisation inside the step)
        self._samples.setdefault(f"{prefix}host_enqueue", []).append(host_ms)

    def _elapsed_ms(self, a, b):
        return a.elapsed_time(b) if self.cuda else (b - a) * 1000.0

    def summary(self, group=None):
        """{interval: median ms}, MAX over ranks when a process group is up.

        Every rank must have recorded the same interval names (the same step
        kinds), since the reduction is one collective over the sorted names.
        """
        names = sorted(self._samples)
        med = []
        for n in names:
            v = sorted(self._samples[n])
            med.append(v[len(v) // 2])
        if dist.is_available() and dist.is_initialized() and names:
            t = torch.tensor(med, dtype=torch.float64,
                             device=self.device if self.cuda else torch.device("cpu"))
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            med = t.tolist()
        return dict(zip(names, med))


def step_kind(engine):
    """``"refresh"`` when the next step of ``engine`` runs the TILLER response refresh, else ``"plain"``."""
    probe = getattr(engine.optimizer, "eager_step_required", None)
    return "refresh" if probe is not None and probe() else "plain"


def main(argv=None):
    from ..models.transformer import CausalTransformer, model_args
    from ..optim import composite
    from ..parallel import param_ready
    from ..parallel.dist import cleanup_distributed, setup_distributed
    from ..parallel.grad_sync import GradientSynchronizer
    from ..train.data import PinnedBatcher, zipf_tokens
    from ..train.engine import TrainEngine

    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=MODEL["layers"])
    ap.add_argument("--global-batch", type=int, default=32)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--warmup", type=int, default=4)
    a = ap.parse_args(argv)
    info = setup_distributed()
    cfg = dict(MODEL, layers=a.layers)
    args = model_args(**cfg, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1, muon_momentum=0.95,
                      muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(1337)
    model = CausalTransformer(args, VOCAB).to(info.device)
    if info.is_distributed:
        for p in model.parameters():
            dist.broadcast(p.data, 0)
    engine = TrainEngine(model, composite.configure_optimizer(model, args), grad_clip=1.0,
                         synchronizer=GradientSynchronizer(model))
    tokens = zipf_tokens(4_000_000, VOCAB, alpha=1.1, seed=0)
    batcher = PinnedBatcher(tokens, a.global_batch // info.world_size, cfg["seq_len"], seed=0,
                            rank=info.rank)
    staged = [batcher.to_device(info.device, batcher.next_host().clone()) for _ in range(4)]
    timer = PhaseTimer.attach(engine)
    for i in range(a.warmup + a.steps):
        timer.begin_step(step_kind(engine))
        engine.step([staged[i % len(staged)]], lr=3e-4)
        param_ready.wait_all()  # owners' deferred broadcasts inside the step
        timer.end_step(record=i >= a.warmup)
    result = timer.summary()
    timer.detach()
    if info.rank == 0:
        for name, ms in result.items():
            print(json.dumps({"phase": name, "median_ms": round(ms, 3), "ranks": info.world_size}))
    del engine, staged
    cleanup_distributed(info)


if __name__ == "__main__":
    main()
