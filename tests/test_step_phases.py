"""PhaseTimer splits engine steps into consecutive intervals (CPU, host clock)."""
import torch

from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
from rational_optimizer_b200.optim import composite
from rational_optimizer_b200.parallel.grad_sync import GradientSynchronizer
from rational_optimizer_b200.train.engine import TrainEngine
from rational_optimizer_b200.utils.step_phases import PhaseTimer


def test_phase_timer_on_tiller_engine():
    args = model_args(layers=2, d_model=64, heads=4, ffn_dim=128, seq_len=16, activation="grain",
                      rational_group_size=32, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(0)
    model = CausalTransformer(args, 100)
    engine = TrainEngine(model, composite.configure_optimizer(model, args),
                         synchronizer=GradientSynchronizer(model))
    original = engine.optimizer.optimizers[0].step
    timer = PhaseTimer.attach(engine)
    gen = torch.Generator().manual_seed(1)
    for i in range(4):
        t = torch.randint(0, 100, (2, 17), generator=gen)
        timer.begin_step()
        engine.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
        timer.end_step(record=i == 3)  # one recorded step: its intervals add up exactly
    out = timer.summary()
    timer.detach()
    assert engine.optimizer.optimizers[0].step == original
    names = [n for n in out if n not in ("total", "host_enqueue")]
    assert "step->grad_sync>" in names and "router_apply>->router_apply<" in names
    assert any(n.startswith("TILLERRouter[0]>") for n in names)
    assert all(v >= 0.0 for v in out.values())
    # consecutive intervals add up to the whole step
    assert abs(sum(out[n] for n in names) - out["total"]) <= 1e-6 * out["total"] + 1e-6


def test_phase_timer_keys_samples_by_step_kind():
    from rational_optimizer_b200.utils.step_phases import step_kind

    args = model_args(layers=2, d_model=64, heads=4, ffn_dim=128, seq_len=16, activation="grain",
                      rational_group_size=32, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(0)
    model = CausalTransformer(args, 100)
    engine = TrainEngine(model, composite.configure_optimizer(model, args),
                         synchronizer=GradientSynchronizer(model))
    timer = PhaseTimer.attach(engine)
    gen = torch.Generator().manual_seed(1)
    kinds = []
    for _ in range(10):
        t = torch.randint(0, 100, (2, 17), generator=gen)
        kinds.append(step_kind(engine))
        timer.begin_step(kinds[-1])
        engine.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
        timer.end_step()
    out = timer.summary()
    timer.detach()
    # the response refresh runs on router transitions 0 and 8 (cadence 8)
    assert kinds == ["refresh"] + ["plain"] * 7 + ["refresh", "plain"]
    assert "refresh:total" in out and "plain:total" in out
    assert "plain:host_enqueue" in out and "total" not in out


def test_composite_step_matches_children_in_order():
    """The TILLER composite (router with deferred apply, then attention and
    AdamW, then the router's apply) equals stepping the children in order."""
    import copy

    args = model_args(layers=2, d_model=64, heads=4, ffn_dim=128, seq_len=16, activation="grain",
                      rational_group_size=32, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(0)
    base = CausalTransformer(args, 100)
    models = [copy.deepcopy(base), copy.deepcopy(base)]
    opts = [composite.configure_optimizer(m, args) for m in models]

    class Sequential:
        def __init__(self, opt):
            self.opt = opt

        def __getattr__(self, name):
            return getattr(self.opt, name)

        def step(self):
            for child in self.opt.optimizers:
                child.step()

    engines = [TrainEngine(models[0], opts[0], synchronizer=GradientSynchronizer(models[0])),
               TrainEngine(models[1], Sequential(opts[1]), synchronizer=GradientSynchronizer(models[1]))]
    gen = torch.Generator().manual_seed(2)
    for _ in range(10):
        t = torch.randint(0, 100, (2, 17), generator=gen)
        for e in engines:
            e.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
    assert opts[0].router._pending_apply is None
    for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
        assert torch.equal(a, b), n
