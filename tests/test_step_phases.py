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
        timer.end_step(record=i >= 1)
    out = timer.summary()
    timer.detach()
    assert engine.optimizer.optimizers[0].step == original
    names = [n for n in out if n != "total"]
    assert "step->grad_sync>" in names and "router_apply>->router_apply<" in names
    assert any(n.startswith("TILLERRouter[0]>") for n in names)
    assert all(v >= 0.0 for v in out.values())
    # consecutive intervals add up to the whole step
    assert abs(sum(out[n] for n in names) - out["total"]) <= 0.05 * out["total"] + 1e-3
