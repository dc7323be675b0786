"""Published optimizer baselines against the reference implementations (CPU, fp32)."""
import importlib
from types import SimpleNamespace

import pytest
import torch

from rational_optimizer_b200.optim import baselines
from reference_oracle import require_reference


def _params(seed):
    gen = torch.Generator().manual_seed(seed)
    shapes = [(160, 136), (96, 48), (130,), (7, 5)]
    return [torch.randn(*s, generator=gen) for s in shapes]


def _grads(seed, step, params):
    gen = torch.Generator().manual_seed(seed * 1000 + step)
    return [torch.randn(p.shape, generator=gen) * 0.1 for p in params]


CASES = {
    "Lion": dict(lr=1e-3, betas=(0.9, 0.99), weight_decay=0.1),
    "AdEMAMix": dict(lr=1e-3, betas=(0.9, 0.999, 0.9999), eps=1e-8, weight_decay=0.1, alpha=5.0,
                     beta3_warmup=4, alpha_warmup=3),
    "ScheduleFreeAdamW": dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.1,
                              warmup_steps=2),
    "CAMEStyleAdamW": dict(lr=1e-3, betas=(0.9, 0.999, 0.999), eps=1e-8, weight_decay=0.1,
                           factored_min_dim=64, clip_threshold=1.0),
    "SOAPStyleAdamW": dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                           precondition_frequency=3, large_side_identity_threshold=150),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_baseline_matches_reference(name):
    require_reference()
    ref_mod = importlib.import_module("training.baseline_optimizers")
    ours_p = [p.clone().requires_grad_(True) for p in _params(3)]
    ref_p = [p.clone().requires_grad_(True) for p in _params(3)]
    groups = lambda ps: [{"params": ps[:2], "weight_decay": CASES[name]["weight_decay"]},
                         {"params": ps[2:], "weight_decay": 0.0}]
    kw = dict(CASES[name])
    kw.pop("weight_decay")
    ours = getattr(baselines, name)(groups(ours_p), **kw)
    ref = getattr(ref_mod, name)(groups(ref_p), **kw)
    for step in range(6):
        for ps in (ours_p, ref_p):
            for p, g in zip(ps, _grads(5, step, ps)):
                p.grad = g.clone()
        ours.step()
        ref.step()
        for a, b in zip(ours_p, ref_p):
            torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-5, atol=2e-6)
    # identical state layout, so state dicts interchange
    sd = ours.state_dict()
    assert sd["state"].keys() == ref.state_dict()["state"].keys()
    for k, v in sd["state"].items():
        assert set(v) == set(ref.state_dict()["state"][k])


def test_ademamix_warmup_resolution():
    assert baselines.resolve_ademamix_warmup(-1, 1000) == 150
    assert baselines.resolve_ademamix_warmup(-1, 2) == 1
    assert baselines.resolve_ademamix_warmup(0, 1000) is None
    assert baselines.resolve_ademamix_warmup(None, 1000) is None
    assert baselines.resolve_ademamix_warmup(25, 1000) == 25


def test_build_from_trainer_flags():
    args = SimpleNamespace(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, steps=100,
                           ademamix_beta3=0.9999, ademamix_alpha=5.0, ademamix_beta3_warmup_steps=-1,
                           ademamix_alpha_warmup_steps=-1, schedule_free_beta1=0.9,
                           schedule_free_warmup_steps=0, came_beta3=0.999, came_confidence_scale=1.0,
                           came_confidence_min=0.25, came_confidence_max=4.0, factored_min_dim=128,
                           factored_clip_threshold=1.0, soap_precondition_frequency=50,
                           soap_large_side_identity_threshold=2048, soap_one_sided=False)
    p = torch.nn.Parameter(torch.randn(4, 4))
    for name, cls in [("lion", baselines.Lion), ("ademamix", baselines.AdEMAMix),
                      ("schedule_free_adamw", baselines.ScheduleFreeAdamW),
                      ("adafactor_came", baselines.CAMEStyleAdamW),
                      ("soap_adamw", baselines.SOAPStyleAdamW)]:
        opt = baselines.build(name, [{"params": [p], "weight_decay": 0.1}], args)
        assert isinstance(opt, cls)
    opt = baselines.build("ademamix", [{"params": [p]}], args)
    assert opt.param_groups[0]["beta3_warmup"] == 15
