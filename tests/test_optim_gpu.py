"""Optimizer kernels against their PyTorch definitions."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200.optim.adamw import FusedAdamW


def test_fused_adamw_matches_torch():
    torch.manual_seed(0)
    shapes = [(1000, 64), (64,), (3, 5, 7), (50304, 16)]
    ps = [torch.randn(s, device="cuda") for s in shapes]
    qs = [p.clone() for p in ps]
    opt_a = FusedAdamW([{"params": ps[:2], "weight_decay": 0.1}, {"params": ps[2:], "weight_decay": 0.0}],
                       lr=1e-3, betas=(0.9, 0.95), eps=1e-8)
    opt_b = torch.optim.AdamW([{"params": qs[:2], "weight_decay": 0.1}, {"params": qs[2:], "weight_decay": 0.0}],
                              lr=1e-3, betas=(0.9, 0.95), eps=1e-8, foreach=False)
    for _ in range(5):
        for p, q in zip(ps, qs):
            g = torch.randn_like(p)
            p.grad = g.clone()
            q.grad = g.clone()
        opt_a.step()
        opt_b.step()
    for p, q in zip(ps, qs):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
    sa, sb = opt_a.state_dict(), opt_b.state_dict()
    for k in sa["state"]:
        for kk in ("exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(sa["state"][k][kk], sb["state"][k][kk], rtol=1e-5, atol=1e-7)
        assert float(sa["state"][k]["step"]) == float(sb["state"][k]["step"])
