"""The fused CUDA TILLER path against the PyTorch restatement on the same GPU."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
from rational_optimizer_b200.optim import composite
from rational_optimizer_b200.train.engine import TrainEngine


def _args():
    return model_args(layers=2, d_model=256, heads=4, ffn_dim=512, seq_len=64, activation="grain",
                      rational_group_size=128, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)


def test_fused_tiller_matches_torch_path():
    args = _args()
    torch.manual_seed(0)
    base = CausalTransformer(args, 300).cuda().set_compute_dtype(torch.float32)
    m_ref = copy.deepcopy(base)
    m_fus = copy.deepcopy(base)
    o_ref = composite.configure_optimizer(m_ref, args)
    o_fus = composite.configure_optimizer(m_fus, args)
    o_ref.router._force_torch = True
    e_ref, e_fus = TrainEngine(m_ref, o_ref), TrainEngine(m_fus, o_fus)
    gen = torch.Generator().manual_seed(7)
    for _ in range(10):
        t = torch.randint(0, 300, (4, 65), generator=gen).cuda()
        e_ref.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
        e_fus.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
    assert o_fus.router._fused_ok is True and o_ref.router._fused_ok is False
    for (n, a), (_, b), (_, c) in zip(base.named_parameters(), m_ref.named_parameters(),
                                      m_fus.named_parameters()):
        moved = (b - a).abs().max().item()
        diff = (c - b).abs().max().item()
        assert diff <= 0.05 * moved + 1e-6, (n, diff, moved)
    ra, fa = o_ref.router.anchor, o_fus.router.anchor
    for key in ("factorized_adaptive_tangent_rows_row_second_moment",
                "factorized_adaptive_tangent_columns_column_second_moment"):
        torch.testing.assert_close(fa[key], ra[key], rtol=1e-3, atol=1e-9)
