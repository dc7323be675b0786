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


class _SequentialSteps:
    """The TILLER composite stepped child by child, without the side-stream ledger."""

    def __init__(self, opt):
        self.opt = opt

    def __getattr__(self, name):
        return getattr(self.opt, name)

    def step(self):
        for child in self.opt.optimizers:
            child.step()


def test_side_stream_ledger_matches_sequential_steps():
    args = _args()
    torch.manual_seed(0)
    base = CausalTransformer(args, 300).cuda().set_compute_dtype(torch.float32)
    m_seq, m_def = copy.deepcopy(base), copy.deepcopy(base)
    o_seq = composite.configure_optimizer(m_seq, args)
    o_def = composite.configure_optimizer(m_def, args)
    e_seq, e_def = TrainEngine(m_seq, _SequentialSteps(o_seq)), TrainEngine(m_def, o_def)
    gen = torch.Generator().manual_seed(11)
    for _ in range(10):
        t = torch.randint(0, 300, (4, 65), generator=gen).cuda()
        e_seq.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
        e_def.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
    assert o_def.router._fast_ledger_ok() and o_def.router._side_stream is not None
    assert o_def.router._pending_apply is None
    for (n, a), (_, b) in zip(m_seq.named_parameters(), m_def.named_parameters()):
        assert torch.equal(a, b), n


def _ext():
    from rational_optimizer_b200._ext import ext
    return ext()


@pytest.mark.parametrize("P,Q,transpose", [(64, 200, False), (40, 36, False), (128, 192, True),
                                           (72, 40, True), (40, 36, True)])
def test_nesterov_kernel_matches_torch(P, Q, transpose):
    torch.manual_seed(P + Q)
    mu = 0.95
    grads = [torch.randn(P, Q, device="cuda") for _ in range(3)]
    bufs = [torch.randn(P, Q, device="cuda") for _ in range(3)]
    expect_buf = [torch.lerp(b, g, 1 - mu) for b, g in zip(bufs, grads)]
    expect_m = torch.stack([torch.lerp(g, b, mu) for g, b in zip(grads, expect_buf)])
    expect_g = torch.stack(grads)
    if transpose:
        expect_m, expect_g = expect_m.transpose(1, 2), expect_g.transpose(1, 2)
    m, g, m16 = _ext().tiller_nesterov(grads, bufs, transpose, mu)
    for b, e in zip(bufs, expect_buf):
        torch.testing.assert_close(b, e, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(m, expect_m, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(g, expect_g, rtol=0, atol=0)
    torch.testing.assert_close(m16, m.to(torch.bfloat16), rtol=0, atol=0)
    torch.testing.assert_close(m16.float(), expect_m, rtol=8e-3, atol=1e-7)


@pytest.mark.parametrize("shape", [(5, 256, 1024), (3, 40, 36), (2, 7, 9)])
def test_ns_normalize_matches_torch(shape):
    torch.manual_seed(1)
    x = (torch.randn(shape, device="cuda") * 3).to(torch.bfloat16)
    norm = torch.linalg.vector_norm(x.float(), dim=(-2, -1), keepdim=True).clamp_min(1e-7)
    expect = (x.float() / norm.to(torch.bfloat16).float()).to(torch.bfloat16)
    got = _ext().ns_normalize(x)
    torch.testing.assert_close(got.float(), expect.float(), rtol=8e-3, atol=0)


def test_multi_tensor_dot_matches_torch():
    torch.manual_seed(2)
    a = [torch.randn(s, device="cuda") for s in ((1024, 4608), (37,), (3, 5, 7), (4096,))]
    b = [torch.randn_like(t) for t in a]
    got = _ext().multi_tensor_dot(a, b, 0.1)
    expect = sum((x.double() * y.double()).sum() for x, y in zip(a, b)) * 0.1
    assert abs(float(got) - float(expect)) <= 1e-4 * max(1.0, abs(float(expect)))
