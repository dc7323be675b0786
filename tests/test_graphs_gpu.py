"""CUDA-graph replay of the forward/backward gives the eager trajectory bit for bit."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
from rational_optimizer_b200.optim import composite
from rational_optimizer_b200.parallel import param_ready
from rational_optimizer_b200.parallel.grad_sync import GradientSynchronizer
from rational_optimizer_b200.train.engine import TrainEngine
from rational_optimizer_b200.train.graphs import release_all


def _args():
    return model_args(layers=2, d_model=512, heads=8, ffn_dim=1024, seq_len=256, activation="grain",
                      rational_group_size=256, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)


def test_graph_replay_matches_eager(monkeypatch):
    args = _args()
    torch.manual_seed(0)
    base = CausalTransformer(args, 1000).cuda()
    runs = []
    for graphs in ("0", "1"):
        monkeypatch.setenv("RO_CUDA_GRAPH", graphs)
        m = copy.deepcopy(base)
        opt = composite.configure_optimizer(m, args)
        eng = TrainEngine(m, opt, grad_clip=1.0, synchronizer=GradientSynchronizer(m))
        gen = torch.Generator().manual_seed(3)
        losses = []
        refresh_replays = 0
        for i in range(20):  # response refreshes at steps 0 (eager), 8 and 16 (refresh graph)
            if graphs == "1" and i == 10:
                # teardown path: graphs are freed, the next step captures again
                refresh_replays += eng._graphs["refresh"].replays
                release_all()
                assert all(g.graph is None for g in eng._graphs.values())
            t = torch.randint(0, 1000, (4, 257), generator=gen).cuda()
            losses.append(eng.step([(t[:, :-1], t[:, 1:])], lr=3e-4).item())
        param_ready.wait_all()
        torch.cuda.synchronize()
        if graphs == "1":
            refresh_replays += eng._graphs["refresh"].replays
            assert refresh_replays == 2
        runs.append((losses, [p.detach().clone() for p in m.parameters()], eng._graph_state))
    assert runs[0][2] == "off" and runs[1][2] == "on", (runs[0][2], runs[1][2])
    assert runs[0][0] == runs[1][0]
    for a, b in zip(runs[0][1], runs[1][1]):
        assert torch.equal(a, b)


def test_bf16_weight_casts_follow_optimizer_updates(monkeypatch):
    """Every optimizer (custom kernels included) bumps parameter versions, so the
    cached bf16 casts used by the GEMMs always hold the current weights."""
    monkeypatch.setenv("RO_CUDA_GRAPH", "0")
    args = _args()
    torch.manual_seed(0)
    m = CausalTransformer(args, 1000).cuda()
    opt = composite.configure_optimizer(m, args)
    eng = TrainEngine(m, opt, grad_clip=1.0, synchronizer=GradientSynchronizer(m))
    gen = torch.Generator().manual_seed(4)
    for _ in range(3):
        t = torch.randint(0, 1000, (4, 257), generator=gen).cuda()
        eng.step([(t[:, :-1], t[:, 1:])], lr=3e-4)
    t = torch.randint(0, 1000, (4, 257), generator=gen).cuda()
    m.forward_loss(t[:, :-1], t[:, 1:])  # refreshes the casts the forward uses
    torch.cuda.synchronize()
    assert torch.equal(m._head_cache.tensor, m.lm_head.weight.detach().to(torch.bfloat16))
    for mod in m.modules():
        cache = getattr(mod, "_cache", None)
        if cache is not None and cache.tensor is not None and cache.tensor.shape == mod.weight.shape:
            assert torch.equal(cache.tensor, mod.weight.detach().to(torch.bfloat16))
