"""Fixed-SwiGLU TILLER extension (CPU): math identities, training steps, checkpoint round trip."""
import copy

import torch
import torch.nn.functional as F

from rational_optimizer_b200.mha.model import ModernMHADecoder
from rational_optimizer_b200.optim import tiller_swiglu as TS


def _model(seed=0):
    cfg = dict(attention_bias=False, head_dim=4, hidden_size=64, initializer_range=0.02, intermediate_size=128,
               num_attention_heads=16, num_hidden_layers=2, num_key_value_heads=16, rms_norm_eps=1e-6,
               rope_scaling=None, rope_theta=1e6, tie_word_embeddings=True, use_sliding_window=False,
               vocab_size=128)
    torch.manual_seed(seed)
    return ModernMHADecoder(cfg)


def test_factors_are_the_swiglu_derivatives():
    g = torch.randn(7, 5, dtype=torch.float64, requires_grad=True)
    v = torch.randn(7, 5, dtype=torch.float64, requires_grad=True)
    h, dg, dv = TS.swiglu_factors(g, v)
    torch.testing.assert_close(h, F.silu(g) * v)
    gg, gv = torch.autograd.grad(h.sum(), (g, v))
    torch.testing.assert_close(dg, gg)
    torch.testing.assert_close(dv, gv)


def _per_token_loss(model, x, y):
    logits = model(x)
    return F.cross_entropy(logits.flatten(0, 1), y.flatten(), reduction="none").view(y.shape)


def _run(model, opt, batches):
    out = []
    for x, y in batches:
        opt.zero_grad()
        opt.begin_step([torch.ones_like(y, dtype=torch.bool)])
        opt.backward(_per_token_loss(model, x, y))
        out.append(opt.step())
    return out


def test_training_steps_and_checkpoint_round_trip():
    model = _model()
    opt = TS.SwiGLUTILLER(model, group_width=32)
    gen = torch.Generator().manual_seed(1)
    batches = [(torch.randint(0, 128, (4, 16), generator=gen), torch.randint(0, 128, (4, 16), generator=gen))
               for _ in range(11)]
    metrics = _run(model, opt, batches[:9])
    assert [m["functional_refresh"] for m in metrics] == [True] + [False] * 7 + [True]
    assert all(m["budget_residual"] < 1e-6 or not m["proposal_accepted"] for m in metrics)
    assert opt.completed_steps == 9
    twin_model = _model(seed=5)  # fresh modules (a deep copy would carry the first router's hooks)
    twin_model.load_state_dict(model.state_dict())
    twin = TS.SwiGLUTILLER(twin_model, group_width=32)
    twin.load_state_dict(copy.deepcopy(opt.state_dict()))
    a = _run(model, opt, batches[9:])
    b = _run(twin_model, twin, batches[9:])
    for p, q in zip(model.parameters(), twin_model.parameters()):
        assert torch.equal(p, q)
    assert [m["preclip_norm"] for m in a] == [m["preclip_norm"] for m in b]


def test_trajectory_matches_reference_extension():
    """Ten updates (refreshes at 1 and 9) of ours against the reference extension
    (experiments/swiglu_tiller/tiller_swiglu.py) on the same weights and batches."""
    import importlib

    from reference_oracle import require_reference
    require_reference()
    ref_ts = importlib.import_module("experiments.swiglu_tiller.tiller_swiglu")
    ref_model_mod = importlib.import_module("experiments.swiglu_tiller.model")
    mine = _model()
    theirs = ref_model_mod.ModernMHADecoder(mine.config)
    theirs.load_state_dict(mine.state_dict())
    my_opt = TS.SwiGLUTILLER(mine, group_width=32)
    ref_opt = ref_ts.SwiGLUTILLER(theirs, group_width=32)
    gen = torch.Generator().manual_seed(4)
    for step in range(10):
        x = torch.randint(0, 128, (4, 16), generator=gen)
        y = torch.randint(0, 128, (4, 16), generator=gen)
        mask = torch.rand(4, 16, generator=gen) > 0.2
        got = []
        for model, opt in ((mine, my_opt), (theirs, ref_opt)):
            opt.zero_grad()
            opt.begin_step([mask])
            opt.backward(_per_token_loss(model, x, y))
            got.append(opt.step())
        for key in ("functional_refresh", "ledger_step", "proposal_accepted", "total_loss_tokens"):
            assert got[0][key] == got[1][key], (step, key)
        assert abs(got[0]["preclip_norm"] - got[1]["preclip_norm"]) <= 1e-5 * got[1]["preclip_norm"]
        for (n, p), (_, q) in zip(mine.named_parameters(), theirs.named_parameters()):
            torch.testing.assert_close(p, q, rtol=2e-4, atol=2e-6, msg=f"step {step} {n}")
    # checkpoints interchange
    ref_opt.close()
    twin = ref_model_mod.ModernMHADecoder(mine.config)
    twin.load_state_dict(mine.state_dict())
    ref_twin = ref_ts.SwiGLUTILLER(twin, group_width=32)
    ref_twin.load_state_dict(copy.deepcopy(my_opt.state_dict()))
    assert ref_twin.completed_steps == my_opt.completed_steps == 10
