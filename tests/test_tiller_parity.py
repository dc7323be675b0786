"""TILLER trajectory parity against the reference implementation (CPU, fp32).

Follows the reference's 17-step equivalence recipe (training/test_train.py:
305-460): a tiny GRAIN model, one micro-batch, refreshes at steps 1, 9, 17.
"""
import copy
import types

import pytest
import torch

from reference_oracle import require_reference
from rational_optimizer_b200.models.transformer import CausalTransformer
from rational_optimizer_b200.optim import composite
from rational_optimizer_b200.optim import tiller as my_tiller

ARGS = dict(layers=2, d_model=64, heads=4, ffn_dim=128, seq_len=16, activation="grain",
            rational_init="silu", rational_group_size=32, rational_max_groups=32,
            rational_basis_eps=1e-6, init_std=0.02, optimizer="tiller_v1", lr=3e-4,
            weight_decay=0.1, muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95,
            eps=1e-8, muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
VOCAB = 97


def _step(model, opt, router, x, y):
    opt.zero_grad(set_to_none=True)
    logits = model(x)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, VOCAB).float(), y.reshape(-1))
    loss.backward()
    norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    router.record_realized_clipping(float(norm), 1.0)
    opt.step()
    return float(loss.detach())


@pytest.mark.parametrize("steps", [17])
def test_tiller_matches_reference(steps):
    ref = require_reference()
    args = types.SimpleNamespace(**ARGS)
    torch.manual_seed(0)
    ref_model = ref["train"].CausalTransformer(args, VOCAB)
    ref["entry"].set_experiment_layout(microbatches=1, decay_tied_embedding=False)
    ref_opt = ref["entry"].configure_candidate_optimizer(ref_model, args)
    mine = CausalTransformer(args, VOCAB)
    mine.load_state_dict(ref_model.state_dict())
    my_tiller.configure_microbatch_count(1)
    my_opt = composite.build_tiller(mine, args, microbatches=1)
    gen = torch.Generator().manual_seed(1)
    for step in range(steps):
        tokens = torch.randint(0, VOCAB, (2, 17), generator=gen)
        x, y = tokens[:, :-1], tokens[:, 1:]
        l_ref = _step(ref_model, ref_opt, ref_opt.optimizers[0], x, y)
        l_me = _step(mine, my_opt, my_opt.router, x, y)
        assert abs(l_ref - l_me) < 1e-5 * max(1.0, abs(l_ref)), (step, l_ref, l_me)
        for (n1, p1), (n2, p2) in zip(ref_model.named_parameters(), mine.named_parameters()):
            assert n1 == n2
            torch.testing.assert_close(p2, p1, rtol=2e-4, atol=2e-6, msg=f"step {step} {n1}")
    ra = ref_opt.optimizers[0].state[ref_opt.optimizers[0].pairs[0]["in_weight"]]
    ma = my_opt.router.anchor
    assert set(ra.keys()) == set(ma.keys())
    assert ma["factorized_rfd_step"] == steps
    assert ma["cadence8_transition"] == steps
    # RFD factors agree up to row rotation: compare S^T S.
    s1 = ra["factorized_rfd_persistent_scores"].double()
    s2 = ma["factorized_rfd_persistent_scores"].double()
    torch.testing.assert_close(s2.T @ s2, s1.T @ s1, rtol=1e-3, atol=1e-9)
    ref_sd = ref_opt.state_dict()
    my_sd = my_opt.state_dict()
    assert my_sd["schema"] == ref_sd["schema"] and tuple(my_sd["roles"]) == tuple(ref_sd["roles"])
    for c_ref, c_me in zip(ref_sd["children"], my_sd["children"]):
        g_ref = {k: v for k, v in c_ref["param_groups"][0].items() if k != "params"}
        g_me = {k: v for k, v in c_me["param_groups"][0].items() if k != "params"}
        if "foreach" in g_ref:  # AdamW implementation flags differ
            for k in ("foreach", "fused", "capturable", "differentiable", "maximize", "amsgrad",
                      "decoupled_weight_decay"):
                g_ref.pop(k, None)
                g_me.pop(k, None)
        assert g_ref == g_me


def test_tiller_state_dict_loads_into_reference_and_back():
    ref = require_reference()
    args = types.SimpleNamespace(**ARGS)
    torch.manual_seed(0)
    mine = CausalTransformer(args, VOCAB)
    my_tiller.configure_microbatch_count(1)
    my_opt = composite.build_tiller(mine, args, microbatches=1)
    gen = torch.Generator().manual_seed(3)
    for _ in range(3):
        tokens = torch.randint(0, VOCAB, (2, 17), generator=gen)
        _step(mine, my_opt, my_opt.router, tokens[:, :-1], tokens[:, 1:])
    ref_model = ref["train"].CausalTransformer(args, VOCAB)
    ref_model.load_state_dict(mine.state_dict())
    ref["entry"].set_experiment_layout(microbatches=1, decay_tied_embedding=False)
    ref_opt = ref["entry"].configure_candidate_optimizer(ref_model, args)
    ref_opt.load_state_dict(copy.deepcopy(my_opt.state_dict()))
    # and back into a fresh one of ours
    mine2 = CausalTransformer(args, VOCAB)
    mine2.load_state_dict(ref_model.state_dict())
    opt2 = composite.build_tiller(mine2, args, microbatches=1)
    opt2.load_state_dict(copy.deepcopy(ref_opt.state_dict()))
    for _ in range(2):
        tokens = torch.randint(0, VOCAB, (2, 17), generator=gen)
        x, y = tokens[:, :-1], tokens[:, 1:]
        _step(ref_model, ref_opt, ref_opt.optimizers[0], x, y)
        _step(mine2, opt2, opt2.router, x, y)
    for (n1, p1), (_, p2) in zip(ref_model.named_parameters(), mine2.named_parameters()):
        torch.testing.assert_close(p2, p1, rtol=2e-4, atol=2e-6, msg=n1)
