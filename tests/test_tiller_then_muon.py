"""Two-stage TILLER -> Muon switch against the reference (CPU, fp32).

The reference fixes the switch at update 1000 through a module constant
(optimizer_design/tiller_then_muon.py:18, read at step time); the test moves
it to update 3 after construction so the hand-off and three Muon steps run.
"""
import copy
import types

import torch

from reference_oracle import require_reference
from rational_optimizer_b200.models.transformer import CausalTransformer
from rational_optimizer_b200.optim import composite
from rational_optimizer_b200.optim.tiller_then_muon import (TillerThenMuonOptimizer,
                                                             configure_microbatch_count)

ARGS = dict(layers=2, d_model=64, heads=4, ffn_dim=128, seq_len=16, activation="grain",
            rational_init="silu", rational_group_size=32, rational_max_groups=32,
            rational_basis_eps=1e-6, init_std=0.02, optimizer="tiller_then_muon_v1", lr=3e-4,
            weight_decay=0.1, muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95,
            eps=1e-8, muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
VOCAB = 97
SWITCH = 3


def _step(model, opt, x, y):
    opt.zero_grad(set_to_none=True)
    logits = model(x)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, VOCAB).float(), y.reshape(-1))
    loss.backward()
    norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    opt.record_realized_clipping(float(norm), 1.0)
    opt.set_telemetry_capture(True)
    opt.step()
    return float(loss.detach())


def _ours(args, state):
    model = CausalTransformer(args, VOCAB)
    model.load_state_dict(state)
    configure_microbatch_count(1)
    blocks = composite.collect_blocks(model, args)
    _, decay, no_decay = composite.partition_parameters(model, blocks)
    groups = [{"params": decay, "weight_decay": args.weight_decay},
              {"params": no_decay, "weight_decay": 0.0}]
    opt = TillerThenMuonOptimizer(blocks, adam_groups=groups, lr=args.lr,
                                  weight_decay=args.weight_decay, momentum=args.muon_momentum,
                                  ns_steps=args.muon_ns_steps, beta1=args.beta1, beta2=args.beta2,
                                  eps=args.eps, adjust_lr_fn=args.muon_adjust_lr_fn,
                                  switch_after_step=SWITCH)
    return model, opt


def test_switch_matches_reference(monkeypatch):
    ref = require_reference()
    import importlib
    ref_mod = importlib.import_module("optimizer_design.tiller_then_muon")
    args = types.SimpleNamespace(**ARGS)
    torch.manual_seed(0)
    ref_model = ref["train"].CausalTransformer(args, VOCAB)
    ref_opt = ref["train"].configure_optimizer(ref_model, args)
    monkeypatch.setattr(ref_mod, "SWITCH_AFTER_STEP", SWITCH)
    mine, my_opt = _ours(args, ref_model.state_dict())
    gen = torch.Generator().manual_seed(5)
    for step in range(2 * SWITCH):
        tokens = torch.randint(0, VOCAB, (2, 17), generator=gen)
        x, y = tokens[:, :-1], tokens[:, 1:]
        l_ref = _step(ref_model, ref_opt, x, y)
        l_me = _step(mine, my_opt, x, y)
        assert abs(l_ref - l_me) < 1e-5 * max(1.0, abs(l_ref)), (step, l_ref, l_me)
        assert my_opt.stage == ref_opt.stage
        t_ref, t_me = ref_opt.telemetry(), my_opt.telemetry()
        for key in ("tiller_then_muon_completed_steps", "tiller_then_muon_stage_before_step",
                    "tiller_then_muon_stage_after_step", "tiller_then_muon_switched_to_muon"):
            assert t_me[key] == t_ref[key], (step, key)
        for (n, p1), (_, p2) in zip(ref_model.named_parameters(), mine.named_parameters()):
            torch.testing.assert_close(p2, p1, rtol=2e-4, atol=2e-6, msg=f"step {step} {n}")
    assert my_opt.stage == "muon" and my_opt.completed_steps == 2 * SWITCH
    # Muon's momentum continues from TILLER's; AdamW's state was never reset
    for group_ref, group_me in zip(ref_opt.ordinary_muon.param_groups, my_opt.ordinary_muon.param_groups):
        for p1, p2 in zip(group_ref["params"], group_me["params"]):
            torch.testing.assert_close(my_opt.ordinary_muon.state[p2]["momentum_buffer"],
                                       ref_opt.ordinary_muon.state[p1]["momentum_buffer"],
                                       rtol=2e-4, atol=2e-6)
    assert my_opt.adamw.state[next(iter(my_opt.adamw.state))]["step"] == 2 * SWITCH
    sd_ref, sd_me = ref_opt.state_dict(), my_opt.state_dict()
    for key in ("schema", "optimizer_id", "completed_steps", "stage", "state_transition"):
        assert sd_me[key] == sd_ref[key], key
    assert set(sd_me["children"]) == set(sd_ref["children"])


def test_checkpoint_before_and_after_switch_resumes(monkeypatch):
    args = types.SimpleNamespace(**ARGS)
    torch.manual_seed(0)
    base = CausalTransformer(args, VOCAB).state_dict()
    gen = torch.Generator().manual_seed(7)
    batches = [torch.randint(0, VOCAB, (2, 17), generator=gen) for _ in range(2 * SWITCH + 2)]
    straight, opt = _ours(args, base)
    for t in batches:
        _step(straight, opt, t[:, :-1], t[:, 1:])
    for cut in (SWITCH - 1, SWITCH + 1):
        model, opt = _ours(args, base)
        for t in batches[:cut]:
            _step(model, opt, t[:, :-1], t[:, 1:])
        saved_model, saved_opt = copy.deepcopy(model.state_dict()), copy.deepcopy(opt.state_dict())
        model2, opt2 = _ours(args, saved_model)
        opt2.load_state_dict(saved_opt)
        assert opt2.stage == ("muon" if cut >= SWITCH else "tiller")
        for t in batches[cut:]:
            _step(model2, opt2, t[:, :-1], t[:, 1:])
        for (n, p1), (_, p2) in zip(straight.named_parameters(), model2.named_parameters()):
            assert torch.equal(p1, p2), (cut, n)


def test_rejects_foreign_checkpoint():
    args = types.SimpleNamespace(**ARGS)
    torch.manual_seed(0)
    _, opt = _ours(args, CausalTransformer(args, VOCAB).state_dict())
    sd = opt.state_dict()
    sd["schema"] = "something_else"
    try:
        opt.load_state_dict(sd)
    except RuntimeError as exc:
        assert "schema" in str(exc)
    else:
        raise AssertionError("foreign schema accepted")
