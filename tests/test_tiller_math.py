"""TILLER math helpers on CPU."""




def test_stacked_group_scores_match_the_per_layer_scores():
    import torch
    from rational_optimizer_b200.optim import tiller_math as tm
    torch.manual_seed(0)
    L, P, d, G, w = 3, 5, 16, 4, 8
    H = G * w
    inputs, cot = torch.randn(L, P, d), torch.randn(L, P, d)
    features, adjoint = torch.randn(L, P, H), torch.randn(L, P, G, w)
    inc, out_t = torch.randn(L, H, d), torch.randn(L, H, d)
    stacked = tm.group_scores_stacked(inputs, features, cot, inc, out_t, adjoint, groups=G, width=w)
    for l in range(L):
        one = tm.group_scores(inputs[l], features[l], cot[l], inc[l], out_t[l], adjoint[l], groups=G, width=w)
        torch.testing.assert_close(stacked[l], one, rtol=1e-5, atol=1e-5)


def test_stacked_probe_packets_equal_the_per_layer_packets():
    import torch
    from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
    from rational_optimizer_b200.optim import composite
    args = model_args(layers=3, d_model=64, heads=4, ffn_dim=128, seq_len=32, activation="grain",
                      rational_group_size=32, optimizer="tiller_v1", lr=3e-4, weight_decay=0.1,
                      muon_momentum=0.95, muon_ns_steps=5, beta1=0.9, beta2=0.95, eps=1e-8,
                      muon_adjust_lr_fn="match_rms_adamw", grad_accum=1)
    torch.manual_seed(0)
    model = CausalTransformer(args, 128)
    router = composite.configure_optimizer(model, args).optimizers[0]
    x = torch.randint(0, 128, (4, 33))
    with router.probes_forced():
        model.forward_loss(x[:, :-1], x[:, 1:]).backward()
    router.record_realized_clipping(0.5, 1.0)
    records = router.take_probe_records()
    router.restore_probe_records(records)
    per_layer = router._consume_probes()
    router.restore_probe_records(records)
    stacked = router._consume_probes_stacked()
    assert len(per_layer) == len(stacked) == 3
    for a, b in zip(per_layer, stacked):
        for u, v in zip(a, b):
            assert torch.equal(u, v)
