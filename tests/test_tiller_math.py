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
