"""Own tcgen05 flash attention against the fp32 PyTorch oracle (small and odd shapes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200.ops.attention import attention_reference, flash_attention_forward


def _planes(B, S, H, hd, seed, ld=None):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    ld = ld or H * hd
    q, k, v = (torch.randn(B, S, ld, device="cuda", generator=gen).to(torch.bfloat16) for _ in range(3))
    return q, k, v


@pytest.mark.parametrize("B,S,H,hd,causal", [(2, 256, 4, 64, True), (1, 1024, 2, 64, True),
                                             (3, 200, 3, 64, True), (2, 130, 2, 128, True),
                                             (2, 384, 2, 64, False), (1, 2048, 1, 128, True)])
def test_forward_matches_fp32_oracle(B, S, H, hd, causal):
    q, k, v = _planes(B, S, H, hd, S + H)
    out = flash_attention_forward(q, k, v, H, hd, causal=causal)
    assert out is not None
    o, lse2 = out
    ref_o, ref_lse2 = attention_reference(q, k, v, H, hd, causal=causal)
    torch.cuda.synchronize()
    torch.testing.assert_close(o.float(), ref_o, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse2, ref_lse2, rtol=1e-3, atol=1e-3)


def test_forward_reads_heads_inside_wider_rows():
    # planes whose row holds more columns than H * hd (e.g. a slice of a fused buffer)
    q, k, v = _planes(2, 256, 2, 64, 7, ld=256)
    o, lse2 = flash_attention_forward(q, k, v, 2, 64)
    ref_o, _ = attention_reference(q, k, v, 2, 64)
    torch.testing.assert_close(o.float(), ref_o, rtol=2e-2, atol=2e-2)


def _grad_reference(q, k, v, do, H, hd, causal):
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    o, _ = attention_reference(qf, kf, vf, H, hd, causal=causal)
    o.backward(do.float())
    return qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("B,S,H,hd,causal", [(2, 256, 2, 64, True), (1, 384, 3, 64, True),
                                             (2, 200, 2, 64, True), (1, 256, 2, 128, True),
                                             (1, 256, 2, 64, False)])
def test_backward_matches_fp32_oracle(B, S, H, hd, causal):
    from rational_optimizer_b200 import _ext
    q, k, v = _planes(B, S, H, hd, 11 + S)
    gen = torch.Generator(device="cuda").manual_seed(5)
    do = torch.randn(B, S, H * hd, device="cuda", generator=gen).to(torch.bfloat16)
    o, lse2 = flash_attention_forward(q, k, v, H, hd, causal=causal)
    dq, dk, dv = _ext.ext().attention_backward(q, k, v, o, do, lse2, H, hd, hd ** -0.5, causal)
    rq, rk, rv = _grad_reference(q, k, v, do, H, hd, causal)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        err = (got.float() - ref).abs().max().item()
        assert err <= 3e-2 * max(1.0, ref.abs().max().item()), err


def test_backward_is_deterministic():
    from rational_optimizer_b200 import _ext
    q, k, v = _planes(2, 512, 4, 64, 3)
    do = torch.randn_like(q, dtype=torch.float32).to(torch.bfloat16)
    o, lse2 = flash_attention_forward(q, k, v, 4, 64)
    first = _ext.ext().attention_backward(q, k, v, o, do, lse2, 4, 64, 0.125, True)
    second = _ext.ext().attention_backward(q, k, v, o, do, lse2, 4, 64, 0.125, True)
    for a, b in zip(first, second):
        assert torch.equal(a, b)


def test_model_attention_uses_own_kernel_and_matches_sdpa(monkeypatch):
    """The model path (fused q/k/v + RoPE projection -> own attention) against
    the same path on PyTorch's SDPA, forward and input/weight gradients."""
    from rational_optimizer_b200.ops import attention as A
    torch.manual_seed(0)
    B, S, H, hd = 2, 256, 8, 64
    d = H * hd
    x = (torch.randn(B, S, d, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(3 * d, d, device="cuda") * d ** -0.5)
    cos, sin = A.precompute_rope(S, hd)
    cos, sin = cos.cuda(), sin.cuda()
    results = []
    for own in ("1", "0"):
        monkeypatch.setenv("RO_OWN_ATTENTION", own)
        q_probe = torch.empty(B, S, H, hd, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
        assert A.own_attention_supported(q_probe) == (own == "1")
        xi = x.clone().requires_grad_()
        wi = w.clone().requires_grad_()
        y = A.fused_qkv_attention(xi, wi, wi.to(torch.bfloat16), B, S, H, hd, cos, sin)
        y.float().square().mean().backward()
        results.append((y.detach().float(), xi.grad.float(), wi.grad.float()))
    for a, b in zip(*results):
        torch.testing.assert_close(a, b, rtol=5e-2, atol=5e-3)
