"""Causal attention at seq 2048 with head_dim 64 / 96 / 128 through the model (CPU).

The model's attention path (RoPE + causal attention) is checked against a
plain fp32 restatement at the sequence length of the MHA study (2048) and
the head widths it supports; the gradient must reach every parameter.
"""
import math

import pytest
import torch

from rational_optimizer_b200.models.transformer import CausalTransformer, model_args
from rational_optimizer_b200.ops.attention import apply_rope, causal_self_attention, precompute_rope


def _oracle(qkv, B, S, H, hd, cos, sin):
    d = H * hd
    q, k, v = qkv.reshape(B, S, 3 * d).chunk(3, dim=-1)
    q, k, v = (t.reshape(B, S, H, hd).transpose(1, 2) for t in (q, k, v))
    q = apply_rope(q, cos[:, :, :S], sin[:, :, :S])
    k = apply_rope(k, cos[:, :, :S], sin[:, :, :S])
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(hd)
    mask = torch.ones(S, S, dtype=torch.bool).tril()
    scores = scores.masked_fill(~mask, float("-inf"))
    return (scores.softmax(-1) @ v).transpose(1, 2).reshape(B, S, d)


@pytest.mark.parametrize("hd", [64, 96, 128])
def test_causal_attention_seq2048_matches_oracle(hd):
    torch.manual_seed(hd)
    B, S, H = 1, 2048, 2
    cos, sin = precompute_rope(S, hd)
    qkv = torch.randn(B * S, 3 * H * hd)
    y = causal_self_attention(qkv, B, S, H, hd, cos, sin)
    ref = _oracle(qkv, B, S, H, hd, cos, sin)
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("hd", [96, 128])
def test_model_trains_at_seq2048(hd):
    torch.manual_seed(0)
    heads = 2
    args = model_args(layers=1, d_model=heads * hd, heads=heads, ffn_dim=256, seq_len=2048, activation="grain",
                      rational_group_size=64)
    model = CausalTransformer(args, 128)
    x = torch.randint(0, 128, (1, 2049))
    loss = model.forward_loss(x[:, :-1], x[:, 1:])
    loss.backward()
    assert math.isfinite(loss.item())
    missing = [n for n, p in model.named_parameters() if p.requires_grad and p.grad is None]
    assert not missing, missing
