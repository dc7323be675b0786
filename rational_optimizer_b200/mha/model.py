"""Random-initialised modern MHA decoder (reference experiments/mha_1b_tokens/model.py:9-113).

Architecture and parameter names follow the reference exactly (``embed_tokens``,
``layers.{i}.input_layernorm``, ``attn.{q_proj,k_proj,v_proj,out,q_norm,k_norm}``,
``mlp.{gate,value,down}`` or ``mlp.{in_proj,rlb_activation,out_proj}``,
``norm``, tied ``lm_head``), so checkpoints interchange.  Execution is the
B200 path of this package: fp32 master weights with bf16 tensor-core GEMMs,
the RMSNorm and GRAIN sm_100a kernels (GRAIN algebra in fp32 registers on
bf16 inputs), cuDNN/flash SDPA, and the fused linear cross-entropy for the
tied head.  The reference runs the same graph under bf16 autocast; its
RMSNorm rounds the normalised value to bf16 before the weight multiply, this
one multiplies in fp32 and rounds once.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..models.grain import GRAIN
from ..ops.cross_entropy import linear_cross_entropy
from ..ops.linear import Linear, _WeightCache, cached_cast
from ..ops.norm import rms_norm


class RMSNorm(nn.Module):
    def __init__(self, width, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.eps = eps
        self.out_dtype = None

    def forward(self, x):
        if x.is_cuda:
            return rms_norm(x, self.weight, self.eps, self.out_dtype or x.dtype)
        normalized = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + self.eps)
        return self.weight * normalized.to(x.dtype)


def _bias_free(cfg):
    if cfg["attention_bias"]:
        raise ValueError("this decoder is bias-free")
    return False


def rope_split_half(t, cos, sin):
    """Split-half rotary embedding: (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin)."""
    half = t.shape[-1] // 2
    rotated = torch.cat((-t[..., half:], t[..., :half]), dim=-1)
    return t * cos + rotated * sin


class Attention(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.heads, self.kv_heads, self.head_dim = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        if self.heads != self.kv_heads or self.heads * self.head_dim != c["hidden_size"]:
            raise ValueError("this package requires equal QKV heads and a square attention output")
        _bias_free(c)
        width = self.heads * self.head_dim
        self.q_proj = Linear(c["hidden_size"], width)
        self.k_proj = Linear(c["hidden_size"], width)
        self.v_proj = Linear(c["hidden_size"], width)
        self.out = Linear(width, c["hidden_size"])
        self.q_norm = RMSNorm(self.head_dim, c["rms_norm_eps"])
        self.k_norm = RMSNorm(self.head_dim, c["rms_norm_eps"])
        inv = 1.0 / (c["rope_theta"] ** (torch.arange(0, self.head_dim, 2, dtype=torch.float32) / self.head_dim))
        self.register_buffer("inv_freq", inv, persistent=False)

    def forward(self, x):
        b, s, _ = x.shape
        q = self.q_norm(self.q_proj(x).view(b, s, self.heads, self.head_dim)).transpose(1, 2)
        k = self.k_norm(self.k_proj(x).view(b, s, self.heads, self.head_dim)).transpose(1, 2)
        v = self.v_proj(x).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        phases = torch.outer(torch.arange(s, device=x.device, dtype=torch.float32), self.inv_freq.float())
        phases = torch.cat((phases, phases), -1)[None, None]
        cos, sin = phases.cos().to(q.dtype), phases.sin().to(q.dtype)
        q, k = rope_split_half(q, cos, sin), rope_split_half(k, cos, sin)
        y = F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=True)
        return self.out(y.transpose(1, 2).reshape(b, s, self.heads * self.head_dim))


class SwiGLU(nn.Module):
    """``down(silu(gate(x)) * value(x))``.

    ``tap``: optional instrumentation callable; when set, every forward calls
    ``tap(self, x, gate, value, features, output)`` with the tensors the
    forward actually computed (the SwiGLU-TILLER optimizer records its probe
    rows this way).  It does not change the computation.
    """

    def __init__(self, c):
        super().__init__()
        d, h = c["hidden_size"], c["intermediate_size"]
        self.gate, self.value, self.down = Linear(d, h), Linear(d, h), Linear(h, d)
        self.tap = None

    def forward(self, x):
        g, v = self.gate(x), self.value(x)
        h = F.silu(g) * v
        y = self.down(h)
        if self.tap is not None:
            self.tap(self, x, g, v, h, y)
        return y


class GrainMLP(nn.Module):
    def __init__(self, c, groups):
        super().__init__()
        d, h = c["hidden_size"], 3 * c["intermediate_size"] // 2
        if 2 * h != 3 * c["intermediate_size"] or h % groups:
            raise ValueError("GRAIN width/group mismatch")
        self.hidden_dim, self.groups = h, groups
        self.in_proj = Linear(d, h)
        self.rlb_activation = GRAIN(h, groups, init="silu", fit_range=5.0, eps=c["rms_norm_eps"])
        self.out_proj = Linear(h, d)

    def forward(self, x):
        return self.out_proj(self.rlb_activation(self.in_proj(x)))


class Block(nn.Module):
    def __init__(self, c, grain, groups):
        super().__init__()
        d, eps = c["hidden_size"], c["rms_norm_eps"]
        self.input_layernorm = RMSNorm(d, eps)
        self.post_attention_layernorm = RMSNorm(d, eps)
        self.attn = Attention(c)
        self.mlp = GrainMLP(c, groups) if grain else SwiGLU(c)

    def forward(self, x):
        x = x + self.attn(self.input_layernorm(x))
        return x + self.mlp(self.post_attention_layernorm(x))


class ModernMHADecoder(nn.Module):
    def __init__(self, config, *, grain=False, groups=18):
        super().__init__()
        self.config, self.grain, self.groups = dict(config), grain, groups
        if config.get("rope_scaling") is not None or config.get("use_sliding_window") or not config["tie_word_embeddings"]:
            raise ValueError("unsupported configuration change")
        self.embed_tokens = nn.Embedding(config["vocab_size"], config["hidden_size"])
        self.layers = nn.ModuleList([Block(config, grain, groups) for _ in range(config["num_hidden_layers"])])
        self.norm = RMSNorm(config["hidden_size"], config["rms_norm_eps"])
        self.lm_head = nn.Linear(config["hidden_size"], config["vocab_size"], bias=False)
        self.lm_head.weight = self.embed_tokens.weight
        self._head_cache = _WeightCache()
        with torch.no_grad():
            for name, p in self.named_parameters():
                if "rlb_activation" in name:
                    continue  # keep the canonical rational coefficients
                if p.ndim >= 2:
                    nn.init.normal_(p, mean=0.0, std=config["initializer_range"])
                elif name.endswith("weight"):
                    p.fill_(1.0)
                else:
                    p.zero_()
        for m in self.modules():
            if isinstance(m, RMSNorm):
                m.out_dtype = torch.bfloat16

    def hidden(self, ids):
        x = self.embed_tokens(ids)
        for layer in self.layers:
            x = layer(x)
        self.norm.out_dtype = torch.bfloat16 if x.is_cuda else None
        return self.norm(x)

    def forward(self, ids):
        h = self.hidden(ids)
        if h.is_cuda:
            w = cached_cast(self.lm_head.weight, torch.bfloat16, self._head_cache)
            return (h.to(torch.bfloat16) @ w.t()).float()
        return self.lm_head(h)

    def forward_loss(self, ids, labels):
        """Mean next-token cross-entropy; the logits are never materialised on CUDA."""
        h = self.hidden(ids)
        h2 = h.reshape(-1, h.shape[-1])
        w = cached_cast(self.lm_head.weight, torch.bfloat16, self._head_cache) if h.is_cuda else None
        return linear_cross_entropy(h2, self.lm_head.weight, labels.reshape(-1), w_compute=w)


@torch.no_grad()
def copy_shared(source, target):
    """Copy every attention/norm/embedding tensor of ``source`` into ``target`` and verify it."""
    original = dict(source.named_parameters())
    copied = []
    for name, p in target.named_parameters():
        if ".mlp." in name:
            continue
        if name not in original or p.shape != original[name].shape:
            raise RuntimeError("shared parameter inventory mismatch: " + name)
        p.copy_(original[name])
        if not torch.equal(p, original[name]):
            raise RuntimeError("initial parameter mismatch: " + name)
        copied.append(name)
    if set(copied) != {n for n in original if ".mlp." not in n}:
        raise RuntimeError("incomplete initial shared parameter copy")
    return copied
