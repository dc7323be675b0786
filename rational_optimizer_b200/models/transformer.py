"""Decoder-only Transformer with GRAIN or SwiGLU feed-forward blocks.

Module tree and parameter names are those of training/train.py:24-272 so
checkpoints interchange with the reference (``token_embedding.weight``,
``layers.{i}.{attn_norm,ffn_norm}.weight``, ``layers.{i}.attn.{qkv,out}.weight``,
``layers.{i}.mlp.{in_proj,out_proj}.weight``, ``layers.{i}.mlp.rlb_activation.*``,
``norm.weight``, tied ``lm_head.weight``; RoPE tables are non-persistent).

Execution differs: parameters are fp32 masters, GEMMs run in bf16 on CUDA
with fp32 accumulation, the residual stream stays fp32, RMSNorm/RoPE/GRAIN
are single sm_100a kernels, and :meth:`CausalTransformer.forward_loss` fuses
the tied ``lm_head`` with the cross-entropy so full logits are never stored.
"""
from __future__ import annotations

import math
from types import SimpleNamespace

import torch
import torch.nn as nn

from ..ops.attention import causal_self_attention, fused_qkv_attention, precompute_rope, qkv_rope_supported
from ..ops.cross_entropy import linear_cross_entropy
from ..ops.grain import grain_mlp, in_proj_grain_supported
from ..ops.linear import Linear, cached_cast, cached_cast_t, _WeightCache
from ..parallel import param_ready as _ready
from ..ops.norm import add_rms_norm, fused_add_norm_supported, rms_norm
from .grain import GRAIN

GRAIN_ACTIVATION = "grain"
LEGACY_GRAIN_ACTIVATION = "rlb_fused_global_rational"
ACTIVATIONS = ("silu", GRAIN_ACTIVATION)
ACCEPTED_ACTIVATIONS = (*ACTIVATIONS, LEGACY_GRAIN_ACTIVATION)
GRAIN_ACTIVATION_IDS = {GRAIN_ACTIVATION, LEGACY_GRAIN_ACTIVATION}


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps
        self.out_dtype = None  # None: same as input; bf16 feeds the next GEMM on CUDA

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps, self.out_dtype if x.is_cuda else None)


class CausalSelfAttention(nn.Module):
    def __init__(self, dim, heads, seq_len):
        super().__init__()
        if dim % heads != 0:
            raise ValueError("dim must be divisible by heads")
        self.heads = heads
        self.head_dim = dim // heads
        self.qkv = Linear(dim, 3 * dim, bias=False)
        self.out = Linear(dim, dim, bias=False)
        cos, sin = precompute_rope(seq_len, self.head_dim)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def forward(self, x):
        batch, seq_len, dim = x.shape
        if (self.qkv.compute_dtype == torch.bfloat16 and self.qkv.weight.dtype == torch.float32
                and seq_len <= self.rope_cos.shape[-2] and qkv_rope_supported(x, dim, self.head_dim)):
            # projection + RoPE in one GEMM (rotation in the epilogue)
            if _ready.pending():
                _ready.wait(self.qkv.weight)
            w = cached_cast(self.qkv.weight, torch.bfloat16, self.qkv._cache)
            y = fused_qkv_attention(x, self.qkv.weight, w, batch, seq_len, self.heads, self.head_dim,
                                    self.rope_cos[:, :, :seq_len], self.rope_sin[:, :, :seq_len])
            return self.out(y)
        qkv = self.qkv(x)
        if seq_len > self.rope_cos.shape[-2]:
            raise ValueError("sequence longer than the precomputed RoPE table")
        y = causal_self_attention(qkv, batch, seq_len, self.heads, self.head_dim,
                                  self.rope_cos[:, :, :seq_len], self.rope_sin[:, :, :seq_len])
        return self.out(y)


def resolve_group_count(hidden_dim, group_size, max_groups):
    """Largest divisor of ``hidden_dim`` not above min(max_groups, ceil(H/group_size))."""
    target = min(int(max_groups), max(1, math.ceil(int(hidden_dim) / int(group_size))))
    target = min(target, int(hidden_dim))
    for groups in range(target, 0, -1):
        if hidden_dim % groups == 0:
            return groups
    return 1


def grain_settings(ffn_dim, group_size, max_groups):
    """Parameter-matched GRAIN width ``3*ffn/2`` and its group count."""
    hidden_dim = (3 * int(ffn_dim)) // 2
    return {
        "hidden_dim": hidden_dim,
        "groups": resolve_group_count(hidden_dim, group_size, max_groups),
        "base_init": "silu",
        "centers": (),
        "coeff_limit": 0.0,
        "beta": 0.0,
        "input_affine": False,
        "center_odd": False,
        "train_centers": False,
        "atom_scale_init": None,
        "atom_scale_limit": 1.0,
        "fused": True,
    }


class SwiGLU(nn.Module):
    def __init__(self, dim, ffn_dim):
        super().__init__()
        self.activation_name = "silu"
        self.gate = Linear(dim, ffn_dim, bias=False)
        self.value = Linear(dim, ffn_dim, bias=False)
        self.down = Linear(ffn_dim, dim, bias=False)

    def forward(self, x):
        g = self.gate(x)
        v = self.value(x)
        return self.down(torch.nn.functional.silu(g) * v)


class GRAINMLP(nn.Module):
    """``in_proj -> GRAIN -> out_proj`` (parameter-matched SwiGLU replacement)."""

    def __init__(self, dim, ffn_dim, group_size, max_groups, eps=1e-6, hidden_dim=None,
                 groups=None):
        super().__init__()
        settings = grain_settings(ffn_dim, group_size, max_groups)
        self.activation_name = GRAIN_ACTIVATION
        self.hidden_dim = int(hidden_dim) if hidden_dim is not None else settings["hidden_dim"]
        self.groups = int(groups) if groups is not None else (
            settings["groups"] if hidden_dim is None
            else resolve_group_count(self.hidden_dim, group_size, max_groups))
        self.in_proj = Linear(dim, self.hidden_dim, bias=False)
        self.rlb_activation = GRAIN(self.hidden_dim, self.groups, init=settings["base_init"],
                                    fit_range=5.0, eps=eps)
        self.out_proj = Linear(self.hidden_dim, dim, bias=False)
        self._out_t_cache = _WeightCache()  # bf16 out_proj.weight^T for the fused backward

    def forward(self, x):
        act = self.rlb_activation
        if (self.in_proj.compute_dtype == torch.bfloat16 and self.in_proj.weight.dtype == torch.float32
                and self.out_proj.weight.dtype == torch.float32
                and in_proj_grain_supported(x, act.hidden_dim, act.groups)):
            # GRAIN evaluated in the GEMM epilogues (forward and backward)
            if _ready.pending():
                _ready.wait(self.in_proj.weight)
                _ready.wait(self.out_proj.weight)
            w_in = cached_cast(self.in_proj.weight, torch.bfloat16, self.in_proj._cache)
            w_out = cached_cast(self.out_proj.weight, torch.bfloat16, self.out_proj._cache)
            w_out_t = cached_cast_t(self.out_proj.weight, torch.bfloat16, self._out_t_cache)
            o, h, y = grain_mlp(x, self.in_proj.weight, w_in, act.numerator, act.denominator,
                                self.out_proj.weight, w_out, w_out_t, act.eps, act.groups)
            act(h, precomputed=y)  # the activation's statistics and forward hooks see (h, y)
            return o
        return self.out_proj(act(self.in_proj(x)))


def apply_rlb_positive_gauge(model: nn.Module, log_scale: float, seed: int) -> int:
    """Per-group positive in/out rescaling used by the fairness audit (train.py:165-193)."""
    if log_scale <= 0.0:
        return 0
    generator = torch.Generator(device="cpu")
    generator.manual_seed(int(seed))
    count = 0
    with torch.no_grad():
        for module in model.modules():
            if not isinstance(module, GRAINMLP):
                continue
            groups = int(module.groups)
            width = int(module.hidden_dim // module.groups)
            logs = torch.empty(groups, dtype=torch.float32).uniform_(
                -float(log_scale), float(log_scale), generator=generator)
            scales = torch.exp(logs).to(device=module.in_proj.weight.device,
                                        dtype=module.in_proj.weight.dtype)
            module.in_proj.weight.view(groups, width, -1).mul_(scales.view(groups, 1, 1))
            module.out_proj.weight.view(module.out_proj.weight.shape[0], groups, width).mul_(
                scales.reciprocal().view(1, groups, 1))
            count += groups
    return count


class TransformerBlock(nn.Module):
    def __init__(self, dim, heads, ffn_dim, seq_len, activation, rational_init,
                 rational_group_size, rational_max_groups, rational_eps, grain_hidden=None,
                 grain_groups=None):
        super().__init__()
        self.attn_norm = RMSNorm(dim)
        self.ffn_norm = RMSNorm(dim)
        self.attn = CausalSelfAttention(dim, heads, seq_len)
        if activation == "silu":
            self.mlp = SwiGLU(dim, ffn_dim)
        elif activation in GRAIN_ACTIVATION_IDS:
            if rational_init != "silu":
                raise ValueError("GRAIN uses the published SiLU initialization")
            self.mlp = GRAINMLP(dim, ffn_dim, rational_group_size, rational_max_groups,
                                rational_eps, hidden_dim=grain_hidden, groups=grain_groups)
        else:
            raise ValueError(f"unknown activation {activation!r}")

    def forward(self, x):
        x = x + self.attn(self.attn_norm(x))
        x = x + self.mlp(self.ffn_norm(x))
        return x


def init_weights(module, init_std):
    if isinstance(module, nn.Linear):
        if getattr(module, "zero_init", False):
            nn.init.zeros_(module.weight)
        else:
            nn.init.normal_(module.weight, mean=0.0, std=init_std)
    elif isinstance(module, nn.Embedding):
        nn.init.normal_(module.weight, mean=0.0, std=init_std)


class CausalTransformer(nn.Module):
    """Reference-compatible LM (training/train.py:234-263)."""

    def __init__(self, args, vocab_size):
        super().__init__()
        self.args = args
        self.token_embedding = nn.Embedding(vocab_size, args.d_model)
        self.layers = nn.ModuleList([
            TransformerBlock(args.d_model, args.heads, args.ffn_dim, args.seq_len, args.activation,
                             args.rational_init, args.rational_group_size,
                             args.rational_max_groups, args.rational_basis_eps,
                             getattr(args, "grain_hidden_dim", None),
                             getattr(args, "grain_groups", None))
            for _ in range(args.layers)
        ])
        self.norm = RMSNorm(args.d_model)
        self.lm_head = nn.Linear(args.d_model, vocab_size, bias=False)
        self.lm_head.weight = self.token_embedding.weight
        self.apply(lambda module: init_weights(module, args.init_std))
        self._head_cache = _WeightCache()
        self.fuse_residual_norm = True
        self.compute_dtype = torch.float32
        self.set_compute_dtype(torch.bfloat16)

    def set_compute_dtype(self, dtype):
        """bf16 (default) or fp32 GEMM/activation dtype for CUDA execution."""
        self.compute_dtype = dtype
        for module in self.modules():
            if isinstance(module, Linear):
                module.compute_dtype = dtype
        for name, module in self.named_modules():
            if isinstance(module, RMSNorm):
                module.out_dtype = None if name == "norm" else dtype
        self.norm.out_dtype = dtype
        return self

    def hidden_states(self, input_ids):
        x = self.token_embedding(input_ids)
        if (self.fuse_residual_norm and self.compute_dtype == torch.bfloat16
                and fused_add_norm_supported(x)):
            return self._hidden_states_fused(x)
        for layer in self.layers:
            x = layer(x)
        return self.norm(x)

    def _hidden_states_fused(self, x):
        """Same computation with every residual add fused into the following RMSNorm.

        Each block's two branch outputs are carried as a pending bf16 delta and
        added inside the next norm kernel (whose backward also folds the
        residual-gradient accumulation), so no standalone add runs.
        """
        pending = None
        for layer in self.layers:
            x, h = add_rms_norm(x, pending, layer.attn_norm.weight, layer.attn_norm.eps)
            a = layer.attn(h)
            x, h = add_rms_norm(x, a, layer.ffn_norm.weight, layer.ffn_norm.eps)
            pending = layer.mlp(h)
        _, h = add_rms_norm(x, pending, self.norm.weight, self.norm.eps)
        return h

    def forward(self, input_ids):
        h = self.hidden_states(input_ids)
        if h.is_cuda and self.compute_dtype != torch.float32:
            w = cached_cast(self.lm_head.weight, self.compute_dtype, self._head_cache)
            return (h.to(w.dtype) @ w.t()).float()
        return self.lm_head(h)

    def forward_loss(self, input_ids, targets):
        """Mean next-token cross-entropy without materialising the logits."""
        h = self.hidden_states(input_ids)
        h2 = h.reshape(-1, h.shape[-1])
        w = None
        if h.is_cuda and self.compute_dtype != torch.float32:
            w = cached_cast(self.lm_head.weight, self.compute_dtype, self._head_cache)
        return linear_cross_entropy(h2, self.lm_head.weight, targets.reshape(-1), w_compute=w)


def model_args(**overrides):
    """Namespace with the reference trainer's model defaults (train.py:1904-2101)."""
    base = dict(layers=12, d_model=768, heads=12, ffn_dim=2048, seq_len=256, activation="silu",
                rational_init="silu", rational_group_size=256, rational_max_groups=32,
                rational_basis_eps=1e-6, init_std=0.02)
    base.update(overrides)
    return SimpleNamespace(**base)


def preset(name: str, **overrides):
    """Named configurations of the published studies."""
    presets = {
        "18l_1024d": dict(layers=18, d_model=1024, heads=16, ffn_dim=3072),
        "12l_768d": dict(layers=12, d_model=768, heads=12, ffn_dim=2048),
    }
    cfg = dict(presets[name])
    cfg.update(overrides)
    return model_args(**cfg)
