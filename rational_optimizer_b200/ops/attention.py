"""Causal self-attention core with interleaved-pair RoPE.

``qkv`` is the fused projection output ``[B*S, 3*d]`` (q | k | v, heads
contiguous), as produced by ``CausalSelfAttention.qkv`` of the reference
(training/train.py:48-73).  CUDA: one kernel splits q/k/v into token-major
``[B, S, H, hd]`` storage returned as ``[B, H, S, hd]`` views, applying RoPE
to q and k (fp32 tables); its backward applies the inverse rotation and
re-packs into ``[B*S, 3d]``.  The attention runs PyTorch's SDPA (cuDNN on
sm_100), which allocates its output and gradients in the layout of q, so
the ``[B, S, H*hd]`` output needed by the projection is a view, not a copy.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from .. import _ext


def precompute_rope(seq_len, head_dim, theta=10000.0):
    """fp32 cos/sin tables [1,1,S,hd/2] (same formula as the reference)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    positions = torch.arange(seq_len, dtype=torch.float32)
    freqs = torch.outer(positions, inv_freq)
    return freqs.cos()[None, None, :, :], freqs.sin()[None, None, :, :]


def apply_rope(x, cos, sin):
    x_even = x[..., 0::2]
    x_odd = x[..., 1::2]
    rotated = torch.stack((x_even * cos - x_odd * sin, x_even * sin + x_odd * cos), dim=-1)
    return rotated.flatten(-2)


class _RopeQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos2d, sin2d, B, S, H, hd):
        q, k, v = _ext.ext().rope_qkv_forward(qkv.contiguous(), cos2d, sin2d, B, S, H, hd)
        ctx.save_for_backward(cos2d, sin2d)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos2d, sin2d = ctx.saved_tensors
        dqkv = _ext.ext().rope_qkv_backward(dq, dk, dv, cos2d, sin2d)
        return dqkv, None, None, None, None, None, None


class _QKVRopeFunction(torch.autograd.Function):
    """``q, k, v`` of ``RoPE(x W_qkv^T)`` with the rotation in the GEMM epilogue.

    Forward: ``qkv_rope_forward`` (csrc/gemm2_sm100.cu) writes the rotated q, k
    and v as three token-major ``[B*S, d]`` planes, returned as ``[B, H, S, hd]``
    views, so neither the fused projection output nor a separate RoPE pass is
    materialised.  Backward: the inverse rotation and re-pack
    (``rope_qkv_backward``), then the projection's input and weight gradients
    (the weight gradient accumulates in the GEMM into a managed ``.grad``).
    """

    @staticmethod
    def forward(ctx, x, weight, w_compute, cos2d, sin2d, B, S, H, hd):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != w_compute.dtype:
            x2 = x2.to(w_compute.dtype)
        x2 = x2.contiguous()
        planes = _ext.ext().qkv_rope_forward(x2, w_compute, cos2d, sin2d, S, hd)
        if planes is None:
            raise RuntimeError("fused q/k/v projection rejected a supported shape")
        ctx.save_for_backward(x2, w_compute, cos2d, sin2d)
        ctx.weight = weight
        ctx.in_shape = x.shape
        ctx.x_dtype = x.dtype
        q, k, v = (planes[i].view(B, S, H, hd).transpose(1, 2) for i in range(3))
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        from . import gemm
        from .linear import weight_grad
        x2, w, cos2d, sin2d = ctx.saved_tensors
        dqkv = _ext.ext().rope_qkv_backward(dq, dk, dv, cos2d, sin2d)
        gx = None
        if ctx.needs_input_grad[0]:
            gx = gemm.matmul_nn(dqkv, w).reshape(ctx.in_shape)
            if gx.dtype != ctx.x_dtype:
                gx = gx.to(ctx.x_dtype)
        gw = weight_grad(ctx.weight, dqkv, x2, ctx.needs_input_grad[1])
        return gx, gw, None, None, None, None, None, None, None


def qkv_rope_supported(x, dim, head_dim) -> bool:
    if not (x.is_cuda and x.dtype == torch.bfloat16) or not _ext.available():
        return False
    if os.environ.get("RO_FUSED_QKV_ROPE", "1") == "0":
        return False
    return dim % 256 == 0 and head_dim % 32 == 0 and hasattr(_ext.ext(), "qkv_rope_forward")


def fused_qkv_attention(x, weight, w_compute, batch, seq_len, heads, head_dim, rope_cos, rope_sin):
    """Attention output ``[B, S, H*hd]`` (before the output projection) from the block input."""
    cos2d = rope_cos.reshape(rope_cos.shape[-2], rope_cos.shape[-1]).float().contiguous()
    sin2d = rope_sin.reshape(rope_sin.shape[-2], rope_sin.shape[-1]).float().contiguous()
    q, k, v = _QKVRopeFunction.apply(x, weight, w_compute, cos2d, sin2d, batch, seq_len, heads, head_dim)
    if own_attention_supported(q):
        # the [B, H, S, hd] views are token-major planes: hand the planes over as they are
        planes = [t.transpose(1, 2).reshape(batch, seq_len, heads * head_dim) for t in (q, k, v)]
        return _OwnAttention.apply(*planes, heads, head_dim, True)
    y = causal_attention_core(q, k, v)
    return y.transpose(1, 2).reshape(batch, seq_len, heads * head_dim)


class _OwnAttention(torch.autograd.Function):
    """Attention over token-major ``[B, S, H*hd]`` planes on the package's
    tcgen05 kernels (csrc/attention_sm100.cu): forward saves (o, lse2); the
    backward is deterministic (query-stationary dQ pass, key-stationary dK/dV
    pass, no atomics)."""

    @staticmethod
    def forward(ctx, q, k, v, heads, head_dim, causal):
        scale = 1.0 / math.sqrt(head_dim)
        out = _ext.ext().attention_forward(q, k, v, int(heads), int(head_dim), scale, bool(causal))
        if out is None:
            raise RuntimeError("attention_forward rejected a shape own_attention_supported accepted")
        o, lse2 = out
        ctx.save_for_backward(q, k, v, o, lse2)
        ctx.cfg = (int(heads), int(head_dim), scale, bool(causal))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse2 = ctx.saved_tensors
        heads, head_dim, scale, causal = ctx.cfg
        out = _ext.ext().attention_backward(q, k, v, o, do, lse2, heads, head_dim, scale, causal)
        if out is None:
            raise RuntimeError("attention_backward rejected the forward's tensors")
        dq, dk, dv = out
        return dq, dk, dv, None, None, None


def own_attention_supported(q) -> bool:
    """The package's attention kernels take this ``[B, H, S, hd]`` token-major view.

    Opt-in (``RO_OWN_ATTENTION=1``): at the 18-layer shape the kernels are
    still slower than cuDNN's (forward 0.207 against 0.138 ms, backward 0.775
    against 0.394 ms per layer at 32 x 1024 tokens, one B200).
    """
    if os.environ.get("RO_OWN_ATTENTION", "0") != "1" or not (q.is_cuda and q.dtype == torch.bfloat16):
        return False
    if not _ext.available() or not hasattr(_ext.ext(), "attention_forward"):
        return False
    B, H, S, hd = q.shape
    return hd in (64, 128) and q.stride(3) == 1 and q.stride(1) == hd and q.stride(2) == H * hd \
        and q.stride(0) == S * H * hd


def causal_attention_core(q, k, v):
    """softmax(q k^T / sqrt(hd) + causal mask) v for [B, H, S, hd] tensors."""
    return F.scaled_dot_product_attention(q, k, v, is_causal=True)


def causal_self_attention(qkv, batch, seq_len, heads, head_dim, rope_cos, rope_sin):
    """Return the attention output ``[B, S, H*hd]`` before the output projection."""
    d = heads * head_dim
    if qkv.is_cuda:
        cos2d = rope_cos.reshape(rope_cos.shape[-2], rope_cos.shape[-1]).float().contiguous()
        sin2d = rope_sin.reshape(rope_sin.shape[-2], rope_sin.shape[-1]).float().contiguous()
        q, k, v = _RopeQKV.apply(qkv.reshape(batch * seq_len, 3 * d), cos2d, sin2d, batch,
                                 seq_len, heads, head_dim)
        y = causal_attention_core(q, k, v)
        return y.transpose(1, 2).reshape(batch, seq_len, d)
    q, k, v = qkv.reshape(batch, seq_len, 3 * d).chunk(3, dim=-1)
    q = q.reshape(batch, seq_len, heads, head_dim).transpose(1, 2)
    k = k.reshape(batch, seq_len, heads, head_dim).transpose(1, 2)
    v = v.reshape(batch, seq_len, heads, head_dim).transpose(1, 2)
    cos = rope_cos[:, :, :seq_len, :].to(dtype=q.dtype)
    sin = rope_sin[:, :, :seq_len, :].to(dtype=q.dtype)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return y.transpose(1, 2).reshape(batch, seq_len, d)


def flash_attention_forward(q, k, v, heads, head_dim, *, causal=True, scale=None):
    """Own tcgen05 attention forward over token-major planes.

    ``q``, ``k``, ``v``: bf16 ``[B, S, ld]`` (head ``h`` at columns
    ``h*head_dim``).  Returns ``(o [B, S, heads*head_dim] bf16, lse2 [B, heads, S]
    fp32)`` with ``lse2`` in log2 units of the scaled scores, or None when the
    kernel does not support the arguments.
    """
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    out = _ext.ext().attention_forward(q, k, v, int(heads), int(head_dim), scale, bool(causal))
    return None if out is None else (out[0], out[1])


def attention_reference(q, k, v, heads, head_dim, *, causal=True, scale=None):
    """fp32 oracle of :func:`flash_attention_forward`: (o, lse2) from ``[B, S, ld]`` planes."""
    B, S, _ = q.shape
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)

    def split(t):
        return t[..., : heads * head_dim].float().reshape(B, S, heads, head_dim).transpose(1, 2)

    qf, kf, vf = split(q), split(k), split(v)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2).reshape(B, S, heads * head_dim), lse / math.log(2.0)
