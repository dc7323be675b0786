"""CUDA execution of TILLER's per-role direction pipeline (csrc/tiller.cu).

Per role the work is: one Nesterov pass that also writes the grouped fp32
copies of ``m`` and ``g`` and the bf16 Newton-Schulz input (transposing the
outgoing / attention-output roles on the fly), one batched NS5 on tcgen05
GEMMs, three reduction kernels that update the factorized second moments and
produce the seven block inner products, one tiny kernel that evaluates the
adaptive-tangent chord and the exact/momentum/budget contractions, and one
apply pass (fused with the inverse layout map) after the transaction has
chosen the block coefficients.  The mathematics is that of
:func:`rational_optimizer_b200.optim.tiller_math.adaptive_tangent_chord`.
"""
from __future__ import annotations

import math

import torch
from torch.autograd.graph import increment_version

from .. import _ext
from .newton_schulz import match_rms_adamw_adjustment, ns5_grouped_bf16


def available() -> bool:
    if not _ext.available():
        return False
    C = _ext.ext()
    return all(hasattr(C, n) for n in ("tiller_nesterov", "tiller_chord", "tiller_apply", "ns_normalize"))


def _momentum_buffers(optimizer, params):
    bufs = []
    for p in params:
        st = optimizer.state[p]
        buf = st.get("momentum_buffer")
        if buf is None:
            buf = torch.zeros_like(p)
            st["momentum_buffer"] = buf
        bufs.append(buf)
    return bufs


class FusedRole:
    """One role (set of L same-shape matrices) of TILLER on the GPU.

    ``kind``: ``"incoming"`` ([H, d], G row blocks), ``"outgoing"`` ([d, H],
    transposed to [H, d], G row blocks), ``"qkv"`` / ``"attn_out"`` (one block
    per layer, head-group NS5).
    """

    def __init__(self, optimizer, params, kind, *, groups=1, width=None, momentum=0.95):
        self.opt = optimizer
        self.params = params
        self.kind = kind
        self.momentum = momentum
        self.L = len(params)
        rows, cols = params[0].shape
        self.adj = match_rms_adamw_adjustment(params[0].shape)
        if kind == "incoming":
            self.transpose = False
            self.G, self.R, self.C = groups, width, cols
            self.scale = math.sqrt(min(rows, cols) / (groups * min(width, cols)))
        elif kind == "outgoing":
            self.transpose = True
            self.G, self.R, self.C = groups, width, rows
            self.scale = math.sqrt(min(rows, cols) / (groups * min(rows, width)))
        elif kind == "qkv":
            self.transpose = False
            self.G, self.R, self.C = 1, rows, cols
            self.scale = 1.0 / math.sqrt(3.0)
        elif kind == "attn_out":
            self.transpose = False
            self.G, self.R, self.C = 1, rows, cols
            self.scale = 1.0
        else:
            raise ValueError(kind)
        self.nblocks = self.L * self.G

    def directions(self, row_m, col_m, participation, congruence, step, *, want_selected):
        C = _ext.ext()
        grads = [p.grad for p in self.params]
        bufs = _momentum_buffers(self.opt, self.params)
        m, g, m16 = C.tiller_nesterov(grads, bufs, self.transpose, self.momentum)
        if self.kind in ("incoming", "outgoing"):
            polar = ns5_grouped_bf16(m16.view(self.nblocks, self.R, self.C))
        elif self.kind == "qkv":
            L, r, c = m16.shape
            polar = ns5_grouped_bf16(_qkv_blocks(m16)).view(L, r, c)
        else:  # attention output: NS on per-layer transposed column blocks
            mt = C.tiller_transpose_bf16(m16)
            L, r, c = mt.shape
            pt = ns5_grouped_bf16(_out_blocks(mt)).view(L, r, c)
            polar = C.tiller_transpose_bf16(pt.contiguous())
        self.m, self.g, self.polar = m, g, polar.contiguous()
        self.row_m, self.col_m = row_m, col_m
        self.step_index = int(step)
        chord, row_total = C.tiller_chord(self.polar, m, g, row_m, col_m,
                                          participation.reshape(-1).float().contiguous(),
                                          congruence.reshape(-1).float().contiguous(), self.nblocks,
                                          self.R, self.C, self.scale, int(step), self.adj)
        self.chord, self.row_total = chord, row_total
        selected = None
        if want_selected:
            ones = torch.ones(self.nblocks, device=m.device, dtype=torch.float32)
            selected = C.tiller_apply(self.params, self.polar, m, row_m, col_m, row_total, chord, ones,
                                      True, False, self.G, self.R, self.C, self.transpose, self.scale,
                                      int(step), 1.0, 0.0, self.adj)
        return chord, selected

    def apply(self, coefficients, *, decay, lr):
        C = _ext.ext()
        coef = coefficients.reshape(-1).float().contiguous()
        C.tiller_apply(self.params, self.polar, self.m, self.row_m, self.col_m, self.row_total,
                       self.chord, coef, False, True, self.G, self.R, self.C, self.transpose,
                       self.scale, self.step_index, float(decay), -float(lr) * self.adj, self.adj)
        for p in self.params:
            increment_version(p)
        self.m = self.g = self.polar = None


def _qkv_blocks(m16):
    """[L, 3d, d] -> [L*3*4, 4*d/16, d] head-group blocks (contiguous view)."""
    L, r, c = m16.shape
    block = 4 * (c // 16)
    return m16.view(L * (r // block), block, c)


def _out_blocks(mt):
    """Transposed attention output [L, d, d] -> [L*4, d/4, d] blocks (contiguous view)."""
    L, r, c = mt.shape
    block = 4 * (r // 16)
    return mt.view(L * (r // block), block, c)


def chord_meta(chord):
    return {"safe": chord[:, 5] > 0.5, "parent_cosine": chord[:, 7], "departure_energy": chord[:, 9],
            "parent_coefficient": chord[:, 0], "adaptive_coefficient": chord[:, 1]}
