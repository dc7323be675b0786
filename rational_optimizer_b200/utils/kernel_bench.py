"""Per-kernel timing and roofline fractions at the 18-layer training shapes.

    python -m rational_optimizer_b200.utils.kernel_bench [--case grain_fwd,grain_bwd,...]
        [--rows 32768] [--iters 20] [--warmup 3]

Each case times one launch of this package's kernel with CUDA events on the
launching stream after ``--warmup`` untimed launches, writing a 512 MiB
buffer between timed launches so every launch starts with a cold L2.  It
prints one JSON line per case: median time, algorithmic bytes (or FLOPs) per
launch, achieved GB/s (TFLOP/s) and the fraction of the measured copy
bandwidth (cuBLAS bf16 throughput) from MEASURED_PEAKS.json next to the
package, or of the fallback figures 6.65 TB/s and 1.59 PFLOP/s when absent.

Shapes (training step of the 18L/1024d model at batch 32 x 1024 tokens):
rows = 32768 tokens, d = 1024, GRAIN hidden 4608 in 18 groups, vocab 50304.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from .. import _ext
from ..ops.grain import GRAIN_DENOMINATOR, GRAIN_NUMERATOR

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _time(fn, iters, warmup):
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def cases(rows):
    C = _ext.ext()
    dev = "cuda"
    bf, f32 = torch.bfloat16, torch.float32
    d, H, G, V = 1024, 4608, 18, 50304
    heads, hd, S = 16, 64, 1024
    B = rows // S
    out = {}

    def grain_inputs():
        x = torch.randn(rows, H, device=dev, dtype=bf)
        gy = torch.randn(rows, H, device=dev, dtype=bf)
        num = torch.tensor(GRAIN_NUMERATOR, device=dev).repeat(G, 1)
        den = torch.tensor(GRAIN_DENOMINATOR, device=dev).repeat(G, 1)
        e = torch.empty(G, 0, device=dev)
        return x, gy, num, den, torch.empty(G, 0, 2, device=dev), e, e

    def grain_fwd():
        x, _, num, den, lg, c, b = grain_inputs()
        return (lambda: C.grain_forward(x, num, den, lg, c, b, 0.0, 1e-6, H, G, -1, False)), 2 * x.numel() * 2, 0

    def grain_bwd():
        x, gy, num, den, lg, c, b = grain_inputs()
        return (lambda: C.grain_backward(gy, x, num, den, lg, c, b, 0.0, 1e-6, H, G, None, None)), 3 * x.numel() * 2, 0

    def add_norm_fwd():
        x = torch.randn(rows, d, device=dev, dtype=f32)
        delta = torch.randn(rows, d, device=dev, dtype=bf)
        w = torch.ones(d, device=dev)
        return (lambda: C.add_rmsnorm_forward(x, delta, w, 1e-6)), rows * d * (4 + 2 + 4 + 2), 0

    def add_norm_bwd():
        x = torch.randn(rows, d, device=dev, dtype=f32)
        w = torch.ones(d, device=dev)
        dy = torch.randn(rows, d, device=dev, dtype=bf)
        dres = torch.randn(rows, d, device=dev, dtype=f32)
        _, _, rstd = C.add_rmsnorm_forward(x, torch.zeros(rows, d, device=dev, dtype=bf), w, 1e-6)
        return (lambda: C.add_rmsnorm_backward(dy, dres, x, w, rstd, True)), rows * d * (2 + 4 + 4 + 4 + 2), 0

    def rope_fwd():
        qkv = torch.randn(rows, 3 * d, device=dev, dtype=bf)
        pos = torch.arange(S, device=dev, dtype=f32)
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=dev, dtype=f32) / hd))
        fr = torch.outer(pos, inv)
        cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
        return (lambda: C.rope_qkv_forward(qkv, cos, sin, B, S, heads, hd)), 2 * qkv.numel() * 2, 0

    def rope_bwd():
        # gradients in the token-major storage the attention produces
        q = torch.randn(B, S, heads, hd, device=dev, dtype=bf).transpose(1, 2)
        k = torch.randn(B, S, heads, hd, device=dev, dtype=bf).transpose(1, 2)
        v = torch.randn(B, S, heads, hd, device=dev, dtype=bf).transpose(1, 2)
        pos = torch.arange(S, device=dev, dtype=f32)
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=dev, dtype=f32) / hd))
        fr = torch.outer(pos, inv)
        cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
        return (lambda: C.rope_qkv_backward(q, k, v, cos, sin)), 6 * q.numel() * 2, 0

    def cross_entropy():
        n = 8192
        logits = torch.randn(n, V, device=dev, dtype=bf)
        tgt = torch.randint(0, V, (n,), device=dev)
        return (lambda: C.cross_entropy_fwd_bwd(logits, tgt, 1.0 / n, -100)), 2 * logits.numel() * 2, 0

    def gemm_in_proj():
        a = torch.randn(rows, d, device=dev, dtype=bf)
        b = torch.randn(H, d, device=dev, dtype=bf)
        return (lambda: C.gemm_bf16(a, b, False, True, False)), 0, 2.0 * rows * d * H

    def gemm2_in_proj():
        a = torch.randn(rows, d, device=dev, dtype=bf)
        b = torch.randn(H, d, device=dev, dtype=bf)
        return (lambda: C.gemm2_bf16(a, b)), 0, 2.0 * rows * d * H

    def grain_in_proj_fused():
        a = torch.randn(rows, d, device=dev, dtype=bf)
        b = (torch.randn(H, d, device=dev) * 0.03).to(bf)
        num = torch.tensor(GRAIN_NUMERATOR, device=dev).repeat(G, 1)
        den = torch.tensor(GRAIN_DENOMINATOR, device=dev).repeat(G, 1)
        return (lambda: C.grain_in_proj_forward(a, b, num, den, 1e-6)), 0, 2.0 * rows * d * H

    def grain_in_proj_unfused():
        a = torch.randn(rows, d, device=dev, dtype=bf)
        b = (torch.randn(H, d, device=dev) * 0.03).to(bf)
        num = torch.tensor(GRAIN_NUMERATOR, device=dev).repeat(G, 1)
        den = torch.tensor(GRAIN_DENOMINATOR, device=dev).repeat(G, 1)
        e = torch.empty(G, 0, device=dev)
        e3 = torch.empty(G, 0, 2, device=dev)

        def run():
            h = a @ b.t()
            return C.grain_forward(h, num, den, e3, e, e, 0.0, 1e-6, H, G, -1, False)
        return run, 0, 2.0 * rows * d * H

    def _grain_bwd_inputs():
        dO = torch.randn(rows, d, device=dev, dtype=bf)
        w_out = (torch.randn(d, H, device=dev) * 0.03).to(bf)
        h = torch.randn(rows, H, device=dev, dtype=bf)
        num = torch.tensor(GRAIN_NUMERATOR, device=dev).repeat(G, 1)
        den = torch.tensor(GRAIN_DENOMINATOR, device=dev).repeat(G, 1)
        return dO, w_out, h, num, den

    def grain_out_proj_bwd_fused():
        dO, w_out, h, num, den = _grain_bwd_inputs()
        wt = w_out.t().contiguous()
        return (lambda: C.grain_out_proj_backward(dO, wt, h, num, den, 1e-6)), 0, 2.0 * rows * d * H

    def grain_out_proj_bwd_unfused():
        dO, w_out, h, num, den = _grain_bwd_inputs()
        e, e3 = torch.empty(G, 0, device=dev), torch.empty(G, 0, 2, device=dev)

        def run():
            gy = dO @ w_out
            return C.grain_backward(gy, h, num, den, e3, e, e, 0.0, 1e-6, H, G, None, None)
        return run, 0, 2.0 * rows * d * H

    def gemm_in_proj_cublas():
        a = torch.randn(rows, d, device=dev, dtype=bf)
        b = torch.randn(H, d, device=dev, dtype=bf)
        return (lambda: a @ b.t()), 0, 2.0 * rows * d * H

    def _ns5(native):
        from ..optim.newton_schulz import ns5_grouped_bf16
        B, r, c = 18 * G, 256, d  # router incoming blocks of one step
        x = torch.randn(B, r, c, device=dev, dtype=bf)
        flops = 5 * B * (2.0 * r * r * c + 2.0 * r * r * r + 2.0 * r * r * c)
        return (lambda: ns5_grouped_bf16(x, native=native)), 0, flops

    def ns5_router_cublas():
        return _ns5(False)

    def ns5_router_native():
        return _ns5(True)

    def _ns5_muon(native):
        # Muon's MLP matrices of all layers in one batch, wide orientation
        from ..optim.newton_schulz import ns5_grouped_bf16
        B, r, c = 18, d, H
        x = torch.randn(B, r, c, device=dev, dtype=bf)
        flops = 5 * B * (2.0 * r * r * c + 2.0 * r * r * r + 2.0 * r * r * c)
        return (lambda: ns5_grouped_bf16(x, native=native)), 0, flops

    def ns5_muon_mlp_cublas():
        return _ns5_muon(False)

    def ns5_muon_mlp_native():
        return _ns5_muon(True)

    def _attn_planes():
        B, S, Hh, hd = rows // 1024, 1024, 16, 64
        q, k, v = (torch.randn(B, S, Hh * hd, device=dev, dtype=bf) for _ in range(3))
        flops = 4.0 * B * Hh * hd * S * (S + 1) / 2  # causal: QK^T and PV over the lower triangle
        return q, k, v, B, S, Hh, hd, flops

    def attn_fwd():
        from ..ops.attention import flash_attention_forward
        q, k, v, B, S, Hh, hd, flops = _attn_planes()
        return (lambda: flash_attention_forward(q, k, v, Hh, hd)), 0, flops

    def attn_fwd_sdpa():
        q, k, v, B, S, Hh, hd, flops = _attn_planes()
        views = [t.view(B, S, Hh, hd).transpose(1, 2) for t in (q, k, v)]

        def run():
            with torch.no_grad():
                torch.nn.functional.scaled_dot_product_attention(*views, is_causal=True)
        return run, 0, flops

    def attn_bwd():
        from ..ops.attention import flash_attention_forward
        q, k, v, B, S, Hh, hd, flops = _attn_planes()
        o, lse2 = flash_attention_forward(q, k, v, Hh, hd)
        do = torch.randn_like(o)
        # algorithmic FLOPs of the backward (5 products; the two-pass kernel
        # recomputes two of them, not counted)
        return (lambda: C.attention_backward(q, k, v, o, do, lse2, Hh, hd, hd ** -0.5, True)), 0, flops * 2.5

    def attn_bwd_sdpa():
        q, k, v, B, S, Hh, hd, flops = _attn_planes()
        views = [t.view(B, S, Hh, hd).transpose(1, 2).detach().requires_grad_() for t in (q, k, v)]
        out = torch.nn.functional.scaled_dot_product_attention(*views, is_causal=True)
        do = torch.randn_like(out)

        def run():
            torch.autograd.grad(out, views, do, retain_graph=True)
        return run, 0, flops * 2.5

    def ledger():
        L = 18
        n = L * G
        layer_ids = torch.arange(L, device=dev).repeat_interleave(G)
        pers = torch.randn(64, n, device=dev) * 1e-3
        diag = torch.rand(n, device=dev) * 1e-6
        cross = torch.randn(n, device=dev) * 1e-7
        scal = torch.zeros(8, device=dev)
        scal[3] = 1e-3
        ws = torch.empty(int(C.tiller_ledger_workspace(n)), device=dev, dtype=torch.float64)
        exact = (torch.rand(2, n, device=dev) + 0.1) * 1e-3
        mom = (torch.rand(2, n, device=dev) + 0.1) * 1e-3
        w = torch.rand(n, device=dev) + 0.5
        dd = torch.full((1,), 1e-5, device=dev)
        p0, d0, c0, s0 = pers.clone(), diag.clone(), cross.clone(), scal.clone()

        def run():
            pers.copy_(p0)
            diag.copy_(d0)
            cross.copy_(c0)
            scal.copy_(s0)
            C.tiller_ledger_transaction(None, None, exact, mom, w, layer_ids, dd, pers, diag, cross, scal, ws,
                                        64, L, 3e-4)
        return run, 0, 0

    for name, fn in [("grain_fwd", grain_fwd), ("grain_bwd", grain_bwd), ("add_rmsnorm_fwd", add_norm_fwd),
                     ("add_rmsnorm_bwd", add_norm_bwd), ("rope_fwd", rope_fwd), ("rope_bwd", rope_bwd),
                     ("cross_entropy", cross_entropy), ("gemm_in_proj", gemm_in_proj),
                     ("gemm_in_proj_cublas", gemm_in_proj_cublas),
                     ("gemm2_in_proj", gemm2_in_proj), ("grain_in_proj_fused", grain_in_proj_fused),
                     ("grain_in_proj_unfused", grain_in_proj_unfused),
                     ("grain_out_proj_bwd_fused", grain_out_proj_bwd_fused),
                     ("grain_out_proj_bwd_unfused", grain_out_proj_bwd_unfused), ("ns5_router_cublas", ns5_router_cublas),
                     ("ns5_router_native", ns5_router_native), ("ns5_muon_mlp_cublas", ns5_muon_mlp_cublas),
                     ("ns5_muon_mlp_native", ns5_muon_mlp_native), ("ledger", ledger),
                     ("attn_fwd", attn_fwd), ("attn_fwd_sdpa", attn_fwd_sdpa), ("attn_bwd", attn_bwd),
                     ("attn_bwd_sdpa", attn_bwd_sdpa)]:
        out[name] = fn
    return out


def ledger_phases(layers=18, groups=18, steps=10, functional_every=3):
    """Phase times of the ledger + transaction kernel from its ``%globaltimer``
    stamps: one JSON line per call, a functional (refresh) call every
    ``functional_every`` calls, the rest surrogate calls."""
    C = _ext.ext()
    dev = "cuda"
    n = layers * groups
    gen = torch.Generator(device=dev).manual_seed(7)
    layer_ids = torch.arange(layers, device=dev).repeat_interleave(groups)
    pers = torch.zeros(64, n, device=dev)
    diag = torch.zeros(n, device=dev)
    cross = torch.zeros(n, device=dev)
    scal = torch.zeros(8, device=dev)
    ws = torch.empty(int(C.tiller_ledger_workspace(n)), device=dev, dtype=torch.float64)
    timing = torch.zeros(16, dtype=torch.int64, device=dev)
    # stamp index -> the phase that ends there
    names = {1: "gram", 2: "gram_eigensolve", 3: "persistent_rows", 4: "transaction_setup", 6: "lanczos",
             7: "tridiagonal_eigensolve", 8: "projection", 9: "acceptance"}
    prev = 0
    for step in range(steps):
        functional = step % functional_every == 0
        exact = (torch.rand(2, n, device=dev, generator=gen) + 0.1) * 1e-3
        mom = (torch.rand(2, n, device=dev, generator=gen) + 0.1) * 1e-3
        w = torch.rand(n, device=dev, generator=gen) + 0.5
        sc = torch.randn(32, n, device=dev, generator=gen) * 1e-3
        dc = torch.randn(32, device=dev, generator=gen) * 1e-4
        dd = torch.randn((), device=dev, generator=gen).abs().reshape(1) * 1e-4
        timing.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        C.tiller_ledger_transaction(sc if functional else None, dc if functional else None, exact, mom, w,
                                    layer_ids, None if functional else dd, pers, diag, cross, scal, ws, prev,
                                    layers, 3e-4, timing=timing)
        end.record()
        torch.cuda.synchronize()
        t = timing.tolist()
        phases, last = {}, t[0]
        for k in sorted(names):
            if t[k]:
                phases[names[k]] = round((t[k] - last) / 1e3, 1)
                last = t[k]
        print(json.dumps({"case": "ledger_phases", "call": step, "functional": functional, "prev_rows": prev,
                          "ms": round(start.elapsed_time(end), 3), "gram_sweeps": t[12],
                          "tridiagonal_sweeps": t[13], "phase_us": phases}), flush=True)
        prev = 32 if prev == 0 else 64


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--rows", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    hbm, tflops, kind = peaks()
    if a.case == "ledger_phases":
        ledger_phases()
        return
    table = cases(a.rows)
    names = list(table) if a.case == "all" else a.case.split(",")
    for name in names:
        fn, nbytes, flops = table[name]()
        ms = _time(fn, a.iters, a.warmup)
        rec = {"case": name, "rows": a.rows, "ms": round(ms, 4)}
        if nbytes:
            gbs = nbytes / ms / 1e6
            rec.update(bytes=nbytes, gb_s=round(gbs, 1), frac_hbm=round(gbs / hbm, 3), peak=kind)
        if flops:
            tf = flops / ms / 1e9
            rec.update(flops=flops, tflops=round(tf, 1), frac_bf16=round(tf / tflops, 3), peak=kind)
        print(json.dumps(rec), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
