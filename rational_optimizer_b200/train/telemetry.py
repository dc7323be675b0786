"""Training telemetry: GRAIN statistics, weight spectra, the fixed probe batch,
optimizer telemetry and GPU metadata (reference training/train.py:845-1343).

Record keys and definitions are the reference's, so JSONL trajectories from
both frameworks aggregate with the same tools.  Everything here runs off the
hot path: on log/eval steps only, on sampled rows or fixed probe inputs.
"""
from __future__ import annotations

import math
import os
import re
import subprocess

import torch
import torch.nn.functional as F

from ..models.transformer import GRAIN_ACTIVATION_IDS, GRAINMLP
from ..optim.composite import collect_rlb_optimizer_groups, unwrap_model
from ..parallel.dist import reduce_mean
from .data import sample_batch
from .tokens import sanitize_name

GPU_FIELDS = ["index", "uuid", "name", "pci.bus_id", "clocks.max.sm", "power.limit", "pstate",
              "utilization.gpu", "memory.used", "driver_version"]


def finite_float(value):
    if value is None:
        return None
    value = float(value)
    return value if math.isfinite(value) else None


def _mean_std(t):
    if t is None or not torch.is_tensor(t) or t.numel() == 0:
        return None, None
    v = t.detach().float().reshape(-1)
    return finite_float(v.mean().item()), finite_float(v.std(unbiased=False).item() if v.numel() > 1 else 0.0)


def _quantiles(t):
    if t is None or not torch.is_tensor(t) or t.numel() == 0:
        return None, None, None
    v = t.detach().float().reshape(-1).cpu()
    return (finite_float(v.min().item()), finite_float(torch.quantile(v, 0.01).item()),
            finite_float(v.median().item()))


def nvidia_smi_metadata(strict=False, expected_count=None, expected_name=None):
    """Rows of ``nvidia-smi --query-gpu`` for the visible GPUs (None if unavailable).

    ``strict`` raises instead of returning None, and checks the GPU count and
    model name when they are given.
    """
    try:
        cmd = ["nvidia-smi"]
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        if visible:
            cmd += ["-i", visible]
        cmd += [f"--query-gpu={','.join(GPU_FIELDS)}", "--format=csv,noheader,nounits"]
        out = subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=30).stdout
        rows = []
        for line in out.splitlines():
            if not line.strip():
                continue
            values = [v.strip() for v in line.split(",")]
            if len(values) != len(GPU_FIELDS):
                raise RuntimeError(f"unexpected nvidia-smi row: {line!r}")
            rows.append(dict(zip(GPU_FIELDS, values)))
        if strict and expected_count is not None and len(rows) != int(expected_count):
            raise RuntimeError(f"expected {expected_count} visible GPUs, found {len(rows)}")
        if strict and expected_name and any(expected_name not in r["name"] for r in rows):
            raise RuntimeError(f"expected only {expected_name} GPUs, found {[r['name'] for r in rows]}")
        return rows
    except (FileNotFoundError, subprocess.CalledProcessError, subprocess.TimeoutExpired, RuntimeError):
        if strict:
            raise
        return None


# ---------------------------------------------------------------------------
# Optimizer telemetry (walks composite optimizers)

def iter_optimizer_tree(optimizer):
    yield optimizer
    for child in getattr(optimizer, "optimizers", []):
        yield from iter_optimizer_tree(child)
    for attr in ("adam", "muon"):
        child = getattr(optimizer, attr, None)
        if child is not None:
            yield child


def set_optimizer_telemetry_capture(optimizer, enabled):
    for item in iter_optimizer_tree(optimizer):
        setter = getattr(item, "set_telemetry_capture", None)
        if setter is not None:
            setter(enabled)


def collect_optimizer_telemetry(optimizer):
    record = {}
    for item in iter_optimizer_tree(optimizer):
        getter = getattr(item, "telemetry", None)
        if getter is not None:
            values = getter()
            if values:
                record.update(values)
    return record


def optimizer_method_specific_sync_active(optimizer):
    checker = getattr(optimizer, "method_specific_sync_active", None)
    return True if checker is None else bool(checker())


def parse_optimizer_telemetry_steps(value, total_steps):
    """Optional ascending list of steps that capture optimizer telemetry."""
    if value in (None, ""):
        return None
    if not isinstance(value, str) or re.fullmatch(r"[1-9][0-9]*(?:,[1-9][0-9]*)*", value) is None:
        raise RuntimeError("TILLER_OPTIMIZER_TELEMETRY_STEPS must be ascending comma-separated positive steps")
    steps = tuple(int(v) for v in value.split(","))
    if tuple(sorted(set(steps))) != steps or steps[-1] > int(total_steps):
        raise RuntimeError("TILLER_OPTIMIZER_TELEMETRY_STEPS is duplicated, unordered, or beyond the run")
    return steps


# ---------------------------------------------------------------------------
# GRAIN telemetry

def enable_rlb_training_telemetry(model, args):
    if not getattr(args, "grain_training_telemetry", True) or args.activation not in GRAIN_ACTIVATION_IDS:
        return
    for module in model.modules():
        if all(hasattr(module, a) for a in ("groups", "hidden_dim", "numerator", "denominator")):
            module._rlb_optimizer_track_stats = True
            module._rlb_optimizer_stat_every = max(1, int(args.telemetry_rlb_stat_every))
            module._rlb_optimizer_stat_samples = max(1, int(args.telemetry_rlb_stat_samples))


def rlb_live_stats_scope(model):
    tracked = consumed = False
    for module in unwrap_model(model).modules():
        if not bool(getattr(module, "_rlb_optimizer_track_stats", False)):
            continue
        tracked = True
        consumed = consumed or bool(getattr(module, "_rlb_optimizer_sync_stats", False))
    if consumed:
        return "optimizer_gains_global_weighted_train_only"
    return "telemetry_only" if tracked else "disabled"


def denominator_probe(group, points=129, probe_range=5.0):
    """|Q(t)| of every group on an evenly spaced grid of ``points`` in [-range, range]."""
    module = group.get("module")
    den = getattr(module, "denominator", None) if module is not None else None
    if den is None:
        return None
    d = den.detach().float().abs()
    if d.dim() != 2 or d.size(-1) < 4:
        return None
    t = torch.linspace(-float(probe_range), float(probe_range), int(points), device=d.device)
    at, t2 = t.abs(), t.square()
    q = 1.0 + d[:, 0:1] * at + d[:, 1:2] * t2 + d[:, 2:3] * (at * t2) + d[:, 3:4] * t2.square()
    values = [q.reshape(-1)]
    centers, beta = getattr(module, "centers", None), getattr(module, "beta", None)
    if centers is not None and beta is not None:
        c = centers.detach().float().unsqueeze(-1)
        b = beta.detach().float().unsqueeze(-1).clamp_min(0.0)
        values.append((1.0 + b * (t.view(1, 1, -1) - c).square()).reshape(-1))
    return torch.cat(values)


def collect_rlb_telemetry(model, args):
    if not getattr(args, "grain_training_telemetry", True) or args.activation not in GRAIN_ACTIVATION_IDS:
        return {}
    groups = collect_rlb_optimizer_groups(unwrap_model(model), args)
    if not groups:
        return {}
    keys = ("output_rms", "derivative_rms", "atom_rms", "abs_moments")
    means = {k: [] for k in keys}
    stds = {k: [] for k in keys}
    dmin, dp01, dmed = [], [], []
    win_m, win_s, wout_m, wout_s, log_ratio, log_prod = [], [], [], [], [], []
    for group in groups:
        module = group.get("module")
        stats = getattr(module, "_rlb_optimizer_stats", None) if module is not None else None
        for k in keys:
            m, s = _mean_std(None if not stats else stats.get(k))
            means[k].append(m)
            stds[k].append(s)
        lo, p01, med = _quantiles(denominator_probe(group, args.telemetry_denominator_probe_points))
        dmin.append(lo)
        dp01.append(p01)
        dmed.append(med)
        G, H = int(group["groups"]), int(group["hidden_dim"])
        w = H // G
        win = group["in_weight"].detach().float().view(G, w, -1)
        wout = group["out_weight"].detach().float()
        wout = wout.view(wout.shape[0], G, w).permute(1, 2, 0)
        rin = torch.sqrt(win.square().mean(dim=(1, 2)) + 1e-12)
        rout = torch.sqrt(wout.square().mean(dim=(1, 2)) + 1e-12)
        for target_m, target_s, r in ((win_m, win_s, rin), (wout_m, wout_s, rout)):
            m, s = _mean_std(r)
            target_m.append(m)
            target_s.append(s)
        log_ratio.append(finite_float((torch.log(rin) - torch.log(rout)).mean().item()))
        log_prod.append(finite_float((torch.log(rin) + torch.log(rout)).mean().item()))
    return {
        "grain_output_rms_mean_by_layer": means["output_rms"],
        "grain_output_rms_std_by_layer": stds["output_rms"],
        "grain_derivative_rms_mean_by_layer": means["derivative_rms"],
        "grain_derivative_rms_std_by_layer": stds["derivative_rms"],
        "grain_atom_rms_mean_by_layer": means["atom_rms"],
        "grain_atom_rms_std_by_layer": stds["atom_rms"],
        "grain_abs_moment_mean_by_layer": means["abs_moments"],
        "grain_abs_moment_std_by_layer": stds["abs_moments"],
        "denominator_abs_min_by_layer": dmin,
        "denominator_abs_p01_by_layer": dp01,
        "denominator_abs_median_by_layer": dmed,
        "w_in_rms_mean_by_layer": win_m,
        "w_in_rms_std_by_layer": win_s,
        "w_out_rms_mean_by_layer": wout_m,
        "w_out_rms_std_by_layer": wout_s,
        "log_w_in_over_w_out_by_layer": log_ratio,
        "log_norm_product_by_layer": log_prod,
    }


# ---------------------------------------------------------------------------
# Weight spectra

def svd_entropy(matrix, max_dim):
    """Normalised entropy of the singular values of an evenly subsampled matrix."""
    w = matrix.detach().float()
    if w.dim() != 2 or min(w.shape) <= 1:
        return None
    rows, cols = w.shape
    if max_dim > 0 and rows > max_dim:
        w = w.index_select(0, torch.linspace(0, rows - 1, max_dim, device=w.device).long())
    if max_dim > 0 and cols > max_dim:
        w = w.index_select(1, torch.linspace(0, cols - 1, max_dim, device=w.device).long())
    try:
        sv = torch.linalg.svdvals(w)
    except RuntimeError:
        return None
    sv = sv.clamp_min(0.0)
    total = sv.sum()
    if not torch.isfinite(total) or total <= 0:
        return None
    p = sv / total
    h = -(p * torch.log(p.clamp_min(1e-12))).sum()
    return finite_float((h / math.log(max(2, p.numel()))).item())


def collect_matrix_spectrum_telemetry(model, args):
    if args.matrix_spectrum_interval <= 0:
        return {}
    raw = unwrap_model(model)
    values = {k: [] for k in ("svd_entropy_attn_q", "svd_entropy_attn_k", "svd_entropy_attn_v",
                              "svd_entropy_attn_o", "svd_entropy_grain_in", "svd_entropy_grain_out")}

    def add(key, weight):
        v = svd_entropy(weight, args.matrix_spectrum_max_dim)
        if v is not None:
            values[key].append(v)

    for layer in getattr(raw, "layers", []):
        attn = getattr(layer, "attn", None)
        if attn is not None and hasattr(attn, "qkv"):
            q, k, v = attn.qkv.weight.chunk(3, dim=0)
            add("svd_entropy_attn_q", q)
            add("svd_entropy_attn_k", k)
            add("svd_entropy_attn_v", v)
        if attn is not None and hasattr(attn, "out"):
            add("svd_entropy_attn_o", attn.out.weight)
        mlp = getattr(layer, "mlp", None)
        if isinstance(mlp, GRAINMLP):
            add("svd_entropy_grain_in", mlp.in_proj.weight)
            add("svd_entropy_grain_out", mlp.out_proj.weight)
    return {k: finite_float(sum(v) / len(v)) for k, v in values.items() if v}


# ---------------------------------------------------------------------------
# Fixed probe batch: logit drift and KL since the previous eval and since step 1

def prepare_probe_batch(tokens, args, offsets, rank, device, out_path, barrier=None):
    if args.probe_batch_size <= 0:
        return None
    gen = torch.Generator(device="cpu")
    gen.manual_seed(args.seed + 2_000_003 + rank)
    x, y = sample_batch(tokens, min(int(args.probe_batch_size), int(args.batch_size)), args.seq_len,
                        offsets, gen, device)
    path = out_path.parent / f"{sanitize_name(args.activation)}_probe_rank{rank}.pt"
    if rank == 0:
        out_path.parent.mkdir(parents=True, exist_ok=True)
    if barrier is not None:
        barrier()
    torch.save({"probe_x": x.detach().cpu(), "probe_y": y.detach().cpu(), "dataset": args.dataset_name,
                "dataset_config": args.dataset_config,
                "validation_skip_tokens": args.validation_skip_tokens, "seed": args.seed, "rank": rank},
               path)
    return {"x": x, "prev_logits": None, "first_logits": None}


@torch.no_grad()
def evaluate_probe(model, probe_state, device, is_distributed):
    if probe_state is None:
        return {}
    model.eval()
    logits = model(probe_state["x"]).detach().float()
    metrics = {"probe_logit_rms": reduce_mean(float(torch.sqrt(logits.square().mean() + 1e-12).item()),
                                              device, is_distributed)}
    for label, ref in (("since_prev_eval", probe_state.get("prev_logits")),
                       ("since_step1", probe_state.get("first_logits"))):
        if ref is None:
            metrics[f"probe_logit_delta_rms_{label}"] = 0.0
            metrics[f"probe_kl_{label}"] = 0.0
            continue
        ref = ref.to(device=device, dtype=torch.float32)
        delta = torch.sqrt((logits - ref).square().mean() + 1e-12)
        lp, rlp = F.log_softmax(logits, dim=-1), F.log_softmax(ref, dim=-1)
        kl = (rlp.exp() * (rlp - lp)).sum(dim=-1).mean()
        metrics[f"probe_logit_delta_rms_{label}"] = reduce_mean(float(delta.item()), device, is_distributed)
        metrics[f"probe_kl_{label}"] = reduce_mean(float(kl.item()), device, is_distributed)
    stored = logits.detach().to(device="cpu", dtype=torch.float16)
    if probe_state.get("first_logits") is None:
        probe_state["first_logits"] = stored.clone()
    probe_state["prev_logits"] = stored
    return metrics


def cpu_probe_state(probe_state):
    if probe_state is None:
        return None
    return {k: None if probe_state.get(k) is None else probe_state[k].detach().cpu()
            for k in ("first_logits", "prev_logits")}
