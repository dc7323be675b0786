"""Pure functions of the TILLER optimizer (no optimizer state).

Each function restates one piece of optimizer_design/_tiller/core.py of the
reference, written as plain tensor programs so they can run replicated on
every rank without collectives:

  probe layout ........ fixed_global_probe_layout / evenly_spaced_indices (core.py:236-268)
  GRAIN factors ....... stacked_factors, evaluate_response (core.py:713-759)
  response adjoint .... response_adjoint (core.py:761-772)
  Jacobian kernels .... jacobian_kernel_inner (core.py:609-632)
  sensor statistics ... intrinsic_and_response_statistics (core.py:774-808),
                        group_participation (core.py:1912-1920),
                        group_congruence / layer_congruence (core.py:2158-2180)
  probe loss scores ... group_scores (core.py:858-881)
  direction ........... adaptive_tangent_chord (core.py:4209-4263)
  ledger .............. rfd_rows, trace_matched_surrogate, functional_row_norm
                        (core.py:1142-1233)
  window rows ......... window32_rows (core.py:3888-3910)
  transaction ......... biatlas_transaction with its Lanczos basis
                        (core.py:69-232)
  accounting .......... tiller_scaling_formula (core.py:4370-4379 and parents)

Host synchronisations that the reference performs for validation are kept
behind ``validate=True`` (the default for CPU tests); the CUDA training path
calls with ``validate=False`` and relies on device-side finiteness flags.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

CURRENT_ROWS = 32
PERSISTENT_ROWS = 64
MAXIMUM_SELECTION_ROWS = 96
KRYLOV_ROWS = 32
MATCHED_BETA2 = 0.95
LOCKED_EPS = 1e-8
REFRESH_INTERVAL = 8
GLOBAL_PROBE_COUNT = 32


# ---------------------------------------------------------------------------
# Probe layout.

@dataclass(frozen=True)
class ProbeLayout:
    global_probe_count: int
    process_count: int
    process_rank: int
    global_start: int
    global_stop: int
    local_probe_count: int


def fixed_global_probe_layout(global_probe_count: int, rank: int, world: int) -> ProbeLayout:
    probes, rank, world = int(global_probe_count), int(rank), int(world)
    if probes < 2 or world < 1 or rank < 0 or rank >= world:
        raise RuntimeError("probe layout needs at least two probes and a rank inside the world")
    start = rank * probes // world
    stop = (rank + 1) * probes // world
    return ProbeLayout(probes, world, rank, start, stop, stop - start)


def evenly_spaced_indices(row_count: int, selected: int, *, device) -> torch.Tensor:
    rows, selected = int(row_count), int(selected)
    if rows < 0 or selected < 0 or selected > rows:
        raise RuntimeError(f"cannot pick {selected} evenly spaced rows out of {rows}")
    if selected == 0:
        return torch.empty(0, device=device, dtype=torch.int64)
    if selected == 1:
        return torch.zeros(1, device=device, dtype=torch.int64)
    num = torch.arange(selected, device=device, dtype=torch.int64) * (rows - 1)
    return torch.div(num, selected - 1, rounding_mode="floor")


# ---------------------------------------------------------------------------
# GRAIN response factors.

def _rational_terms(unit, num, den):
    """f and f' of P5/Q4 with |b| denominator; num/den broadcast against unit."""
    u2 = unit.square()
    u3 = u2 * unit
    u4 = u2.square()
    u5 = u4 * unit
    au = unit.abs()
    n = [num[..., j] for j in range(6)]
    d = [den[..., j] for j in range(4)]
    p = n[0] + n[1] * unit + n[2] * u2 + n[3] * u3 + n[4] * u4 + n[5] * u5
    dp = n[1] + 2.0 * n[2] * unit + 3.0 * n[3] * u2 + 4.0 * n[4] * u3 + 5.0 * n[5] * u4
    q = 1.0 + d[0] * au + d[1] * u2 + d[2] * au * u2 + d[3] * u4
    dq = d[0] * torch.sign(unit) + 2.0 * d[1] * unit + 3.0 * d[2] * unit * au + 4.0 * d[3] * u3
    f = p / q
    df = (dp * q - p * dq) / q.square()
    return f, df


def stacked_factors(preactivation, numerator, denominator, *, groups, width, eps):
    """unit, derivative, radial = f - u f' for ``[L, P, H]`` preactivations."""
    layers = preactivation.shape[0]
    v = preactivation.float().view(layers, -1, int(groups), int(width))
    rms = torch.sqrt(v.square().mean(dim=-1, keepdim=True) + float(eps))
    unit = v / rms
    num = numerator.detach().float()[:, None, :, None, :]
    den = denominator.detach().float().abs()[:, None, :, None, :]
    f, df = _rational_terms(unit, num, den)
    return unit, df, f - unit * df


def evaluate_response(unit, numerator, denominator):
    """f, f' for arbitrary (e.g. frozen) coefficients on stacked ``[L,P,G,w]`` units."""
    num = numerator.float()[:, None, :, None, :]
    den = denominator.float().abs()[:, None, :, None, :]
    return _rational_terms(unit, num, den)


def response_adjoint(cotangents, outgoing_weight, factors, *, groups, width):
    """Pull residual cotangents through out_proj and the GRAIN Jacobian."""
    unit, derivative, radial = factors
    shape = (cotangents.shape[0], cotangents.shape[1], int(groups), int(width))
    pulled = torch.bmm(cotangents.float(), outgoing_weight.float()).view(shape)
    return derivative * pulled + unit * (radial * pulled).mean(dim=-1, keepdim=True)


def jacobian_kernel_inner(unit, fa, da, fb, db):
    """<J_a J_a^T, J_b J_b^T>_F for J = diag(f') + (f - u f') u^T / w, in O(w)."""
    w = float(unit.shape[-1])
    ra = (fa - unit * da) / w
    rb = (fb - unit * db) / w
    pa = da * unit
    pb = db * unit
    sa = da.square()
    sb = db.square()
    e = unit.square().sum(dim=-1)
    diag = (sa * sb).sum(-1)
    diag = diag + 2.0 * (sa * pb * rb).sum(-1)
    diag = diag + e * (sa * rb.square()).sum(-1)
    diag = diag + 2.0 * (sb * pa * ra).sum(-1)
    diag = diag + e * (sb * ra.square()).sum(-1)
    g00 = (pa * pb).sum(-1)
    g01 = (pa * rb).sum(-1)
    g10 = (ra * pb).sum(-1)
    g11 = (ra * rb).sum(-1)
    # sum_ij (C G C)_ij G_ij with C = [[0, 1], [1, e]].
    rank_two = (2.0 * g00 * g11 + 2.0 * g01 * g10 + 2.0 * e * g01 * g11 + 2.0 * e * g10 * g11
                + e * e * g11 * g11)
    return diag + rank_two


def intrinsic_and_response_statistics(preactivation, cotangents, adjoint, factors,
                                      frozen_numerator, frozen_denominator, *, eps):
    """[L,G,4] participation sums and [L,G,2,3] live/frozen response sums."""
    unit, derivative, radial = factors
    w = float(unit.shape[-1])
    f = radial + unit * derivative
    rj = radial / w
    trace = derivative.square().sum(-1)
    trace = trace + 2.0 * (derivative * unit * rj).sum(-1)
    trace = trace + unit.square().sum(-1) * rj.square().sum(-1)
    live_live = jacobian_kernel_inner(unit, f, derivative, f, derivative)
    tiny = torch.finfo(trace.dtype).tiny
    incoming = (trace.square() / (w * live_live.clamp_min(tiny))).clamp(0.0, 1.0)
    energy = f.square().sum(-1)
    fourth = f.pow(4).sum(-1)
    outgoing = (energy.square() / (w * fourth.clamp_min(tiny))).clamp(0.0, 1.0)
    in_w = adjoint.square().mean(-1)
    out_w = cotangents.float().square().mean(-1)[..., None]
    participation = torch.stack(((incoming * in_w).sum(1), in_w.sum(1),
                                 (outgoing * out_w).sum(1), out_w.expand_as(outgoing).sum(1)), dim=-1)
    ff, fd = evaluate_response(unit, frozen_numerator, frozen_denominator)
    in_cross = (jacobian_kernel_inner(unit, f, derivative, ff, fd) * in_w).sum(1)
    in_live = (live_live * in_w).sum(1)
    in_frozen = (jacobian_kernel_inner(unit, ff, fd, ff, fd) * in_w).sum(1)
    v = preactivation.float().view_as(unit)
    rms = torch.sqrt(v.square().mean(-1, keepdim=True) + float(eps))
    live_h = rms * f
    frozen_h = rms * ff
    out_cross = ((live_h * frozen_h).sum(-1).square() * out_w).sum(1)
    out_live = (live_h.square().sum(-1).square() * out_w).sum(1)
    out_frozen = (frozen_h.square().sum(-1).square() * out_w).sum(1)
    response = torch.stack((torch.stack((in_cross, in_live, in_frozen), -1),
                            torch.stack((out_cross, out_live, out_frozen), -1)), dim=-2)
    return participation, response


def group_participation(stats):
    tiny = torch.finfo(stats.dtype).tiny
    inc = stats[..., 0] / stats[..., 1].clamp_min(tiny)
    out = stats[..., 2] / stats[..., 3].clamp_min(tiny)
    valid = torch.isfinite(stats).all(-1) & (stats[..., 1] > 0.0) & (stats[..., 3] > 0.0)
    value = torch.stack((inc, out), -1).clamp(0.0, 1.0)
    return torch.where(valid[..., None], value, torch.ones_like(value))


def group_congruence(stats, exact):
    denom = torch.sqrt(stats[..., 1] * stats[..., 2])
    valid = torch.isfinite(stats).all(dim=(-2, -1)) & (denom > 0.0).all(dim=-1)
    result = (stats[..., 0] / denom.clamp_min(torch.finfo(stats.dtype).tiny)).clamp(0.0, 1.0)
    result = torch.where(exact[..., None], torch.ones_like(result), result)
    return torch.where(valid[..., None], result, torch.ones_like(result))


def layer_congruence(stats, exact):
    layer = stats.sum(dim=1)
    denom = torch.sqrt(layer[..., 1] * layer[..., 2])
    valid = torch.isfinite(layer).all(dim=(-2, -1)) & (denom > 0.0).all(dim=-1)
    role = (layer[..., 0] / denom.clamp_min(torch.finfo(layer.dtype).tiny)).clamp(0.0, 1.0)
    result = torch.sqrt((role[:, 0] * role[:, 1]).clamp_min(0.0))
    result = torch.where(exact.all(dim=-1), torch.ones_like(result), result)
    return torch.where(valid, result, torch.ones_like(result))


def group_scores(inputs, features, cotangents, incoming_direction, outgoing_direction_t, adjoint, *,
                 groups, width, validate=True):
    """First-order loss change of each probe under each group's direction: ``[P, G]``.

    ``incoming_direction`` is ``[H, d]``; ``outgoing_direction_t`` is the
    transposed out_proj direction ``[H, d]``; ``adjoint`` is ``[P, G, w]``.
    """
    shape = (inputs.shape[0], int(groups), int(width))
    perturbation = (inputs.float() @ incoming_direction.float().T).view(shape)
    incoming = (perturbation * adjoint).sum(-1)
    projection = (cotangents.float() @ outgoing_direction_t.float().T).view(shape)
    outgoing = (features.float().view(shape) * projection).sum(-1)
    score = incoming + outgoing
    if validate and not bool(torch.isfinite(score).all()):
        raise RuntimeError("TILLER loss score is nonfinite")
    return score


def group_scores_stacked(inputs, features, cotangents, incoming_direction, outgoing_direction_t, adjoint, *,
                         groups, width):
    """:func:`group_scores` for every layer at once: ``[L, P, G]`` from
    ``inputs`` / ``cotangents`` ``[L, P, d]``, ``features`` ``[L, P, H]``,
    directions ``[L, H, d]`` and ``adjoint`` ``[L, P, G, w]`` (a few batched
    launches instead of a few per layer)."""
    layers, probes = int(inputs.shape[0]), int(inputs.shape[1])
    shape = (layers, probes, int(groups), int(width))
    perturbation = torch.bmm(inputs.float(), incoming_direction.float().transpose(1, 2)).view(shape)
    projection = torch.bmm(cotangents.float(), outgoing_direction_t.float().transpose(1, 2)).view(shape)
    return (perturbation * adjoint.float()).sum(-1) + (features.float().view(shape) * projection).sum(-1)


# ---------------------------------------------------------------------------
# Direction: factorized adaptive-tangent chord.

def group_view(value, *, groups, width, axis):
    """``[L, r, c]`` -> grouped ``[L, G, w, other]`` plus the inverse map."""
    layers, rows, cols = map(int, value.shape)
    if axis == "rows":
        if width is None or rows != int(groups) * int(width):
            raise RuntimeError("row groups do not match the layer's matrix shapes")
        return value.float().view(layers, int(groups), int(width), cols), \
            (lambda sel: sel.reshape(layers, rows, cols))
    if axis == "columns":
        if width is None or cols != int(groups) * int(width):
            raise RuntimeError("column groups do not match the layer's matrix shapes")
        grouped = value.float().transpose(-2, -1).contiguous().view(layers, int(groups), int(width), rows)
        return grouped, (lambda sel: sel.reshape(layers, cols, rows).transpose(-2, -1).contiguous())
    if axis == "matrix":
        if int(groups) != 1 or width is not None:
            raise RuntimeError("a whole-matrix view takes one group and no group width")
        return value.float()[:, None], (lambda sel: sel[:, 0])
    raise ValueError(f"unknown TILLER grouped axis: {axis}")


def grouped_shape(value, *, groups, width, axis):
    layers, rows, cols = map(int, value.shape)
    if axis == "rows":
        return layers, int(groups), int(width), cols
    if axis == "columns":
        return layers, int(groups), int(width), rows
    if axis == "matrix":
        return layers, 1, rows, cols
    raise ValueError(f"unknown TILLER grouped axis: {axis}")


_TINY32 = torch.finfo(torch.float32).tiny


def adaptive_tangent_chord(p, m, g, row_moment, col_moment, participation, congruence, step):
    """Chord toward the factorized-Adam tangent on grouped ``[L, G, w, c]`` blocks.

    Updates ``row_moment``/``col_moment`` in place (beta2 = 0.95, bias
    correction ``1 - 0.95**step``) and returns (selected, metadata).
    """
    sq = g.square()
    row_moment.mul_(0.95).add_(sq.sum(dim=-1), alpha=0.05)
    col_moment.mul_(0.95).add_(sq.sum(dim=-2), alpha=0.05)
    correction = 1.0 - MATCHED_BETA2 ** int(step)
    row_total = row_moment.sum(dim=-1, keepdim=True).clamp_min(_TINY32)
    variance = row_moment[..., :, None] * col_moment[..., None, :] / row_total[..., :, None]
    variance = variance / correction
    adaptive = m / (variance.sqrt() + LOCKED_EPS)
    dims = (-2, -1)
    p2 = p.square().sum(dims)
    a2 = adaptive.square().sum(dims)
    pa = (p * adaptive).sum(dims)
    gp = (g * p).sum(dims)
    ga = (g * adaptive).sum(dims)
    projection = pa / p2.clamp_min(_TINY32)
    tangent2 = (a2 - pa.square() / p2.clamp_min(_TINY32)).clamp_min(0.0)
    tangent_descent = ga - projection * gp
    orientation = torch.where(tangent_descent >= 0.0, torch.ones_like(tangent_descent),
                              -torch.ones_like(tangent_descent))
    info = participation.float().clamp(0.0, 1.0)
    align = congruence.float().clamp(0.0, 1.0)
    departure = (info * (1.0 - align.square()).clamp_min(0.0)).clamp(0.0, 1.0)
    parent_w = torch.sqrt((1.0 - departure).clamp_min(0.0))
    tangent_w = torch.sqrt(departure.clamp_min(0.0))
    ac = tangent_w * torch.sqrt(p2 / tangent2.clamp_min(_TINY32)) * orientation
    pc = parent_w - ac * projection
    cand = pc * gp + ac * ga
    finite = (torch.isfinite(p).all(dims) & torch.isfinite(m).all(dims) & torch.isfinite(g).all(dims)
              & torch.isfinite(adaptive).all(dims) & torch.isfinite(pc) & torch.isfinite(ac)
              & torch.isfinite(cand))
    active = finite & (p2 > 0.0) & (a2 > 0.0) & (tangent2 > _TINY32)
    safe = active & (gp > 0.0) & (cand > 0.0)
    pc = torch.where(safe, pc, torch.ones_like(pc))
    ac = torch.where(safe, ac, torch.zeros_like(ac))
    sel2 = (pc.square() * p2 + ac.square() * a2 + 2.0 * pc * ac * pa).clamp_min(0.0)
    sel_norm = torch.sqrt(sel2)
    p_norm = torch.sqrt(p2.clamp_min(0.0))
    cosine = ((pc * p2 + ac * pa) / (sel_norm * p_norm).clamp_min(LOCKED_EPS)).clamp(-1.0, 1.0)
    budget = (sel_norm - p_norm).abs() / p_norm.clamp_min(1.0)
    selected = p * pc[..., None, None] + adaptive * ac[..., None, None]
    meta = {"active": active, "safe": safe, "parent_cosine": cosine, "budget_residual": budget,
            "departure_energy": departure, "parent_descent": gp, "candidate_descent": cand,
            "parent_coefficient": pc, "adaptive_coefficient": ac, "tangent_orientation": orientation}
    return selected, meta


# ---------------------------------------------------------------------------
# Loss ledger (Robust Frequent Directions on the score rows).

@dataclass(frozen=True)
class LedgerRows:
    selection_scores: torch.Tensor
    selection_diagonal_residual: torch.Tensor
    persistent_scores: torch.Tensor
    persistent_total_diagonal: torch.Tensor
    persistent_diagonal_residual: torch.Tensor
    persistent_decay_cross: torch.Tensor
    history_used: bool
    discarded_energy_fraction: torch.Tensor
    selection_isotropic_tail: torch.Tensor
    persistent_isotropic_tail: torch.Tensor
    fd_shrinkage: torch.Tensor


def functional_row_norm(scores, *, validate=True):
    if scores.ndim != 2 or scores.shape[0] != CURRENT_ROWS or scores.shape[1] < 2:
        raise RuntimeError("functional score rows have the wrong shape for this ledger")
    if validate and not bool(torch.isfinite(scores).all()):
        raise RuntimeError("functional score rows contain non-finite values")
    return torch.sqrt(scores.double().square().sum() / float(CURRENT_ROWS)).to(scores.dtype)


def trace_matched_surrogate(exact_by_role, decay_derivative, reference_row_norm):
    """32 identical rows of the exact gradient score, rescaled to the last functional RMS."""
    gradient_score = exact_by_role.double().sum(dim=0)
    norm = torch.linalg.vector_norm(gradient_score)
    reference = reference_row_norm.double().reshape(())
    tiny = torch.finfo(torch.float64).tiny
    scale = torch.where(norm > tiny, reference / norm.clamp_min(tiny), torch.zeros_like(norm))
    score = (gradient_score * scale).to(exact_by_role.dtype)
    decay = (decay_derivative.double().reshape(()) * scale).to(exact_by_role.dtype)
    scores = score.unsqueeze(0).expand(CURRENT_ROWS, -1).clone()
    decay_action = decay.expand(CURRENT_ROWS).clone()
    return scores, decay_action, scale.to(exact_by_role.dtype)


def rfd_rows(current_scores, current_decay, previous_scores, previous_total_diagonal,
             previous_decay_cross, previous_tail, *, beta2=MATCHED_BETA2, eigh=None,
             validate=True):
    """Advance the matched-beta2 Robust-FD factor by one optimizer step."""
    if float(beta2) != MATCHED_BETA2:
        raise ValueError("the ledger's decay is fixed at beta2 = 0.95")
    if current_scores.ndim != 2 or current_scores.shape[0] != CURRENT_ROWS:
        raise RuntimeError("current ledger rows have the wrong shape")
    if validate and not bool(torch.isfinite(current_scores).all() & torch.isfinite(current_decay).all()):
        raise RuntimeError("current ledger rows contain non-finite values")
    dtype = current_scores.dtype
    s64 = current_scores.double()
    d64 = current_decay.double()
    current_cross = s64.T @ d64 / float(CURRENT_ROWS)
    zero = s64.new_zeros(())
    if previous_scores is None:
        if previous_tail is not None:
            raise RuntimeError("ledger tail mass present without any persistent rows")
        represented = s64.square().sum(0) / float(CURRENT_ROWS)
        tail = torch.zeros_like(represented)
        z = zero.to(dtype)
        return LedgerRows(current_scores, tail.to(dtype), s64.to(dtype), represented.to(dtype),
                          tail.to(dtype), current_cross.to(dtype), False, z, z, z, z)
    if previous_tail is None:
        raise RuntimeError("persistent ledger rows given without their tail mass")
    if validate:
        ok = (torch.isfinite(previous_scores).all() & torch.isfinite(previous_total_diagonal).all()
              & torch.isfinite(previous_decay_cross).all() & (previous_total_diagonal >= 0.0).all()
              & torch.isfinite(previous_tail).all() & (previous_tail >= 0.0).all())
        if not bool(ok):
            raise RuntimeError("persistent ledger state has non-finite or negative entries")
    beta = float(beta2)
    prev_tail = previous_tail.double().reshape(())
    selection = torch.cat((previous_scores * math.sqrt(beta), current_scores * math.sqrt(1.0 - beta)))
    if selection.shape[0] > MAXIMUM_SELECTION_ROWS:
        raise RuntimeError("more live ledger rows than the ledger keeps")
    selection_tail = prev_tail * beta
    decay_cross = previous_decay_cross.double() * beta + current_cross * (1.0 - beta)
    sel64 = selection.double()
    gram = sel64 @ sel64.T
    gram = 0.5 * (gram + gram.T)
    evals, evecs = (eigh or torch.linalg.eigh)(gram)
    evals = evals.clamp_min(0.0)
    physical = int(evals.numel())
    retained = min(PERSISTENT_ROWS, physical)
    discarded = physical - retained
    shrink = evals[discarded - 1] if discarded else zero
    kept = evals[-retained:]
    transform = evecs[:, -retained:].T
    unshrunk = transform @ sel64
    mult = torch.sqrt((kept - shrink).clamp_min(0.0) / kept.clamp_min(torch.finfo(torch.float64).tiny))
    persistent = mult[:, None] * unshrunk
    persistent_tail = selection_tail + shrink / (2.0 * float(CURRENT_ROWS))
    represented = persistent.square().sum(0) / float(CURRENT_ROWS)
    total_diag = represented + persistent_tail
    sel_tail_vec = torch.ones_like(represented) * selection_tail
    per_tail_vec = torch.ones_like(represented) * persistent_tail
    discarded_energy = evals[:discarded].sum() if discarded else zero
    fraction = discarded_energy / evals.sum().clamp_min(torch.finfo(torch.float64).tiny)
    return LedgerRows(selection, sel_tail_vec.to(dtype), persistent.to(dtype), total_diag.to(dtype),
                      per_tail_vec.to(dtype), decay_cross.to(dtype), True, fraction.to(dtype),
                      selection_tail.to(dtype), persistent_tail.to(dtype), shrink.to(dtype))


@dataclass(frozen=True)
class WindowRows:
    selection_scores: torch.Tensor
    selection_decay_action: torch.Tensor
    updated_scores: torch.Tensor
    updated_decay_action: torch.Tensor
    history_used: bool
    relative_innovation: torch.Tensor


def window32_rows(current_scores, current_decay, previous_scores, previous_decay, *, validate=True):
    """Latest 32 functional rows, no temporal mixing; Gram innovation diagnostic."""
    if validate and not bool(torch.isfinite(current_scores).all() & torch.isfinite(current_decay).all()):
        raise RuntimeError("response window rows contain non-finite values")
    if (previous_scores is None) != (previous_decay is None):
        raise RuntimeError("response window score and decay histories must both be present or both absent")
    updated = current_scores.detach().clone()
    updated_decay = current_decay.detach().clone()
    if previous_scores is None:
        return WindowRows(updated, updated_decay, updated, updated_decay, False,
                          current_scores.new_zeros(()))
    cg = current_scores @ current_scores.T
    pg = previous_scores @ previous_scores.T
    xg = current_scores @ previous_scores.T
    tiny = torch.finfo(current_scores.dtype).tiny
    innov = torch.sqrt((cg.square().sum() + pg.square().sum() - 2.0 * xg.square().sum()).clamp_min(0.0)
                       / cg.square().sum().clamp_min(tiny))
    return WindowRows(updated, updated_decay, updated, updated_decay, True, innov)


# ---------------------------------------------------------------------------
# Diagonal-completed biatlas transaction.

@dataclass(frozen=True)
class TransactionResult:
    coefficients: torch.Tensor
    candidate_coefficients: torch.Tensor
    accepted: torch.Tensor
    multiplier: torch.Tensor
    hard_case: torch.Tensor
    budget_residual: torch.Tensor
    parent_score: torch.Tensor
    candidate_score: torch.Tensor
    factor_rank: torch.Tensor
    diagonal_minimum: torch.Tensor
    diagonal_median: torch.Tensor
    diagonal_maximum: torch.Tensor
    cross_layer_coupling_ratio: torch.Tensor


def lanczos_basis(low_rank, diagonal, rhs, steps=KRYLOV_ROWS):
    """Fully re-orthogonalised Lanczos on ``M = diag(D) + L^T L`` from ``rhs``.

    Returns the orthonormal basis Q [C, k] and the symmetric tridiagonal T [k, k].
    Breakdown directions are replaced by orthogonalised cos(i * j) vectors.
    """
    n = int(rhs.numel())
    steps = min(int(steps), n)
    tiny = torch.finfo(rhs.dtype).tiny
    eps = torch.finfo(rhs.dtype).eps
    norm = torch.linalg.vector_norm(rhs)
    basis = torch.zeros(n, steps, dtype=rhs.dtype, device=rhs.device)
    alphas = []
    betas = []
    cur = rhs / norm.clamp_min(tiny)
    prev = torch.zeros_like(cur)
    prev_beta = rhs.new_zeros(())
    coord = torch.arange(n, device=rhs.device, dtype=rhs.dtype) + 1.0
    for i in range(steps):
        basis[:, i] = cur
        active = basis[:, : i + 1]
        action = diagonal * cur + low_rank.T @ (low_rank @ cur)
        alpha = torch.dot(cur, action)
        resid = action - alpha * cur - prev_beta * prev
        for _ in range(2):
            resid = resid - active @ (active.T @ resid)
        beta = torch.linalg.vector_norm(resid)
        alphas.append(alpha)
        if i + 1 < steps:
            threshold = 64.0 * eps * torch.linalg.vector_norm(action).clamp_min(1.0)
            fallback = torch.cos(coord * float(i + 1))
            for _ in range(2):
                fallback = fallback - active @ (active.T @ fallback)
            fnorm = torch.linalg.vector_norm(fallback)
            usable = fnorm > threshold
            fallback = fallback / fnorm.clamp_min(tiny)
            nxt = resid / beta.clamp_min(tiny)
            broke = beta <= threshold
            nxt = torch.where(usable & broke, fallback, nxt)
            beta = torch.where(broke, beta.new_zeros(()), beta)
            betas.append(beta)
            prev = cur
            cur = nxt
            prev_beta = beta
    tri = torch.diag(torch.stack(alphas))
    if steps > 1:
        off = torch.stack(betas)
        tri = tri + torch.diag(off, 1) + torch.diag(off, -1)
    tri = 0.5 * (tri + tri.T)
    return basis, tri


def biatlas_transaction(rows: LedgerRows, exact_by_role, momentum_by_role, weights, layer_ids, *,
                        total_layers, eta, rounds=64, diagnostics=True, validate=True, eigh=None,
                        measure_rows=CURRENT_ROWS):
    """Equal-budget signed coefficients in the diagonal + row-space metric.

    Minimises the quadratic loss model ``-eta <g, c> + eta^2/2 c^T M c + ...``
    over coefficients ``c`` with ``sum w c^2 = sum w`` (the parent budget),
    via a 32-dimensional Krylov space and a 64-round bisection on the secular
    equation; accepts the candidate only if it is finite, not the hard case,
    improves the model, meets the budget to 1e-8 and keeps every layer/role
    contraction positive.  Otherwise every coefficient is 1 (the parent).
    """
    scores = rows.selection_scores
    diag_res = rows.selection_diagonal_residual
    decay_cross = rows.persistent_decay_cross
    factor_rows, coords = scores.shape
    if factor_rows < measure_rows or factor_rows > MAXIMUM_SELECTION_ROWS or coords < 2:
        raise RuntimeError("transaction needs between the measured and the maximum row count and two or more coordinates")
    if validate:
        ok = torch.isfinite(scores).all()
        for v in (diag_res, decay_cross, exact_by_role, momentum_by_role, weights):
            ok = ok & torch.isfinite(v).all()
        ok = ok & (diag_res >= 0.0).all() & (weights > 0.0).all()
        if not bool(ok):
            raise RuntimeError("transaction inputs must be finite, with residuals >= 0 and weights > 0")
        if not bool(((layer_ids >= 0) & (layer_ids < int(total_layers))).all()):
            raise RuntimeError("transaction layer ids must lie in [0, layers)")
    s64 = scores.double()
    diag64 = diag_res.double()
    decay64 = decay_cross.double()
    exact64 = exact_by_role.double()
    mom64 = momentum_by_role.double()
    w64 = weights.double()
    root_w = torch.sqrt(w64)
    inv_root_w = torch.reciprocal(root_w)
    low_rank = s64 * inv_root_w.unsqueeze(0) / math.sqrt(measure_rows)
    if factor_rows < MAXIMUM_SELECTION_ROWS:
        low_rank = torch.cat((low_rank, low_rank.new_zeros(MAXIMUM_SELECTION_ROWS - factor_rows, coords)))
    diag_white = diag64 / w64
    rhs = (exact64.sum(0) / float(eta) - decay64) * inv_root_w
    budget = w64.sum()
    tiny = torch.finfo(torch.float64).tiny
    machine = torch.finfo(torch.float64).eps
    basis, tri = lanczos_basis(low_rank, diag_white, rhs)
    evals, evecs = (eigh or torch.linalg.eigh)(tri)
    evals = evals.clamp_min(0.0)
    proj = evecs.T @ (basis.T @ rhs)
    lower = torch.tensor(machine * float(coords), device=scores.device, dtype=torch.float64)
    upper = torch.linalg.vector_norm(rhs) / torch.sqrt(budget) + evals.amax() + lower
    hard = (proj / (evals + lower)).square().sum() < budget
    lo, hi = lower, upper
    for _ in range(int(rounds)):
        mid = 0.5 * (lo + hi)
        too_large = (proj / (evals + mid)).square().sum() > budget
        lo = torch.where(too_large, mid, lo)
        hi = torch.where(too_large, hi, mid)
    cand_y = basis @ (evecs @ (proj / (evals + hi)))
    cand64 = cand_y * inv_root_w
    cand_budget = (w64 * cand64.square()).sum()
    budget_res = (cand_budget - budget).abs() / budget.clamp_min(1.0)
    ones = torch.ones_like(cand64)
    parent_action = s64 @ ones
    cand_action = s64 @ cand64
    parent_exact = exact64.sum()
    cand_exact = (exact64.sum(0) * cand64).sum()
    e = float(eta)
    parent_score = -e * parent_exact + 0.5 * e * e * (
        parent_action.square().sum() / float(measure_rows) + (diag64 * ones.square()).sum()
        + 2.0 * decay64.sum())
    cand_score = -e * cand_exact + 0.5 * e * e * (
        cand_action.square().sum() / float(measure_rows) + (diag64 * cand64.square()).sum()
        + 2.0 * (decay64 * cand64).sum())
    L = int(total_layers)
    zeros = torch.zeros((2, L), device=scores.device, dtype=torch.float64)
    pe = zeros.clone().index_add_(1, layer_ids, exact64)
    pm = zeros.clone().index_add_(1, layer_ids, mom64)
    ce = zeros.clone().index_add_(1, layer_ids, exact64 * cand64.unsqueeze(0))
    cm = zeros.clone().index_add_(1, layer_ids, mom64 * cand64.unsqueeze(0))
    finite = torch.isfinite(cand64).all() & torch.isfinite(cand_score) & torch.isfinite(budget_res)
    accepted = (finite & ~hard & (cand_score < parent_score) & (budget_res <= 1e-8)
                & (ce > 0.0).all() & (cm > 0.0).all() & (pe > 0.0).all() & (pm > 0.0).all()).reshape(1)
    cand = cand64.to(scores.dtype)
    selected = torch.where(accepted, cand, torch.ones_like(cand))
    if diagnostics:
        sv = torch.linalg.svdvals(low_rank)
        rank = (sv > machine * float(coords) * sv.amax().clamp_min(tiny)).sum().reshape(1)
        meas = float(measure_rows)
        total_sq = ((s64 @ s64.T).square().sum() / (meas * meas)
                    + 2.0 * (diag64 * s64.square().sum(0) / meas).sum() + diag64.square().sum())
        within = torch.zeros_like(total_sq)
        for layer in range(L):
            mask = layer_ids.eq(layer)
            lf = s64[:, mask]
            ld = diag64[mask]
            within = within + ((lf @ lf.T).square().sum() / (meas * meas)
                               + 2.0 * (ld * lf.square().sum(0) / meas).sum() + ld.square().sum())
        coupling = torch.sqrt((total_sq - within).clamp_min(0.0) / total_sq.clamp_min(tiny)).reshape(1)
        dmin, dmed, dmax = diag64.amin().reshape(1), diag64.median().reshape(1), diag64.amax().reshape(1)
    else:
        rank = torch.zeros((1,), device=scores.device, dtype=torch.int64)
        z = s64.new_zeros((1,))
        dmin = dmed = dmax = coupling = z
    return TransactionResult(selected, cand, accepted,
                             torch.where(hard, torch.zeros_like(hi), hi).reshape(1), hard.reshape(1),
                             budget_res.reshape(1), parent_score.reshape(1), cand_score.reshape(1),
                             rank, dmin, dmed, dmax, coupling)


# ---------------------------------------------------------------------------
# Closed-form accounting (state / communication inventory).

def tiller_scaling_formula(*, total_positions: int, total_layers: int, total_groups: int,
                           intermediate_width: int, model_width: int) -> dict:
    values = tuple(map(int, (total_positions, total_layers, total_groups, intermediate_width,
                             model_width)))
    if min(values) <= 0 or int(intermediate_width) % int(total_groups):
        raise ValueError("TILLER scaling dimensions are invalid")
    positions, layers, groups, hidden, model = values
    coords = layers * groups
    rows = CURRENT_ROWS
    # window-32 cadence-8 parent inventory (core.py:3912-3924)
    parent_state = 10 * coords + 2
    factor_state = rows * (coords + 1)
    route_state = 4 * coords + 2 * layers
    response_summary = 21 * coords + 10 * layers
    transaction_summary = rows * rows + 3 * rows + 8 * layers + 8
    refresh_score_summary = rows * (coords + 1)
    result = {
        "total_positions": positions,
        "persistent_state_elements": parent_state + factor_state + route_state,
        "window_factor_elements": factor_state,
        "cached_response_route_elements": route_state,
        "communicated_summary_elements": response_summary + refresh_score_summary
        + transaction_summary + 2 * coords,
        "ordinary_communicated_summary_elements": transaction_summary + 2 * coords,
        "largest_temporal_dense_dimension": rows,
        "largest_dense_solve_dimension": rows,
        "dense_coordinate_metric_elements": 0,
        "owner_count": 0,
        "selected_update_elements_published": 0,
        "response_refresh_interval": REFRESH_INTERVAL,
        "matched_beta2": MATCHED_BETA2,
        "local_direction_arithmetic_elements": 4 * layers * hidden * model,
    }
    # factorized chord (core.py:4065-4077)
    factor = 2 * layers * (hidden + groups * model) + 6 * layers * model
    direction_summary = 3 * factor + 5 * layers * (groups + 1)
    result.update({
        "factorized_row_column_state_elements": factor,
        "persistent_state_elements": result["persistent_state_elements"] + factor,
        "arbitrary_shard_direction_summary_elements": direction_summary,
        "communicated_summary_elements": result["communicated_summary_elements"] + direction_summary,
        "ordinary_communicated_summary_elements": result["ordinary_communicated_summary_elements"]
        + direction_summary,
        "additional_persistent_state_elements": factor,
        "state_depends_on_total_activation_positions": 0,
        "state_scales_linearly_with_width": 1,
        "additional_native_polar_maps_per_role": 0,
        "dense_tangent_projector_elements": 0,
        "additional_dense_solve_dimension": 0,
        "compiled_static_fullgraph": 1,
        "scientific_equation_changed_vs_parent": 0,
        "state_recurrence_changed_vs_parent": 0,
        "additional_persistent_state_elements_vs_parent": 0,
    })
    # ledger (core.py:4370-4379)
    ledger = PERSISTENT_ROWS * coords + 2 * coords + 4
    result.update({
        "family_id": "tiller_v1",
        "coordinate_count": coords,
        "ledger_checkpoint_tensor_elements": ledger,
        "additional_persistent_state_elements": ledger,
        "persistent_state_elements": result["persistent_state_elements"] + ledger,
        "maximum_live_factor_elements": MAXIMUM_SELECTION_ROWS * coords,
        "every_step_gradient_score_ledger": 1,
        "trace_matched_gradient_surrogate": 1,
        "functional_score_refresh_interval": REFRESH_INTERVAL,
        "matched_beta2_every_optimizer_step": 1,
        "robust_fd_midpoint_tail": 1,
        "factorized_parameter_direction_unchanged": 1,
        "adaptive_rank64_cross_coordinate_factor": 1,
        "largest_dense_solve_dimension": MAXIMUM_SELECTION_ROWS,
        "largest_transaction_dense_dimension": 32,
        "largest_temporal_dense_dimension": MAXIMUM_SELECTION_ROWS,
        "state_depends_on_total_activation_positions": 0,
        "owner_count": 0,
        "complete_layer_owners": 0,
        "complete_coordinate_owners": 0,
        "owner_local_mathematics": 0,
        "dense_lg_by_lg_metric_elements": 0,
        "selected_update_elements_published": 0,
        "new_tunable_hyperparameters": 0,
        "state_scales_as": "O(LH + LGd + 64LG)",
    })
    return result
