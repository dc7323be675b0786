"""TILLER: Tangents Informed by a Loss Ledger for Equal-budget Reweighting.

Public API of optimizer_design/tiller.py (``TILLERRouter``,
``TILLERAttentionOptimizer``, ``configure_microbatch_count``,
``tiller_scaling_formula``, ``FAMILY_ID``, ``PREFIX``).  The reference builds
the live algorithm from a 20-class lineage with runtime patching
(optimizer_design/_tiller/core.py:3362-3392, 4120-4150, 4310-4317,
4481-4537); here it is written out once:

Router (GRAIN in_proj / out_proj matrices), every step::

    m      = Nesterov(grad)                         (mu = 0.95, per matrix)
    p      = NS5 per GRAIN group block, rescaled    (rational_group_zero_power)
    q      = factorized adaptive-tangent chord(p, m, g; participation, congruence)
    exact  = <g, adj*q>,  momentum = <m, adj*q>,  weight = ||adj*q||^2 per (layer, group)
    c      = biatlas transaction(ledger rows, exact, momentum, weight)
    W     <- (1 - lr wd) W - lr adj c q

On refresh steps (transitions 0, 8, 16, ... = optimizer steps 1, 9, 17, ...)
the probe packets captured by the module hooks give the response sensor
(participation/congruence, all-reduced), 32 functional loss rows (gathered),
and the ledger is advanced with them; on the other 7 steps the cached route
is reused and the ledger advances with the trace-matched gradient surrogate.
The attention optimizer consumes the router's layer participation and
congruence and applies the same chord to head-group NS5 directions.

State keys, state placement (everything on ``state[in_weight of layer 0]``
except the per-matrix ``momentum_buffer``), parameter-group contents and
parameter order are those of the reference so ``state_dict`` round-trips.
"""
from __future__ import annotations

import contextlib
import math
import os

import torch
import torch.distributed as dist
from torch.autograd.graph import increment_version

from ..parallel import param_ready

from . import tiller_math as tm
from .newton_schulz import (attention_head_group_zero_power, match_rms_adamw_adjustment,
                            rational_group_zero_power)

FAMILY_ID = "tiller_v1"
PREFIX = "tiller_"
MATCHED_BETA2 = tm.MATCHED_BETA2

# Number of gradient-accumulation micro-batches whose probe rows are captured
# per optimizer step (configure_microbatch_count).
_EXPECTED_MICROBATCHES = 4

# Parameter-group contents written by the reference lineage (they appear in
# checkpoints, so they are reproduced verbatim).
_ROUTER_GROUP_KEYS = {
    "ten_probe_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "muon_momentum": 0.95,
    "muon_ns_steps": 5,
    "muon_adjust_lr_fn": "match_rms_adamw",
    "fixed32_transaction_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "response_fisher_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "residual_fisher_attention_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "loss_weighted_intrinsic_sign_attention_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "loss_weighted_four_role_sign_transport_family_id": "loss_weighted_four_role_response_homotopy_muon_v1",
    "loss_weighted_four_role_response_homotopy_family_id": "loss_weighted_four_role_response_homotopy_muon_v1",
    "loss_weighted_four_role_response_homotopy_batched_family_id": "loss_weighted_four_role_response_homotopy_batched_muon_v2",
    "loss_weighted_four_role_response_homotopy_compact_family_id": "loss_weighted_four_role_response_homotopy_compact_muon_v3",
    "global_response_transaction_family_id": "global_response_transaction_muon_v1",
    "lagged_predictive_response_transaction_family_id": "lagged_predictive_response_transaction_muon_v1",
    "temporal_response_group_polar_family_id": "temporal_response_group_polar_muon_v1",
    "posterior_rank64_response_group_polar_family_id": "posterior_rank64_response_group_polar_muon_v1",
    "tiller_family_id": FAMILY_ID,
    "tiller_refresh_interval": tm.REFRESH_INTERVAL,
}
_ATTENTION_GROUP_KEYS = {
    "residual_fisher_attention_family_id": "residual_fisher_attention_muon_v1",
    "loss_weighted_intrinsic_sign_attention_family_id": "loss_weighted_intrinsic_sign_attention_muon_v1",
    "loss_weighted_four_role_sign_transport_family_id": "loss_weighted_four_role_sign_transport_muon_v1",
    "loss_weighted_four_role_response_homotopy_family_id": "loss_weighted_four_role_response_homotopy_muon_v1",
    "loss_weighted_four_role_response_homotopy_batched_family_id": "loss_weighted_four_role_response_homotopy_batched_muon_v2",
    "loss_weighted_four_role_response_homotopy_compact_family_id": "loss_weighted_four_role_response_homotopy_compact_muon_v3",
    "global_response_transaction_family_id": "global_response_transaction_muon_v1",
    "lagged_predictive_response_transaction_family_id": "lagged_predictive_response_transaction_muon_v1",
    "temporal_response_group_polar_family_id": "temporal_response_group_polar_muon_v1",
    "posterior_rank64_response_group_polar_family_id": "posterior_rank64_response_group_polar_muon_v1",
    "tiller_family_id": FAMILY_ID,
}
_ROUTE_NAMES = ("group_participation", "group_congruence", "intrinsic_participation",
                "attention_congruence")


def configure_microbatch_count(count: int) -> None:
    """Set the gradient-accumulation micro-batch count before building a router."""
    global _EXPECTED_MICROBATCHES
    if isinstance(count, bool) or not isinstance(count, int) or count < 1:
        raise ValueError("TILLER microbatch count must be a positive integer")
    _EXPECTED_MICROBATCHES = count


def microbatch_count() -> int:
    return _EXPECTED_MICROBATCHES


def tiller_scaling_formula(**kwargs):
    return tm.tiller_scaling_formula(**kwargs)


def _dist_shape(group):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group=group), dist.get_world_size(group=group)
    return 0, 1


def foreach_nesterov(optimizer, parameters, momentum):
    """``buf.lerp_(g, 1-mu)``; return stacked fp32 ``g.lerp(buf, mu)``."""
    grads, bufs = [], []
    for p in parameters:
        if p.grad is None:
            raise RuntimeError("a TILLER-managed matrix has no gradient this step")
        grads.append(p.grad)
        st = optimizer.state[p]
        buf = st.get("momentum_buffer")
        if buf is None:
            buf = torch.zeros_like(p.grad, memory_format=torch.preserve_format)
            st["momentum_buffer"] = buf
        bufs.append(buf)
    torch._foreach_lerp_(bufs, grads, 1.0 - momentum)
    return torch.stack(torch._foreach_lerp(grads, bufs, momentum)).float()


def foreach_apply(parameters, direction, *, decay, alpha):
    torch._foreach_mul_(parameters, float(decay))
    torch._foreach_add_(parameters, list(direction.to(parameters[0].dtype).unbind(0)),
                        alpha=float(alpha))


def shard_bounds(layers: int, rank: int, world: int):
    """Contiguous, balanced block of layers owned by ``rank`` (may be empty)."""
    return rank * layers // world, (rank + 1) * layers // world


def layer_owner(layer: int, layers: int, world: int) -> int:
    for r in range(world):
        lo, hi = shard_bounds(layers, r, world)
        if lo <= layer < hi:
            return r
    raise ValueError(layer)


def sharding_enabled(world: int) -> bool:
    """Layer-sharded optimizer steps across data-parallel ranks (RO_TILLER_SHARD=0 disables)."""
    return world > 1 and os.environ.get("RO_TILLER_SHARD", "1") != "0"


class OwnerPacking:
    """Layer-sharded weights re-homed into one fp32 buffer ordered by owner.

    ``per_layer[l]`` lists the matrices of layer ``l`` (TILLER: [in_proj,
    out_proj, qkv, attention out]); layer ``l`` is updated on rank
    ``layer_owner(l)``, so the layers an owner updates form one contiguous
    range, replicated with one peer-memory pull (or one broadcast) per owner
    instead of one per tensor.
    """

    @classmethod
    def for_tiller(cls, router, attention):
        L = len(router.pairs)
        per_layer = [[router.pairs[l]["in_weight"], router.pairs[l]["out_weight"],
                      attention.role_parameters["qkv"][l], attention.role_parameters["attn_out"][l]]
                     for l in range(L)]
        return cls(per_layer, router.world_size, router.loss_probe_group)

    def __init__(self, per_layer, world, group=None):
        L = len(per_layer)
        device = per_layer[0][0].device
        total = sum(p.numel() for ps in per_layer for p in ps)
        self.world = int(world)
        self.group = group
        from ..parallel import owner_gather
        self.gather = None
        use_gather = (device.type == "cuda" and self.world > 1 and owner_gather.available()
                      and os.environ.get("RO_WEIGHT_TRANSPORT", "nccl") == "p2p")
        if use_gather:
            raw, self.flat = owner_gather.shared_buffer(total, device)
        else:
            self.flat = torch.empty(total, device=device, dtype=torch.float32)
        self.layer_ranges = []
        self.layer_params = per_layer
        off = 0
        with torch.no_grad():
            for ps in per_layer:
                lo = off
                for p in ps:
                    n = p.numel()
                    view = self.flat[off:off + n].view_as(p)
                    view.copy_(p.data)
                    p.data = view
                    off += n
                self.layer_ranges.append((lo, off))
        self.layers = L
        if use_gather:
            ranges, params = [], []
            for r in range(self.world):
                lo_l, hi_l = shard_bounds(L, r, self.world)
                if hi_l > lo_l:
                    ranges.append((self.layer_ranges[lo_l][0], self.layer_ranges[hi_l - 1][1]))
                else:
                    ranges.append((0, 0))
                params.append([p for l in range(lo_l, hi_l) for p in per_layer[l]])
            self.gather = owner_gather.OwnerGather(raw, self.flat, ranges, params, group=self.group)

    def broadcast(self):
        """Replicate every owner's updated layers: the peer-memory pull
        (:class:`~rational_optimizer_b200.parallel.owner_gather.OwnerGather`) or,
        without it, one deferred NCCL broadcast per owner."""
        if self.gather is not None:
            self.gather.publish()  # the copies are pulled by the next reader (lazily, or in the step graph)
            return
        side = param_ready.side_stream(self.flat.device)
        side.wait_stream(torch.cuda.current_stream(self.flat.device))
        for r in range(self.world):
            lo_l, hi_l = shard_bounds(self.layers, r, self.world)
            if hi_l <= lo_l:
                continue
            lo, hi = self.layer_ranges[lo_l][0], self.layer_ranges[hi_l - 1][1]
            src = dist.get_global_rank(self.group, r) if self.group is not None else r
            with torch.cuda.stream(side):
                dist.broadcast(self.flat[lo:hi], src=src, group=self.group)
                event = torch.cuda.Event()
                event.record(side)
            params = [p for l in range(lo_l, hi_l) for p in self.layer_params[l]]
            param_ready.defer(params, event)
            for p in params:
                increment_version(p)


def broadcast_owned(tensors_by_layer, layers, world, group=None, *, deferred=False):
    """Replicate per-layer tensors from their owners; bumps autograd versions.

    ``deferred``: enqueue the broadcasts on a side stream after the work
    issued so far and return at once; each layer's tensors are marked pending
    until their broadcast completes (``parallel.param_ready``), so the next
    forward overlaps the transfer of later layers.
    """
    flat = [t for tensors in tensors_by_layer for t in tensors]
    deferred = deferred and bool(flat) and flat[0].is_cuda
    if deferred:
        side = param_ready.side_stream(flat[0].device)
        side.wait_stream(torch.cuda.current_stream(flat[0].device))
    for layer, tensors in enumerate(tensors_by_layer):
        src = layer_owner(layer, layers, world)
        src_global = dist.get_global_rank(group, src) if group is not None else src
        if deferred:
            with torch.cuda.stream(side):
                for t in tensors:
                    dist.broadcast(t.data if isinstance(t, torch.nn.Parameter) else t, src=src_global,
                                   group=group)
                event = torch.cuda.Event()
                event.record(side)
            param_ready.defer(tensors, event)
        else:
            for t in tensors:
                dist.broadcast(t.data if isinstance(t, torch.nn.Parameter) else t, src=src_global,
                               group=group)
        for t in tensors:
            increment_version(t)


class TILLERRouter(torch.optim.Optimizer):
    """TILLER on the GRAIN ``in_proj``/``out_proj`` matrices of every layer.

    ``pairs`` is a sequence of dicts with keys ``mlp``, ``module`` (the GRAIN
    activation), ``in_weight``, ``out_weight``, ``numerator``,
    ``denominator``, ``groups``, ``hidden_dim`` and ``eps`` (the inventory of
    ``collect_rlb_optimizer_groups``, training/train.py:1614-1659).
    """

    family_id = FAMILY_ID
    telemetry_prefix = PREFIX

    def __init__(self, pairs, *, lr, weight_decay, momentum, ns_steps, beta2, eps,
                 loss_probe_group=None, strict_validation=None):
        self.pairs = list(pairs)
        if not self.pairs:
            raise ValueError("TILLER requires GRAIN layers")
        self.momentum = float(momentum)
        self.ns_steps = int(ns_steps)
        if self.momentum != 0.95 or self.ns_steps != 5:
            raise ValueError("TILLER requires matched momentum .95 and NS5")
        if float(beta2) != MATCHED_BETA2:
            raise ValueError("TILLER requires locked beta2=.95")
        if float(eps) != tm.LOCKED_EPS:
            raise ValueError("TILLER requires eps=1e-8")
        self.predictive_beta2 = float(beta2)
        self.loss_probe_group = loss_probe_group
        rank, world = _dist_shape(loss_probe_group)
        self.world_size = world
        self.microbatches = _EXPECTED_MICROBATCHES
        self.probe_layout = tm.fixed_global_probe_layout(tm.GLOBAL_PROBE_COUNT, rank, world)
        self.capture_rows = (self.probe_layout.local_probe_count + self.microbatches - 1) // self.microbatches
        first = self.pairs[0]
        self.groups = int(first["groups"])
        self.hidden = int(first["hidden_dim"])
        self.external = int(first["in_weight"].shape[1])
        self.grain_eps = float(first["eps"])
        if self.hidden % self.groups:
            raise ValueError("TILLER hidden width is not group divisible")
        self.width = self.hidden // self.groups
        self.strict = (strict_validation if strict_validation is not None
                       else not first["in_weight"].is_cuda)
        params, seen = [], set()
        for layer, pair in enumerate(self.pairs):
            inc, out = pair["in_weight"], pair["out_weight"]
            if (int(pair["groups"]) != self.groups or int(pair["hidden_dim"]) != self.hidden
                    or float(pair["eps"]) != self.grain_eps
                    or inc.shape != (self.hidden, self.external)
                    or out.shape != (self.external, self.hidden)
                    or pair["numerator"].shape != (self.groups, 6)
                    or pair["denominator"].shape != (self.groups, 4)):
                raise ValueError("TILLER GRAIN inventory changed")
            for p in (inc, out):
                if id(p) in seen:
                    raise ValueError("TILLER matrix ownership overlaps")
                seen.add(id(p))
                params.append(p)
        defaults = {"lr": float(lr), "weight_decay": float(weight_decay), "lr_scale": 1.0}
        defaults.update(_ROUTER_GROUP_KEYS)
        super().__init__([{"params": params}], defaults)
        # probe capture buffers
        self._pending_inputs = [None for _ in self.pairs]
        self._functional_records = [[] for _ in self.pairs]
        self._cotangent_records = [[] for _ in self.pairs]
        self._hook_handles = []
        for layer, pair in enumerate(self.pairs):
            self._hook_handles.extend((
                pair["mlp"].register_forward_pre_hook(self._make_input_hook(layer)),
                pair["module"].register_forward_hook(self._make_feature_hook(layer)),
                pair["mlp"].register_forward_hook(self._make_cotangent_hook(layer)),
            ))
        anchor = self.state[self.pairs[0]["in_weight"]]
        anchor.setdefault("four_role_response_frozen_numerators",
                          torch.stack([p["numerator"].detach().float().clone() for p in self.pairs]))
        anchor.setdefault("four_role_response_frozen_denominators",
                          torch.stack([p["denominator"].detach().float().clone() for p in self.pairs]))
        self._clip_factor = None
        self._capture_telemetry_next_step = False
        self._last_telemetry = {}
        # cadence
        self._cadence_transition = 0
        self._capture_response_this_transition = True
        self._cached_route = None
        self._cached_selection_scores = None
        self._cached_selection_decay = None
        # attention hand-off
        self._attention_update = 0
        self._attention_consumed = True
        self._group_participation = None
        self._group_response_congruence = None
        self._intrinsic_participation = None
        self._attention_response_congruence = None
        # ledger scratch
        self._rfd_rows = None
        self._rfd_decay_derivative = None
        self._rfd_gradient_scale = None
        self._rfd_functional_refresh = False
        self._rfd_selection = None
        self._last_predictive = None
        self._fused_ok = None
        self._fused_role_objs = None
        self.packing = None  # OwnerPacking when weights are re-homed for owner broadcasts
        self._force_torch = False
        self._ledger_bufs = None
        self._pending_apply = None
        self._packing_due = False
        self._side_stream = None

    # -- properties --------------------------------------------------------
    @property
    def anchor(self):
        return self.state[self.pairs[0]["in_weight"]]

    # -- probe hooks -------------------------------------------------------
    def _sample_indices(self, rows, device):
        return tm.evenly_spaced_indices(int(rows), self.capture_rows, device=device)

    def _make_input_hook(self, layer):
        @torch.no_grad()
        def capture(module, inputs):
            if not self._capture_response_this_transition or not module.training:
                return None
            if len(inputs) != 1 or not torch.is_tensor(inputs[0]):
                raise RuntimeError("TILLER MLP input hook changed")
            if self._pending_inputs[layer] is not None:
                raise RuntimeError("TILLER probe input remained pending")
            flat = inputs[0].detach().reshape(-1, self.external)
            idx = self._sample_indices(flat.shape[0], flat.device)
            self._pending_inputs[layer] = (int(flat.shape[0]), idx, flat.index_select(0, idx).clone())
            return None
        return capture

    def _make_feature_hook(self, layer):
        @torch.no_grad()
        def capture(module, inputs, output):
            if not self._capture_response_this_transition or not module.training:
                return None
            pending = self._pending_inputs[layer]
            if pending is None:
                raise RuntimeError("TILLER feature lacks aligned input")
            rows, idx, sampled = pending
            pre = inputs[0].detach().reshape(-1, self.hidden)
            feat = output.detach().reshape(-1, self.hidden)
            if pre.shape[0] != rows or feat.shape[0] != rows:
                raise RuntimeError("TILLER x/z/h rows differ")
            self._functional_records[layer].append(
                (sampled, pre.index_select(0, idx).clone(), feat.index_select(0, idx).clone()))
            self._pending_inputs[layer] = None
            return None
        return capture

    def _make_cotangent_hook(self, layer):
        def capture(module, _inputs, output):
            if not self._capture_response_this_transition or not module.training:
                return None
            if not torch.is_tensor(output) or not output.requires_grad:
                raise RuntimeError("TILLER MLP output hook changed")
            flat = output.reshape(-1, self.external)
            rows = int(flat.shape[0])
            idx = self._sample_indices(rows, flat.device)

            def capture_gradient(cotangent):
                with torch.no_grad():
                    value = cotangent.detach().reshape(-1, self.external)
                    if value.shape[0] != rows:
                        raise RuntimeError("TILLER output/cotangent rows differ")
                    self._cotangent_records[layer].append((value.index_select(0, idx).clone(), rows))
                return cotangent
            output.register_hook(capture_gradient)
            return None
        return capture

    # -- probe records for captured steps ------------------------------------
    @contextlib.contextmanager
    def probes_forced(self, enabled=True):
        """Switch the probe hooks on or off regardless of the cadence (graph captures)."""
        saved = self._capture_response_this_transition
        self._capture_response_this_transition = bool(enabled)
        try:
            yield
        finally:
            self._capture_response_this_transition = saved

    def take_probe_records(self):
        """Detach and return the records the hooks made; the router holds none afterwards."""
        if any(p is not None for p in self._pending_inputs):
            raise RuntimeError("TILLER probe input remained unmatched")
        records = (self._functional_records, self._cotangent_records)
        self._functional_records = [[] for _ in self.pairs]
        self._cotangent_records = [[] for _ in self.pairs]
        return records

    def restore_probe_records(self, records):
        """Install records made by a captured forward/backward (their tensors are
        rewritten by every replay of that graph) as this step's probes."""
        functional, cotangent = records
        self._functional_records = [list(r) for r in functional]
        self._cotangent_records = [list(r) for r in cotangent]

    def remove_hooks(self):
        for h in self._hook_handles:
            h.remove()
        self._hook_handles = []
        self._pending_inputs = [None for _ in self.pairs]
        self._functional_records = [[] for _ in self.pairs]
        self._cotangent_records = [[] for _ in self.pairs]
        self._clip_factor = None

    def _consume_probes(self):
        mb = self.microbatches
        first = self._functional_records[0][0][0] if self._functional_records[0] else None
        if not self.strict and first is not None and first.is_cuda:
            return self._consume_probes_stacked()
        packets = []
        for layer in range(len(self.pairs)):
            if self._pending_inputs[layer] is not None:
                raise RuntimeError("TILLER probe input remained unmatched")
            records = self._functional_records[layer]
            cots = self._cotangent_records[layer]
            self._functional_records[layer] = []
            self._cotangent_records[layer] = []
            if len(records) != mb or len(cots) != mb:
                raise RuntimeError("TILLER microbatch inventory changed")
            inputs = torch.cat([r[0] for r in records])
            pre = torch.cat([r[1] for r in records])
            feat = torch.cat([r[2] for r in records])
            clip = self._clip_factor if torch.is_tensor(self._clip_factor) else float(self._clip_factor)
            scaled = torch.cat([v.float() * float(rows * mb) for v, rows in cots]) * clip
            captured = self.capture_rows * mb
            if inputs.shape != (captured, self.external) or pre.shape != (captured, self.hidden):
                raise RuntimeError("TILLER captured packet changed")
            sel = tm.evenly_spaced_indices(captured, self.probe_layout.local_probe_count,
                                           device=inputs.device)
            packets.append((inputs.index_select(0, sel).float(), pre.index_select(0, sel).float(),
                            feat.index_select(0, sel).float(), scaled.index_select(0, sel).float()))
        return packets

    def _consume_probes_stacked(self):
        """The per-layer packets of :meth:`_consume_probes` built for all layers at
        once (a few launches instead of a dozen per layer); same values."""
        mb = self.microbatches
        L = len(self.pairs)
        records, cots = self._functional_records, self._cotangent_records
        if any(p is not None for p in self._pending_inputs):
            raise RuntimeError("TILLER probe input remained unmatched")
        if any(len(r) != mb for r in records) or any(len(c) != mb for c in cots):
            raise RuntimeError("TILLER microbatch inventory changed")
        self._functional_records = [[] for _ in range(L)]
        self._cotangent_records = [[] for _ in range(L)]
        factors = {rows * mb for layer in cots for _, rows in layer}
        if len(factors) != 1:
            raise RuntimeError("TILLER cotangent row counts differ across layers")

        def stacked(parts):
            return torch.stack([part[0] if mb == 1 else torch.cat(part) for part in parts])

        inputs = stacked([[r[0] for r in rec] for rec in records])
        pre = stacked([[r[1] for r in rec] for rec in records])
        feat = stacked([[r[2] for r in rec] for rec in records])
        clip = self._clip_factor if torch.is_tensor(self._clip_factor) else float(self._clip_factor)
        scaled = stacked([[v.float() for v, _ in c] for c in cots]) * float(factors.pop()) * clip
        captured = self.capture_rows * mb
        if inputs.shape[1:] != (captured, self.external) or pre.shape[1:] != (captured, self.hidden):
            raise RuntimeError("TILLER captured packet changed")
        sel = tm.evenly_spaced_indices(captured, self.probe_layout.local_probe_count, device=inputs.device)
        inputs, pre, feat, scaled = (t.index_select(1, sel).float() for t in (inputs, pre, feat, scaled))
        return [(inputs[l], pre[l], feat[l], scaled[l]) for l in range(L)]

    # -- trainer contract --------------------------------------------------
    def record_realized_clipping(self, preclip_norm, max_norm):
        """Store ``min(1, max_norm / (norm + 1e-6))`` for the probe cotangent scale.

        A device tensor norm is kept on the device (no host synchronisation);
        a Python float is validated immediately as in the reference.
        """
        if self._clip_factor is not None:
            raise RuntimeError("TILLER observed multiple clipping calls")
        maximum = float(max_norm)
        if maximum != 1.0:
            raise RuntimeError("TILLER received invalid clipping")
        if torch.is_tensor(preclip_norm) and preclip_norm.is_cuda:
            self._clip_factor = (maximum / (preclip_norm.float() + 1e-6)).clamp(max=1.0)
            return
        value = float(preclip_norm)
        if not math.isfinite(value) or value < 0.0:
            raise RuntimeError("TILLER received invalid clipping")
        self._clip_factor = min(1.0, maximum / (value + 1e-6))

    def set_telemetry_capture(self, enabled=True):
        self._capture_telemetry_next_step = bool(enabled)

    def telemetry(self):
        return dict(self._last_telemetry)

    def lr_wd_fairness_audit(self):
        keys = ("global_lr_scale", "rlb_incoming_lr_scale", "rlb_outgoing_lr_scale",
                "fixed32_loss_measure_lr_scale", "group_intrinsic_participation_lr_scale",
                "loss_weighted_frozen_response_lr_scale", "postpolar_homotopy_lr_scale",
                "batched_sensor_lr_scale", "foreach_realization_lr_scale",
                "moment_exact_compact_lr_scale", "fixed32_global_loss_measure_lr_scale",
                "signed_global_group_transaction_lr_scale", "row_space_equality_budget_lr_scale",
                "matched_beta2_predictive_loss_image_lr_scale",
                "preupdate_history_selection_lr_scale",
                "rotation_invariant_temporal_response_sketch_lr_scale",
                "rational_group_polar_lr_scale", "nominal_polar_rank_calibration_lr_scale",
                "posterior_rank64_subspace_lr_scale", "truncated_svd_response_metric_lr_scale",
                "elapsed_beta2_cadence8_response_metric_lr_scale",
                "current_linear_transaction_every_step_lr_scale",
                "cached_scalar_response_route_lr_scale", "current_window32_response_metric_lr_scale",
                "no_temporal_covariance_smearing_lr_scale",
                "matched_beta2_factorized_tangent_lr_scale", "response_energy_chord_lr_scale",
                "signed_current_gradient_orientation_lr_scale", "exact_native_budget_lr_scale",
                "compiled_static_fullgraph_execution_lr_scale",
                "every_step_gradient_score_ledger_lr_scale",
                "trace_matched_gradient_surrogate_lr_scale", "robust_fd_midpoint_tail_lr_scale",
                "matrix_free_rfd_krylov_transaction_lr_scale",
                "unchanged_compiled_factorized_direction_lr_scale",
                "signed_rfd_coefficients_lr_scale", "weight_decay_scale")
        return {k: 1.0 for k in keys}

    def consume_response_homotopy(self):
        if self._attention_consumed:
            raise RuntimeError("TILLER response route was consumed twice")
        if self._intrinsic_participation is None or self._attention_response_congruence is None:
            raise RuntimeError("TILLER attention route is incomplete")
        self._attention_consumed = True
        return self._intrinsic_participation, self._attention_response_congruence, int(self._attention_update)

    # -- sensor ------------------------------------------------------------
    def _response_sensor(self, packets):
        anchor = self.anchor
        frozen_num = anchor.get("four_role_response_frozen_numerators")
        frozen_den = anchor.get("four_role_response_frozen_denominators")
        L = len(self.pairs)
        if (frozen_num is None or frozen_num.shape != (L, self.groups, 6) or frozen_den is None
                or frozen_den.shape != (L, self.groups, 4)):
            raise RuntimeError("TILLER frozen inventory changed")
        pre = torch.stack([pk[1] for pk in packets])
        cot = torch.stack([pk[3] for pk in packets])
        nums = torch.stack([p["numerator"].detach() for p in self.pairs])
        dens = torch.stack([p["denominator"].detach() for p in self.pairs])
        outw = torch.stack([p["out_weight"].detach() for p in self.pairs])
        factors = tm.stacked_factors(pre, nums, dens, groups=self.groups, width=self.width,
                                     eps=self.grain_eps)
        adjoint = tm.response_adjoint(cot, outw, factors, groups=self.groups, width=self.width)
        part_stats, resp_stats = tm.intrinsic_and_response_statistics(
            pre, cot, adjoint, factors, frozen_num, frozen_den, eps=self.grain_eps)
        first = part_stats.numel()
        packed = torch.cat((part_stats.reshape(-1), resp_stats.reshape(-1)))
        exact = (torch.all(nums.float() == frozen_num, dim=-1)
                 & torch.all(dens.float() == frozen_den, dim=-1)).to(torch.int32)
        if self.world_size > 1:
            dist.all_reduce(packed, op=dist.ReduceOp.SUM, group=self.loss_probe_group)
            dist.all_reduce(exact, op=dist.ReduceOp.MIN, group=self.loss_probe_group)
        part_stats = packed[:first].view_as(part_stats)
        resp_stats = packed[first:].view_as(resp_stats)
        participation = tm.group_participation(part_stats)
        self._group_participation = participation
        self._group_response_congruence = tm.group_congruence(resp_stats, exact.bool())
        self._attention_response_congruence = tm.layer_congruence(resp_stats, exact.bool())
        incoming = participation[..., 0].mean(-1)
        outgoing = participation[..., 1].mean(-1)
        self._intrinsic_participation = torch.sqrt((incoming * outgoing).clamp(0.0, 1.0))
        return participation, factors, adjoint

    # -- direction ----------------------------------------------------------
    def _chord_state(self, parent, *, groups, width, axis, key_prefix):
        shape = tm.grouped_shape(parent, groups=groups, width=width, axis=axis)
        anchor = self.anchor
        rk, ck = key_prefix + "_row_second_moment", key_prefix + "_column_second_moment"
        row, col = anchor.get(rk), anchor.get(ck)
        if row is None:
            row = torch.zeros(shape[:-1], device=parent.device, dtype=torch.float32)
            anchor[rk] = row
        if col is None:
            col = torch.zeros(shape[:2] + shape[-1:], device=parent.device, dtype=torch.float32)
            anchor[ck] = col
        if row.shape != shape[:-1] or col.shape != shape[:2] + shape[-1:]:
            raise RuntimeError("saved chord state does not match this optimizer's layout")
        return row, col

    def _role_directions(self, participation, congruence):
        """Nesterov -> group NS5 -> chord for both roles; returns per-role records."""
        L = len(self.pairs)
        step = int(self.anchor.get("predictive_response_transaction_updates", 0)) + 1
        records = {}
        for role, index, axis in (("incoming", 0, "rows"), ("outgoing", 1, "columns")):
            key = "in_weight" if role == "incoming" else "out_weight"
            params = [p[key] for p in self.pairs]
            momenta = foreach_nesterov(self, params, self.momentum)
            grads = torch.stack([p.grad.detach() for p in params]).float()
            parent = rational_group_zero_power(momenta, self.ns_steps, groups=self.groups,
                                               width=self.width).float()
            row, col = self._chord_state(parent, groups=self.groups, width=self.width, axis=axis,
                                         key_prefix="factorized_adaptive_tangent_" + axis)
            pg, restore = tm.group_view(parent, groups=self.groups, width=self.width, axis=axis)
            mg, _ = tm.group_view(momenta, groups=self.groups, width=self.width, axis=axis)
            gg, _ = tm.group_view(grads, groups=self.groups, width=self.width, axis=axis)
            sel_g, meta = tm.adaptive_tangent_chord(pg, mg, gg, row, col, participation[..., index],
                                                    congruence[..., index], step)
            selected = restore(sel_g).to(parent.dtype)
            adjustment = match_rms_adamw_adjustment(params[0].shape)
            if role == "incoming":
                sb = selected.view(L, self.groups, self.width, self.external)
                gb = grads.view_as(sb)
                mb = momenta.view_as(sb)
            else:
                sb = selected.view(L, self.external, self.groups, self.width).permute(0, 2, 3, 1)
                gb = grads.view(L, self.external, self.groups, self.width).permute(0, 2, 3, 1)
                mb = momenta.view(L, self.external, self.groups, self.width).permute(0, 2, 3, 1)
            scaled = sb.float() * adjustment
            records[role] = {
                "params": params, "selected": selected, "adjustment": adjustment, "meta": meta,
                "scaled_blocks": scaled,
                "exact": (gb * scaled).sum(dim=(-2, -1)),
                "momentum": (mb.float() * scaled).sum(dim=(-2, -1)),
            }
        return records

    def _use_fused(self):
        if self._fused_ok is None:
            from . import tiller_fused
            first = self.pairs[0]["in_weight"]
            self._fused_ok = (first.is_cuda and first.dtype == torch.float32 and tiller_fused.available()
                              and not self._force_torch)
        return self._fused_ok

    def _shard(self):
        """(lo, hi, sharded): the layers whose directions this rank computes.

        With several data-parallel ranks on the GPU path each rank owns a
        contiguous block of layers: it runs the per-layer pipeline (Nesterov,
        NS5, chord, apply) for those layers only, the per-coordinate
        contractions and functional scores are assembled with one all-reduce,
        the ledger and transaction run replicated on identical inputs, and
        the updated weights are broadcast from their owners.
        """
        L = len(self.pairs)
        if sharding_enabled(self.world_size) and self._use_fused():
            rank = dist.get_rank(group=self.loss_probe_group)
            lo, hi = shard_bounds(L, rank, self.world_size)
            return lo, hi, True
        return 0, L, False

    def _fused_roles(self):
        if self._fused_role_objs is None:
            from .tiller_fused import FusedRole
            lo, hi, _ = self._shard()
            owned = self.pairs[lo:hi]
            self._fused_role_objs = {} if not owned else {
                "incoming": FusedRole(self, [p["in_weight"] for p in owned], "incoming",
                                      groups=self.groups, width=self.width, momentum=self.momentum),
                "outgoing": FusedRole(self, [p["out_weight"] for p in owned], "outgoing",
                                      groups=self.groups, width=self.width, momentum=self.momentum),
            }
        return self._fused_role_objs

    def _sync_shards(self):
        """Make every rank's optimizer state complete (checkpoints; collective)."""
        lo, hi, sharded = self._shard()
        if not sharded:
            return
        L = len(self.pairs)
        anchor = self.anchor
        keys = [k for k in ("factorized_adaptive_tangent_rows_row_second_moment",
                            "factorized_adaptive_tangent_rows_column_second_moment",
                            "factorized_adaptive_tangent_columns_row_second_moment",
                            "factorized_adaptive_tangent_columns_column_second_moment") if k in anchor]
        per_layer = []
        for layer, pair in enumerate(self.pairs):
            tensors = [self.state[pair[k]].setdefault("momentum_buffer", torch.zeros_like(pair[k]))
                       for k in ("in_weight", "out_weight")]
            tensors += [anchor[k][layer] for k in keys]
            per_layer.append(tensors)
        broadcast_owned(per_layer, L, self.world_size, self.loss_probe_group)

    def state_dict(self):
        self.finish_step()
        param_ready.wait_all()
        self._sync_shards()
        return super().state_dict()

    def _directions(self, participation, congruence, *, want_selected):
        """Both roles' directions and the contractions the transaction needs.

        Returns ``exact_by_role`` [2, C], ``momentum_by_role`` [2, C],
        ``weights`` [C], ``selected`` {role: adj*q as [L, H, d] or None},
        ``meta`` and ``apply(coefficients [L, G], lr, wd)``.
        """
        L = len(self.pairs)
        step = int(self.anchor.get("predictive_response_transaction_updates", 0)) + 1
        if self._use_fused():
            from .tiller_fused import chord_meta
            lo, hi, sharded = self._shard()
            G = self.groups
            roles = self._fused_roles()
            device = self.pairs[0]["in_weight"].device
            chords, sels = {}, {}
            for role, index, axis in (("incoming", 0, "rows"), ("outgoing", 1, "columns")):
                shape = (L, G, self.width, self.external)
                row, col = self._chord_state_shaped(shape, key_prefix="factorized_adaptive_tangent_" + axis,
                                                    device=device)
                if hi == lo:
                    continue
                chord, sel = roles[role].directions(row[lo:hi], col[lo:hi],
                                                    participation[lo:hi, :, index].contiguous(),
                                                    congruence[lo:hi, :, index].contiguous(), step,
                                                    want_selected=want_selected)
                chords[role] = chord
                sels[role] = None if sel is None else sel.view(hi - lo, self.hidden, self.external)
            packed = torch.zeros(5, L * G, device=device, dtype=torch.float32)
            if hi > lo:
                ci, co = chords["incoming"], chords["outgoing"]
                packed[:, lo * G:hi * G] = torch.stack((ci[:, 2], co[:, 2], ci[:, 3], co[:, 3], ci[:, 4] + co[:, 4]))
            if sharded:
                # one nonzero contributor per entry: the sum is exact
                dist.all_reduce(packed, group=self.loss_probe_group)

            def apply(coefficients, lr, wd):
                for role in roles:
                    roles[role].apply(coefficients[lo:hi], decay=1.0 - lr * wd, lr=lr)
                if sharded and self.packing is None:
                    broadcast_owned([(p["in_weight"], p["out_weight"]) for p in self.pairs], L,
                                    self.world_size, self.loss_probe_group, deferred=True)

            metas = {r: chord_meta(chords[r]) for r in chords}
            return {"exact_by_role": packed[0:2], "momentum_by_role": packed[2:4], "weights": packed[4],
                    "selected": sels, "meta": metas, "apply": apply, "owned": (lo, hi, sharded)}
        rec = self._role_directions(participation, congruence)
        inc_b = rec["incoming"]["scaled_blocks"]
        out_b = rec["outgoing"]["scaled_blocks"]

        def apply(coefficients, lr, wd):
            inc_sel = rec["incoming"]["selected"]
            inc_sel.view(L, self.groups, self.width, self.external).mul_(
                coefficients[..., None, None].to(inc_sel.dtype))
            out_sel = rec["outgoing"]["selected"]
            out_sel.view(L, self.external, self.groups, self.width).permute(0, 2, 3, 1).mul_(
                coefficients[..., None, None].to(out_sel.dtype))
            for role in ("incoming", "outgoing"):
                foreach_apply(rec[role]["params"], rec[role]["selected"], decay=1.0 - lr * wd,
                              alpha=-lr * rec[role]["adjustment"])

        return {"exact_by_role": torch.stack([rec[r]["exact"].reshape(-1) for r in ("incoming", "outgoing")]),
                "momentum_by_role": torch.stack([rec[r]["momentum"].reshape(-1) for r in ("incoming", "outgoing")]),
                "weights": (inc_b.square().sum(dim=(-2, -1)) + out_b.square().sum(dim=(-2, -1))).reshape(-1),
                "selected": {"incoming": inc_b.reshape(L, self.hidden, self.external),
                             "outgoing": out_b.reshape(L, self.hidden, self.external)},
                "meta": {r: rec[r]["meta"] for r in ("incoming", "outgoing")}, "apply": apply,
                "owned": (0, L, False)}

    def _chord_state_shaped(self, shape, *, key_prefix, device):
        anchor = self.anchor
        rk, ck = key_prefix + "_row_second_moment", key_prefix + "_column_second_moment"
        row, col = anchor.get(rk), anchor.get(ck)
        if row is None:
            row = torch.zeros(shape[:-1], device=device, dtype=torch.float32)
            anchor[rk] = row
        if col is None:
            col = torch.zeros(shape[:2] + shape[-1:], device=device, dtype=torch.float32)
            anchor[ck] = col
        if row.shape != shape[:-1] or col.shape != shape[:2] + shape[-1:]:
            raise RuntimeError("saved chord state does not match this optimizer's layout")
        return row, col

    # -- ledger + transaction ----------------------------------------------
    def _previous_ledger(self):
        a = self.anchor
        vals = tuple(a.get(k) for k in ("factorized_rfd_persistent_scores",
                                        "factorized_rfd_persistent_total_diagonal",
                                        "factorized_rfd_persistent_decay_cross",
                                        "factorized_rfd_persistent_isotropic_tail"))
        if all(v is None for v in vals):
            return (None, None, None, None)
        if any(not torch.is_tensor(v) for v in vals):
            raise RuntimeError("saved TILLER ledger state is only partly present")
        return vals

    def _advance_rows(self, scores, decay_action, *, functional):
        anchor = self.anchor
        ps, pd, pc, pt = self._previous_ledger()
        rows = tm.rfd_rows(scores, decay_action, ps, pd, pc, pt, validate=self.strict)
        anchor["factorized_rfd_persistent_scores"] = rows.persistent_scores.detach().clone()
        anchor["factorized_rfd_persistent_total_diagonal"] = rows.persistent_total_diagonal.detach().clone()
        anchor["factorized_rfd_persistent_decay_cross"] = rows.persistent_decay_cross.detach().clone()
        anchor["factorized_rfd_persistent_isotropic_tail"] = rows.persistent_isotropic_tail.detach().clone()
        anchor["factorized_rfd_discarded_energy_fraction"] = rows.discarded_energy_fraction.detach().clone()
        anchor["factorized_rfd_shrinkage"] = rows.fd_shrinkage.detach().clone()
        anchor["factorized_rfd_step"] = int(anchor.get("factorized_rfd_step", 0)) + 1
        if functional:
            anchor["factorized_rfd_reference_row_norm"] = tm.functional_row_norm(
                scores, validate=False).detach().clone()
            self._rfd_gradient_scale = scores.new_ones(())
        self._rfd_rows = rows
        self._rfd_functional_refresh = bool(functional)
        return rows

    def _transaction(self, exact_by_role, momentum_by_role, weights, layer_ids, *, eta):
        if self._rfd_rows is None:
            reference = self.anchor.get("factorized_rfd_reference_row_norm")
            decay = self._rfd_decay_derivative
            if not torch.is_tensor(reference) or not torch.is_tensor(decay):
                raise RuntimeError("the ledger needs a functional refresh before its first surrogate step")
            scores, decay_action, scale = tm.trace_matched_surrogate(exact_by_role, decay, reference)
            self._rfd_gradient_scale = scale
            self._advance_rows(scores, decay_action, functional=False)
        result = tm.biatlas_transaction(self._rfd_rows, exact_by_role, momentum_by_role, weights,
                                        layer_ids, total_layers=len(self.pairs), eta=float(eta),
                                        rounds=64, diagnostics=bool(self._capture_telemetry_next_step),
                                        validate=self.strict)
        self._rfd_selection = result
        return result

    @property
    def _ledger_timing(self):
        if os.environ.get("RO_LEDGER_TIMING") != "1":
            return None
        if not hasattr(self, "ledger_timings"):
            self.ledger_timings = []
        return torch.zeros(16, dtype=torch.int64, device=self.pairs[0]["in_weight"].device)

    def _fast_ledger_ok(self):
        return (self._use_fused() and not self.strict and not self._capture_telemetry_next_step
                and hasattr(__import__("rational_optimizer_b200._ext", fromlist=["ext"]).ext(),
                            "tiller_ledger_transaction"))

    def _ledger_fast(self, *, functional, scores, decay, exact_by_role, momentum_by_role, weights,
                     layer_ids, eta, stream=None):
        """Ledger advance + transaction in one single-CTA fp64 kernel (csrc/ledger.cu).

        ``stream``: run the kernel there, after the work queued so far on the
        current stream; its inputs are recorded on that stream and its outputs
        on the current one, so the caching allocator keeps both alive across
        the two streams.
        """
        from .._ext import ext
        C = ext()
        anchor = self.anchor
        n = int(weights.numel())
        dev = weights.device
        if self._ledger_bufs is None or self._ledger_bufs[0].shape[1] != n:
            self._ledger_bufs = (torch.zeros(tm.PERSISTENT_ROWS, n, device=dev),
                                 torch.zeros(n, device=dev), torch.zeros(n, device=dev),
                                 torch.zeros(8, device=dev),
                                 torch.empty(int(C.tiller_ledger_workspace(n)), device=dev,
                                             dtype=torch.float64))
        pers, diag, cross, scal, ws = self._ledger_bufs
        prev = anchor.get("factorized_rfd_persistent_scores")
        prev_rows = 0 if prev is None else int(prev.shape[0])
        if prev is not None and prev.data_ptr() != pers.data_ptr():
            pers[:prev_rows].copy_(prev)
            diag.copy_(anchor["factorized_rfd_persistent_total_diagonal"])
            cross.copy_(anchor["factorized_rfd_persistent_decay_cross"])
            scal[0].copy_(anchor["factorized_rfd_persistent_isotropic_tail"].reshape(()))
        if not functional:
            ref = anchor.get("factorized_rfd_reference_row_norm")
            if not torch.is_tensor(ref) or not torch.is_tensor(self._rfd_decay_derivative):
                raise RuntimeError("the ledger needs a functional refresh before its first surrogate step")
            if ref.data_ptr() != scal[3].data_ptr():
                scal[3].copy_(ref.reshape(()))
        dd = None if functional else self._rfd_decay_derivative.reshape(1).float().contiguous()
        timing = None if stream is not None else self._ledger_timing
        inputs = [scores.float().contiguous() if functional else None,
                  decay.float().contiguous() if functional else None,
                  exact_by_role.float().contiguous(), momentum_by_role.float().contiguous(),
                  weights.float().contiguous(), layer_ids.contiguous(), dd]
        if stream is None:
            coef, cand, result = C.tiller_ledger_transaction(*inputs, pers, diag, cross, scal, ws, prev_rows,
                                                             len(self.pairs), float(eta), timing=timing)
        else:
            main = torch.cuda.current_stream(dev)
            stream.wait_stream(main)
            for t in inputs:
                if t is not None:
                    t.record_stream(stream)
            with torch.cuda.stream(stream):
                coef, cand, result = C.tiller_ledger_transaction(*inputs, pers, diag, cross, scal, ws,
                                                                 prev_rows, len(self.pairs), float(eta),
                                                                 timing=None)
            for t in (coef, cand, result):
                t.record_stream(main)
        if timing is not None:
            # diagnostics (RO_LEDGER_TIMING=1): phase clock stamps and eigensolver sweeps
            # (-1: arrowhead path) of every ledger call, kept on the host
            self.ledger_timings.append(timing.cpu().tolist())
        new_rows = tm.CURRENT_ROWS if prev_rows == 0 else tm.PERSISTENT_ROWS
        anchor["factorized_rfd_persistent_scores"] = pers[:new_rows]
        anchor["factorized_rfd_persistent_total_diagonal"] = diag
        anchor["factorized_rfd_persistent_decay_cross"] = cross
        anchor["factorized_rfd_persistent_isotropic_tail"] = scal[0]
        anchor["factorized_rfd_discarded_energy_fraction"] = scal[1]
        anchor["factorized_rfd_shrinkage"] = scal[2]
        anchor["factorized_rfd_reference_row_norm"] = scal[3]
        anchor["factorized_rfd_step"] = int(anchor.get("factorized_rfd_step", 0)) + 1
        self._rfd_gradient_scale = result[6]
        self._rfd_functional_refresh = bool(functional)
        self._rfd_rows = tm.LedgerRows(
            selection_scores=pers.new_empty((prev_rows + tm.CURRENT_ROWS if prev_rows else tm.CURRENT_ROWS, 0)),
            selection_diagonal_residual=None, persistent_scores=pers[:new_rows],
            persistent_total_diagonal=diag, persistent_diagonal_residual=None,
            persistent_decay_cross=cross, history_used=prev_rows > 0,
            discarded_energy_fraction=scal[1], selection_isotropic_tail=None,
            persistent_isotropic_tail=scal[0], fd_shrinkage=scal[2])
        zero = result.new_zeros(1)
        sel = tm.TransactionResult(coef, cand, result[0:1] > 0.5, result[1:2], result[2:3] > 0.5,
                                   result[3:4], result[4:5], result[5:6],
                                   torch.zeros(1, dtype=torch.int64, device=dev), zero, zero, zero, zero)
        self._rfd_selection = sel
        return sel

    def _sharded_scores(self, packets, adjoint, selected, lo, hi, wd):
        """Functional score rows [32, C + 1] when layers are sharded across ranks.

        Every rank's probe data (inputs, features, cotangents, adjoints) is
        gathered so each owner scores its layers on all 32 global probes; the
        score columns (one owner each) and the decay column (sum of per-owner
        partial sums) are then assembled with one all-reduce, in the global
        probe order of the unsharded path.
        """
        L, G = len(self.pairs), self.groups
        world = self.world_size
        probes = tm.GLOBAL_PROBE_COUNT
        counts = [(r + 1) * probes // world - r * probes // world for r in range(world)]
        width = max(counts)
        local = torch.stack([torch.cat((pk[0].float(), pk[2].float(), pk[3].float(),
                                        adjoint[i].reshape(adjoint.shape[1], -1).float()), dim=1)
                             for i, pk in enumerate(packets)])  # [L, n_local, K]
        padded = local.new_zeros((L, width, local.shape[-1]))
        if local.shape[1]:
            padded[:, : local.shape[1]] = local
        gathered = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(gathered, padded, group=self.loss_probe_group)
        rows = torch.cat([g[:, :n] for g, n in zip(gathered, counts)], dim=1)  # [L, 32, K]
        d_ext, hid = self.external, self.hidden
        full = rows.new_zeros((probes, L * G + 1))
        for layer in range(lo, hi):
            pair = self.pairs[layer]
            r = rows[layer]
            inputs, features = r[:, :d_ext], r[:, d_ext:d_ext + hid]
            cot = r[:, d_ext + hid:2 * d_ext + hid]
            adj = r[:, 2 * d_ext + hid:].reshape(r.shape[0], G, self.width)
            s = tm.group_scores(inputs, features, cot, selected["incoming"][layer - lo],
                                selected["outgoing"][layer - lo], adj, groups=G, width=self.width,
                                validate=self.strict)
            d = tm.group_scores(inputs, features, cot, pair["in_weight"].float() * wd,
                                pair["out_weight"].T.float() * wd, adj, groups=G, width=self.width,
                                validate=self.strict).sum(-1)
            full[:, layer * G:(layer + 1) * G] = s
            full[:, -1] += d
        dist.all_reduce(full, group=self.loss_probe_group)
        return full

    def _gather_rows(self, packet):
        if self.world_size == 1:
            if packet.shape[0] != tm.GLOBAL_PROBE_COUNT:
                raise RuntimeError("the gathered probe rows do not add up to the fixed probe count")
            return packet
        probes = tm.GLOBAL_PROBE_COUNT
        counts = [(r + 1) * probes // self.world_size - r * probes // self.world_size
                  for r in range(self.world_size)]
        maximum = max(counts)
        padded = packet.new_zeros((maximum, packet.shape[1]))
        if packet.shape[0]:
            padded[: packet.shape[0]].copy_(packet)
        gathered = [torch.empty_like(padded) for _ in range(self.world_size)]
        dist.all_gather(gathered, padded, group=self.loss_probe_group)
        return torch.cat([g[:n] for g, n in zip(gathered, counts)], dim=0)

    # -- step -----------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None, *, defer_apply=False):
        """One router transition.

        ``defer_apply``: when the single-CTA ledger kernel runs, launch it on a
        side stream and return before the weights are updated, so the caller
        can run independent work (the attention optimizer, AdamW) beside it;
        :meth:`finish_step` then waits for the ledger and applies the update.
        The attention route is published before returning in both cases.
        """
        if self._pending_apply is not None:
            raise RuntimeError("TILLER router step started before the previous one finished")
        if self._clip_factor is None:
            raise RuntimeError("TILLER lacks realized clipping")
        if not self._attention_consumed:
            raise RuntimeError("TILLER would overwrite attention state")
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        group = self.param_groups[0]
        if float(group.get("lr_scale", 1.0)) != 1.0:
            raise RuntimeError("TILLER refuses nonunit LR scale")
        lr = float(group["lr"])
        wd = float(group["weight_decay"])
        publish = bool(self._capture_telemetry_next_step)
        self._last_telemetry = {}
        self._rfd_rows = None
        self._rfd_functional_refresh = False
        self._rfd_gradient_scale = None
        self._rfd_selection = None
        refresh = bool(self._capture_response_this_transition)
        for pair in self.pairs:
            for key in ("in_weight", "out_weight"):
                if pair[key].grad is None:
                    raise RuntimeError("a TILLER-managed matrix has no gradient this step")
        if not refresh:
            self._rfd_decay_derivative = self._decay_derivative(wd)
        L = len(self.pairs)
        anchor = self.anchor
        if refresh:
            packets = self._consume_probes()
            participation, factors, adjoint = self._response_sensor(packets)
        else:
            self._restore_route()
            participation = self._group_participation
        congruence = self._group_response_congruence
        dirs = self._directions(participation, congruence, want_selected=refresh)
        weights = dirs["weights"]
        exact_by_role = dirs["exact_by_role"]
        momentum_by_role = dirs["momentum_by_role"]
        layer_ids = torch.arange(L, device=weights.device, dtype=torch.int64).repeat_interleave(self.groups)
        side = None
        if defer_apply and weights.is_cuda and self._fast_ledger_ok() and self._ledger_timing is None:
            side = self._ledger_side_stream(weights.device)
        if refresh:
            lo, hi, sharded = dirs["owned"]
            if sharded:
                global_packet = self._sharded_scores(packets, adjoint, dirs["selected"], lo, hi, wd)
            elif not self.strict and packets[0][0].is_cuda:
                # every layer at once (batched GEMMs); the per-layer loop below is the
                # CPU oracle's path
                inputs = torch.stack([pk[0] for pk in packets])
                features = torch.stack([pk[2] for pk in packets])
                cot = torch.stack([pk[3] for pk in packets])
                s = tm.group_scores_stacked(inputs, features, cot, dirs["selected"]["incoming"],
                                            dirs["selected"]["outgoing"], adjoint, groups=self.groups,
                                            width=self.width)
                w_in = torch.stack([p["in_weight"] for p in self.pairs])
                w_out_t = torch.stack([p["out_weight"].T for p in self.pairs])
                decay = (tm.group_scores_stacked(inputs, features, cot, w_in, w_out_t, adjoint,
                                                 groups=self.groups, width=self.width).sum(-1) * wd).sum(0)
                lattice = s.transpose(0, 1).reshape(self.probe_layout.local_probe_count, L * self.groups)
                global_packet = self._gather_rows(torch.cat((lattice, decay[:, None]), dim=1))
            else:
                inc_b = dirs["selected"]["incoming"]
                out_b = dirs["selected"]["outgoing"]
                scores, decay = [], None
                for layer, (pair, packet) in enumerate(zip(self.pairs, packets)):
                    inputs, _pre, features, cot = packet
                    adj = adjoint[layer]
                    s = tm.group_scores(inputs, features, cot, inc_b[layer], out_b[layer], adj,
                                        groups=self.groups, width=self.width, validate=self.strict)
                    d = tm.group_scores(inputs, features, cot, pair["in_weight"].float() * wd,
                                        pair["out_weight"].T.float() * wd, adj, groups=self.groups,
                                        width=self.width, validate=self.strict).sum(-1)
                    scores.append(s)
                    decay = d if decay is None else decay + d
                lattice = torch.stack(scores, dim=1).reshape(self.probe_layout.local_probe_count,
                                                             L * self.groups)
                packet = torch.cat((lattice, decay[:, None]), dim=1)
                global_packet = self._gather_rows(packet)
            g_scores, g_decay = global_packet[:, :-1], global_packet[:, -1]
            predictive = tm.window32_rows(g_scores, g_decay, anchor.get("predictive_global_score_ema"),
                                          anchor.get("predictive_global_decay_ema"),
                                          validate=self.strict)
            if self._fast_ledger_ok():
                selection = self._ledger_fast(functional=True, scores=g_scores, decay=g_decay,
                                              exact_by_role=exact_by_role,
                                              momentum_by_role=momentum_by_role, weights=weights,
                                              layer_ids=layer_ids, eta=lr, stream=side)
            else:
                self._advance_rows(g_scores, g_decay, functional=True)
                selection = self._transaction(exact_by_role, momentum_by_role, weights, layer_ids,
                                              eta=lr)
            anchor["predictive_global_score_ema"] = predictive.updated_scores.detach().clone()
            anchor["predictive_global_decay_ema"] = predictive.updated_decay_action.detach().clone()
            self._last_predictive = predictive
        else:
            if self._cached_selection_scores is None or self._cached_selection_decay is None:
                raise RuntimeError("TILLER selection factor is missing")
            if self._fast_ledger_ok():
                selection = self._ledger_fast(functional=False, scores=None, decay=None,
                                              exact_by_role=exact_by_role,
                                              momentum_by_role=momentum_by_role, weights=weights,
                                              layer_ids=layer_ids, eta=lr, stream=side)
            else:
                selection = self._transaction(exact_by_role, momentum_by_role, weights, layer_ids,
                                              eta=lr)
        updates = int(anchor.get("predictive_response_transaction_updates", 0)) + 1
        anchor["predictive_response_transaction_updates"] = updates
        self._attention_update = updates
        self._attention_consumed = False
        tail = (selection, dirs, refresh, publish, lr, wd)
        if side is not None:
            event = torch.cuda.Event()
            event.record(side)
            self._pending_apply = (event, tail)
            return loss
        self._complete_step(*tail)
        return loss

    def finish_step(self):
        """Apply a deferred transition (no-op when nothing is pending)."""
        pending, self._pending_apply = self._pending_apply, None
        if pending is None:
            return
        event, tail = pending
        torch.cuda.current_stream(self.pairs[0]["in_weight"].device).wait_event(event)
        with torch.no_grad():
            self._complete_step(*tail)
        if self._packing_due:
            self._packing_due = False
            self.packing.broadcast()

    def _ledger_side_stream(self, device):
        if self._side_stream is None:
            self._side_stream = torch.cuda.Stream(device=device)
        return self._side_stream

    def _complete_step(self, selection, dirs, refresh, publish, lr, wd):
        coefficients = selection.coefficients.view(len(self.pairs), self.groups)
        dirs["apply"](coefficients, lr, wd)
        if refresh:
            self._cache_refresh_state()
        if publish:
            self._publish_telemetry(refresh, coefficients, dirs["meta"], selection)
        self._advance_cadence()
        self._rfd_decay_derivative = None
        self._capture_telemetry_next_step = False
        self._clip_factor = None

    def _decay_derivative(self, wd):
        """wd * sum over routed matrices of <grad, weight> (optimizer_design/_tiller/core.py:4511-4519).

        Layer-sharded: each rank sums over the layers it owns (whose averaged
        gradient it holds, whatever the gradient transport) and the partial
        sums are all-reduced, so every rank gets the same value.
        """
        lo, hi, sharded = self._shard()
        if sharded:
            pairs = self.pairs[lo:hi]
            tensors = [(p[k].grad.detach(), p[k].detach()) for p in pairs for k in ("in_weight", "out_weight")]
            device = self.pairs[0]["in_weight"].device
            if tensors:
                from .._ext import ext
                part = ext().multi_tensor_dot([g for g, _ in tensors], [w for _, w in tensors], float(wd))
                part = part.reshape(1).clone()
            else:
                part = torch.zeros(1, device=device, dtype=torch.float32)
            dist.all_reduce(part, group=self.loss_probe_group)
            return part.reshape(())
        tensors = [(p[k].grad.detach(), p[k].detach()) for p in self.pairs for k in ("in_weight", "out_weight")]
        if self._use_fused() and all(g.dtype == torch.float32 and g.is_contiguous() and w.is_contiguous()
                                     for g, w in tensors):
            from .._ext import ext
            return ext().multi_tensor_dot([g for g, _ in tensors], [w for _, w in tensors], float(wd))
        terms = [(g.float() * w.float()).sum() for g, w in tensors]
        return torch.stack(terms).sum() * wd

    def _cache_refresh_state(self):
        route = {
            "group_participation": self._group_participation.detach().clone(),
            "group_congruence": self._group_response_congruence.detach().clone(),
            "intrinsic_participation": self._intrinsic_participation.detach().clone(),
            "attention_congruence": self._attention_response_congruence.detach().clone(),
        }
        self._cached_route = route
        anchor = self.anchor
        for name, value in route.items():
            anchor["cadence8_" + name] = value
        anchor["cadence8_relative_score_innovation"] = self._last_predictive.relative_innovation.detach().clone()
        self._cached_selection_scores = anchor["predictive_global_score_ema"]
        self._cached_selection_decay = anchor["predictive_global_decay_ema"]
        anchor["cadence8_transition"] = int(self._cadence_transition)

    def _restore_route(self):
        route = self._cached_route
        if route is None or set(route) != set(_ROUTE_NAMES):
            raise RuntimeError("TILLER cached response route is incomplete")
        self._group_participation = route["group_participation"]
        self._group_response_congruence = route["group_congruence"]
        self._intrinsic_participation = route["intrinsic_participation"]
        self._attention_response_congruence = route["attention_congruence"]

    def _advance_cadence(self):
        self._cadence_transition += 1
        self.anchor["cadence8_transition"] = self._cadence_transition
        self._capture_response_this_transition = self._cadence_transition % tm.REFRESH_INTERVAL == 0

    def _publish_telemetry(self, refresh, coefficients, meta, selection):
        flat = coefficients.reshape(-1).float()
        safe = torch.cat([meta[r]["safe"].reshape(-1) for r in ("incoming", "outgoing")])
        cosine = torch.cat([meta[r]["parent_cosine"].reshape(-1) for r in ("incoming", "outgoing")])
        energy = torch.cat([meta[r]["departure_energy"].reshape(-1) for r in ("incoming", "outgoing")])
        rows = self._rfd_rows
        scaling = tiller_scaling_formula(total_positions=1, total_layers=len(self.pairs),
                                         total_groups=self.groups, intermediate_width=self.hidden,
                                         model_width=self.external)
        P = PREFIX
        self._last_telemetry = {
            P + "family_id": FAMILY_ID,
            P + "response_refreshed": int(refresh),
            P + "response_age": 0 if refresh else self._cadence_transition % tm.REFRESH_INTERVAL,
            P + "functional_score_refresh": int(self._rfd_functional_refresh),
            P + "trace_matched_gradient_surrogate": int(not self._rfd_functional_refresh),
            P + "gradient_score_scale": float(self._rfd_gradient_scale.item()),
            P + "ledger_step": int(self.anchor["factorized_rfd_step"]),
            P + "selection_factor_rows": int(rows.selection_scores.shape[0]),
            P + "persistent_factor_rows": int(rows.persistent_scores.shape[0]),
            P + "persistent_isotropic_tail": float(rows.persistent_isotropic_tail.item()),
            P + "fd_shrinkage": float(rows.fd_shrinkage.item()),
            P + "transaction_accepted": int(selection.accepted.item()),
            P + "rank": int(selection.factor_rank.item()),
            P + "budget_residual": float(selection.budget_residual.item()),
            P + "cross_layer_coupling_ratio": float(selection.cross_layer_coupling_ratio.item()),
            P + "coefficient_min": float(flat.amin().item()),
            P + "coefficient_median": float(flat.median().item()),
            P + "coefficient_max": float(flat.amax().item()),
            P + "adaptive_tangent_safe_fraction": float(safe.float().mean().item()),
            P + "adaptive_tangent_parent_cosine_median": float(cosine.median().item()),
            P + "departure_energy_median": float(energy.median().item()),
            P + "state_coordinate_count": scaling["persistent_state_elements"],
            P + "ledger_checkpoint_tensor_elements": scaling["ledger_checkpoint_tensor_elements"],
            P + "realized_clip_factor": float(self._clip_factor),
        }

    # -- checkpoint ------------------------------------------------------------
    def load_state_dict(self, state_dict):
        result = super().load_state_dict(state_dict)
        anchor = self.anchor
        step = anchor.get("cadence8_transition")
        if not isinstance(step, int) or step < 0:
            raise RuntimeError("the saved refresh-cadence step is missing or negative")
        self._cadence_transition = step
        self._capture_response_this_transition = step % tm.REFRESH_INTERVAL == 0
        route = {name: anchor.get("cadence8_" + name) for name in _ROUTE_NAMES}
        if any(not torch.is_tensor(v) for v in route.values()):
            raise RuntimeError("the saved refresh-cadence route tensors are missing")
        self._cached_route = route
        self._cached_selection_scores = anchor.get("predictive_global_score_ema")
        self._cached_selection_decay = anchor.get("predictive_global_decay_ema")
        if not torch.is_tensor(self._cached_selection_scores) or not torch.is_tensor(self._cached_selection_decay):
            raise RuntimeError("the saved selection-factor tensors are missing")
        innov = anchor.get("cadence8_relative_score_innovation")
        if innov is not None and (not torch.is_tensor(innov) or innov.numel() != 1):
            raise RuntimeError("the saved score-innovation record is not a single value")
        self._previous_ledger()
        ref = anchor.get("factorized_rfd_reference_row_norm")
        st = anchor.get("factorized_rfd_step")
        if not torch.is_tensor(ref) or ref.numel() != 1 or type(st) is not int or st < 1:
            raise RuntimeError("the saved ledger reference norm or step counter is missing or invalid")
        self._rfd_rows = None
        self._rfd_gradient_scale = None
        self._rfd_selection = None
        self._rfd_decay_derivative = None
        self._attention_update = 0
        self._attention_consumed = True
        return result


class TILLERAttentionOptimizer(torch.optim.Optimizer):
    """TILLER on the attention ``qkv``/``out`` matrices, driven by the router's route."""

    _ROLES = ("qkv", "attn_out")

    def __init__(self, blocks, router: TILLERRouter, *, lr, weight_decay, momentum, ns_steps, beta2,
                 eps, adjust_lr_fn):
        if (float(lr) != 0.0003 or float(weight_decay) != 0.1 or float(momentum) != 0.95
                or int(ns_steps) != 5 or float(beta2) != 0.95 or float(eps) != 1e-08
                or adjust_lr_fn != "match_rms_adamw"):
            raise ValueError("TILLER attention requires the locked cell")
        self.blocks = sorted((dict(b) for b in blocks), key=lambda b: int(b["layer_index"]))
        if [int(b["layer_index"]) for b in self.blocks] != list(range(len(self.blocks))):
            raise ValueError("TILLER attention layer inventory changed")
        self.router = router
        self.momentum = float(momentum)
        self.ns_steps = int(ns_steps)
        self.role_parameters = {"qkv": [b["qkv_weight"] for b in self.blocks],
                                "attn_out": [b["attn_out_weight"] for b in self.blocks]}
        params = []
        seen = {id(pair[r]) for pair in router.pairs for r in ("in_weight", "out_weight")}
        for role in self._ROLES:
            for p in self.role_parameters[role]:
                if p.ndim != 2 or id(p) in seen:
                    raise ValueError("TILLER attention ownership changed")
                seen.add(id(p))
                params.append(p)
        group = {"params": params, "lr": float(lr), "weight_decay": float(weight_decay), "lr_scale": 1.0}
        group.update(_ATTENTION_GROUP_KEYS)
        super().__init__([group], {})
        self._capture_telemetry_next_step = False
        self._last_telemetry = {}
        self._fused = {}

    def lr_wd_fairness_audit(self):
        keys = ("global_lr_scale", "qkv_lr_scale", "attention_output_lr_scale",
                "residual_coordinate_fisher_lr_scale", "single_ns5_per_attention_role_lr_scale",
                "moment_exact_compact_lr_scale", "lagged_predictive_response_attention_lr_scale",
                "attention_head_group_polar_lr_scale",
                "attention_nominal_polar_rank_calibration_lr_scale",
                "posterior_rank64_attention_lr_scale", "posterior_rank64_cadence8_attention_lr_scale",
                "window32_cadence8_attention_lr_scale",
                "attention_matched_beta2_factorized_tangent_lr_scale",
                "attention_response_energy_chord_lr_scale",
                "attention_signed_current_gradient_orientation_lr_scale",
                "attention_compiled_static_fullgraph_execution_lr_scale",
                "unchanged_compiled_factorized_attention_lr_scale", "weight_decay_scale")
        return {k: 1.0 for k in keys}

    def set_telemetry_capture(self, enabled=True):
        self._capture_telemetry_next_step = bool(enabled)

    def telemetry(self):
        return dict(self._last_telemetry)

    def _sync_shards(self):
        """Complete every rank's state when layers are sharded (collective)."""
        if not hasattr(self.router, "_shard"):
            return
        _, _, sharded = self.router._shard()
        if not sharded:
            return
        L = len(self.blocks)
        anchor = self.state[self.role_parameters["qkv"][0]]
        keys = [k for k in ("factorized_adaptive_tangent_qkv_row_second_moment",
                            "factorized_adaptive_tangent_qkv_column_second_moment",
                            "factorized_adaptive_tangent_attention_output_row_second_moment",
                            "factorized_adaptive_tangent_attention_output_column_second_moment") if k in anchor]
        per_layer = []
        for layer in range(L):
            tensors = [self.state[self.role_parameters[r][layer]].setdefault(
                "momentum_buffer", torch.zeros_like(self.role_parameters[r][layer])) for r in self._ROLES]
            tensors += [anchor[k][layer] for k in keys]
            per_layer.append(tensors)
        broadcast_owned(per_layer, L, self.router.world_size, self.router.loss_probe_group)

    def state_dict(self):
        param_ready.wait_all()
        self._sync_shards()
        return super().state_dict()

    @torch.no_grad()
    def step(self, closure=None):
        self._last_telemetry = {}
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        group = self.param_groups[0]
        if float(group.get("lr_scale", 1.0)) != 1.0:
            raise RuntimeError("TILLER attention refuses nonunit LR scale")
        lr = float(group["lr"])
        wd = float(group["weight_decay"])
        participation, congruence, router_update = self.router.consume_response_homotopy()
        anchor = self.state[self.role_parameters["qkv"][0]]
        previous = int(anchor.get("compact_response_homotopy_router_update", 0))
        if int(router_update) != previous + 1:
            raise RuntimeError("TILLER attention missed a router update")
        anchor["compact_response_homotopy_router_update"] = int(router_update)
        update = int(anchor.get("factorized_adaptive_tangent_updates", 0)) + 1
        metas = []
        first = self.role_parameters["qkv"][0]
        from . import tiller_fused
        fused = (first.is_cuda and first.dtype == torch.float32 and tiller_fused.available()
                 and not getattr(self.router, "_force_torch", False))
        for role, key in (("qkv", "qkv"), ("attn_out", "attention_output")):
            params = self.role_parameters[role]
            rows, cols = params[0].shape
            shape = (len(params), 1, rows, cols)
            rk = "factorized_adaptive_tangent_" + key + "_row_second_moment"
            ck = "factorized_adaptive_tangent_" + key + "_column_second_moment"
            row, col = anchor.get(rk), anchor.get(ck)
            if row is None:
                row = torch.zeros(shape[:-1], device=first.device, dtype=torch.float32)
                anchor[rk] = row
            if col is None:
                col = torch.zeros(shape[:2] + shape[-1:], device=first.device, dtype=torch.float32)
                anchor[ck] = col
            if fused:
                lo, hi, sharded = self.router._shard() if hasattr(self.router, "_shard") else (0, len(params), False)
                if hi > lo:
                    if role not in self._fused:
                        self._fused[role] = tiller_fused.FusedRole(self, params[lo:hi], role,
                                                                   momentum=self.momentum)
                    fr = self._fused[role]
                    chord, _ = fr.directions(row[lo:hi], col[lo:hi], participation[lo:hi].contiguous(),
                                             congruence[lo:hi].contiguous(), update, want_selected=False)
                    fr.apply(torch.ones(hi - lo, device=first.device), decay=1.0 - lr * wd, lr=lr)
                    metas.append(tiller_fused.chord_meta(chord))
                if sharded and self.router.packing is None:
                    broadcast_owned([(p,) for p in params], len(params), self.router.world_size,
                                    self.router.loss_probe_group, deferred=True)
                continue
            momenta = foreach_nesterov(self, params, self.momentum)
            grads = torch.stack([p.grad.detach() for p in params]).float()
            parent = attention_head_group_zero_power(momenta, self.ns_steps).float()
            pg, restore = tm.group_view(parent, groups=1, width=None, axis="matrix")
            mg, _ = tm.group_view(momenta, groups=1, width=None, axis="matrix")
            gg, _ = tm.group_view(grads, groups=1, width=None, axis="matrix")
            sel, meta = tm.adaptive_tangent_chord(pg, mg, gg, row, col, participation[:, None],
                                                  congruence[:, None], update)
            metas.append(meta)
            adjustment = match_rms_adamw_adjustment(params[0].shape)
            foreach_apply(params, restore(sel).to(parent.dtype), decay=1.0 - lr * wd,
                          alpha=-lr * adjustment)
        anchor["factorized_adaptive_tangent_updates"] = update
        if fused and self.router.packing is not None and self.router._shard()[2]:
            if self.router._pending_apply is not None:
                # the router's deferred update lands in the same owner buffer
                self.router._packing_due = True
            else:
                self.router.packing.broadcast()
        if self._capture_telemetry_next_step:
            safe = torch.cat([m["safe"].reshape(-1) for m in metas])
            cosine = torch.cat([m["parent_cosine"].reshape(-1) for m in metas])
            self._last_telemetry = {
                PREFIX + "attention_family_id": FAMILY_ID,
                PREFIX + "attention_router_update": int(router_update),
                PREFIX + "attention_adaptive_tangent_safe_fraction": float(safe.float().mean()),
                PREFIX + "attention_adaptive_tangent_parent_cosine_median": float(cosine.median()),
            }
        self._capture_telemetry_next_step = False
        return loss
