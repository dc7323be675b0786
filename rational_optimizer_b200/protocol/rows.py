"""Matrix rows of the matched TILLER experiments and their trainer arguments.

Formats (interfaces, kept as published; reference
experiments/protocol/build_matrix.py and suite.py:39-247):

* ``matrix.json`` - ``{"schema", "rows": [row, ...], ...}``; a row is a flat
  dict holding every trainer hyper-parameter plus ``control_*`` /
  ``candidate_*`` activation and optimizer, ``phase``, ``dataset``,
  ``matrix_index`` and the source-manifest identifiers;
* ``activation_optimizer_manifest.csv`` - one run per line with the same
  hyper-parameter columns (``row_index``, ``row_id``, ``method``, ...).

:func:`training_argv` yields the trainer flags of one arm (run name,
fairness contract, identity, data, model, schedule, telemetry), exactly the
flags the published protocol passes, so a row reproduces the published
configuration.  :func:`rebalance` re-derives ``batch_size`` / ``grad_accum``
for a different number of GPUs at the SAME global tokens per step (the
published rows were laid out for 4 GPUs; one B200 node has 8).
"""
from __future__ import annotations

import csv
import json
from pathlib import Path
from typing import Any

EXACT_OPTIMIZER_KEY = "tiller_v1"
TWO_STAGE_OPTIMIZER_KEY = "tiller_then_muon_v1"
PRIMARY_PHASE = "18l_1024d_100m_tokens_3050_steps"
EXACT_LR_WD_CONTRACT = "exact_lr_wd_v1"
TILLER_EXPERIMENT_IDENTITY = "tiller_matrix_v1"
TILLER_THEN_MUON_EXPERIMENT_IDENTITY = "tiller_then_muon_matrix_v1"
ARMS = ("control", "candidate")


def load_matrix(path) -> dict:
    payload = json.loads(Path(path).read_text(encoding="utf-8"))
    if not isinstance(payload, dict) or not isinstance(payload.get("rows"), list):
        raise RuntimeError(f"{path} is not a matrix payload with a rows list")
    for i, row in enumerate(payload["rows"]):
        if int(row.get("matrix_index", -1)) != i:
            raise RuntimeError(f"matrix row {i} carries matrix_index {row.get('matrix_index')}")
    return payload


def row_at(payload: dict, index: int) -> dict:
    rows = payload["rows"]
    if not 0 <= int(index) < len(rows):
        raise IndexError(f"matrix index {index} outside 0..{len(rows) - 1}")
    return dict(rows[int(index)])


def load_manifest(path) -> list[dict[str, str]]:
    with open(path, newline="", encoding="utf-8") as fh:
        rows = list(csv.DictReader(fh))
    for i, row in enumerate(rows):
        if int(row["row_index"]) != i:
            raise RuntimeError(f"manifest line {i} carries row_index {row['row_index']}")
    return rows


def contract(row) -> str:
    return EXACT_LR_WD_CONTRACT


def experiment_identity(row) -> str:
    if row["candidate_optimizer"] == TWO_STAGE_OPTIMIZER_KEY:
        return TILLER_THEN_MUON_EXPERIMENT_IDENTITY
    return TILLER_EXPERIMENT_IDENTITY


def _arm_prefix(arm: str) -> str:
    if arm not in ARMS:
        raise RuntimeError(f"unknown arm {arm!r}")
    return arm


def run_name(row, arm: str) -> str:
    _arm_prefix(arm)
    if arm == "control":
        suffix = "control"
    else:
        suffix = {EXACT_OPTIMIZER_KEY: "tiller", TWO_STAGE_OPTIMIZER_KEY: "tiller_then_muon"}.get(
            row["candidate_optimizer"])
        if suffix is None:
            raise RuntimeError("unrecognized TILLER candidate optimizer")
    return f"{row['phase']}-{row['dataset']}-seed{row['seed']}-{suffix}"


def jsonl_path(row, arm: str, output_root) -> Path:
    root = Path(output_root)
    if _arm_prefix(arm) == "control":
        return root / row["phase"] / row["dataset"] / row["source_manifest_row_id"] / f"{row['control_activation']}.jsonl"
    return root / run_name(row, arm) / f"{row['candidate_activation']}.jsonl"


def rebalance(row, world_size: int, *, max_batch_per_gpu: int | None = None) -> dict:
    """Per-GPU batch and accumulation for ``world_size`` GPUs at the row's global tokens.

    global_tokens_per_step = batch_size * grad_accum * world * seq_len is
    preserved; the largest per-GPU batch (fewest accumulation steps) that
    divides the per-GPU share and respects ``max_batch_per_gpu`` is chosen.
    """
    seq = int(row["seq_len"])
    total = int(row["global_tokens_per_step"])
    if total % (seq * int(world_size)):
        raise ValueError(f"{total} tokens per step do not split over {world_size} GPUs x {seq} tokens")
    per_gpu = total // (seq * int(world_size))
    limit = per_gpu if max_batch_per_gpu is None else min(per_gpu, int(max_batch_per_gpu))
    for batch in range(limit, 0, -1):
        if per_gpu % batch == 0:
            return {"batch_size": batch, "grad_accum": per_gpu // batch, "world_size": int(world_size)}
    raise ValueError("no per-GPU batch divides the share")


def training_argv(row, arm: str, output_root, *, world_size: int | None = None, timing: bool = False,
                  max_batch_per_gpu: int | None = None) -> list[str]:
    """Trainer argument list (without the program) for one arm of ``row``."""
    side = _arm_prefix(arm)
    name = run_name(row, arm) + ("-timing" if timing else "")
    batch, accum = int(row["batch_size"]), int(row["grad_accum"])
    if world_size is not None:
        plan = rebalance(row, world_size, max_batch_per_gpu=max_batch_per_gpu)
        batch, accum = plan["batch_size"], plan["grad_accum"]
    values = [
        ("--activation", row[f"{side}_activation"]), ("--optimizer", row[f"{side}_optimizer"]),
        ("--run-name", name), ("--fairness-contract", contract(row)),
        ("--experiment-identity", experiment_identity(row)),
        ("--dataset-name", row["dataset_name"]), ("--dataset-config", row["dataset_config"]),
        ("--dataset-revision", row["dataset_revision"]), ("--dataset-text-column", row["dataset_text_column"]),
        ("--train-split", row["train_split"]), ("--validation-split", row["validation_split"]),
        ("--train-skip-documents", row["train_skip_documents"]),
        ("--validation-skip-documents", row["validation_skip_documents"]),
        ("--train-skip-tokens", row["train_skip_tokens"]), ("--validation-skip-tokens", row["validation_skip_tokens"]),
        ("--cache-dir", row["cache_dir"]), ("--hf-cache", "experiments/cache/huggingface"),
        ("--output-dir", output_root), ("--max-train-tokens", row["max_train_tokens"]),
        ("--max-val-tokens", row["max_val_tokens"]), ("--steps", row["steps"]), ("--layers", row["layers"]),
        ("--d-model", row["d_model"]), ("--heads", row["heads"]), ("--ffn-dim", row["ffn_dim"]),
        ("--seq-len", row["seq_len"]), ("--batch-size", batch), ("--grad-accum", accum),
        ("--eval-interval", row["eval_interval"]), ("--eval-batches", row["eval_batches"]),
        ("--log-interval", row["log_interval"]), ("--seed", row["seed"]), ("--lr", row["lr"]),
        ("--min-lr", row["min_lr"]), ("--warmup-steps", row["warmup_steps"]),
        ("--weight-decay", row["weight_decay"]), ("--beta1", row["beta1"]), ("--beta2", row["beta2"]),
        ("--eps", row["eps"]), ("--grad-clip", row["grad_clip"]), ("--muon-momentum", row["muon_momentum"]),
        ("--muon-ns-steps", row["muon_ns_steps"]), ("--muon-adjust-lr-fn", row["muon_adjust_lr_fn"]),
        ("--init-std", row["init_std"]), ("--rational-init", row["rational_init"]),
        ("--post-rational-init", row["post_rational_init"]),
        ("--rational-group-size", row["rational_group_size"]),
        ("--rational-max-groups", row["rational_max_groups"]), ("--probe-batch-size", row["probe_batch_size"]),
        ("--matrix-spectrum-interval", row["matrix_spectrum_interval"]),
        ("--telemetry-rlb-stat-every", row["telemetry_rlb_stat_every"]), ("--sam-rho", row["sam_rho"]),
        ("--tokenizer", row["tokenizer"]), ("--tokenizer-revision", row["tokenizer_revision"]),
        ("--early-stop-min-step", 0), ("--early-stop-max-val-loss", 0.0), ("--early-stop-loss-increase", 0.0),
        ("--timing-guard-min-step", 0), ("--timing-guard-max-seconds-per-step", 0.0),
        ("--timing-guard-max-optimizer-step-seconds", 0.0),
    ]
    argv = []
    for flag, value in values:
        argv += [flag, str(value)]
    argv += ["--dataset-streaming" if row.get("dataset_streaming", True) else "--no-dataset-streaming",
             "--no-sam-adaptive"]
    if row["phase"] == PRIMARY_PHASE:
        argv.append("--no-grain-training-telemetry")
    return argv


def expected_args(row, arm: str, *, world_size: int | None = None, max_batch_per_gpu=None) -> dict[str, Any]:
    """Parsed-argument values a run of ``arm`` must carry (for :func:`verify_args`)."""
    side = _arm_prefix(arm)
    batch, accum = int(row["batch_size"]), int(row["grad_accum"])
    if world_size is not None:
        plan = rebalance(row, world_size, max_batch_per_gpu=max_batch_per_gpu)
        batch, accum = plan["batch_size"], plan["grad_accum"]
    keys = ("dataset_name", "dataset_config", "dataset_revision", "dataset_text_column", "train_split",
            "validation_split", "train_skip_documents", "validation_skip_documents", "train_skip_tokens",
            "validation_skip_tokens", "max_train_tokens", "max_val_tokens", "steps", "layers", "d_model",
            "heads", "ffn_dim", "seq_len", "eval_interval", "eval_batches", "log_interval", "seed", "lr",
            "min_lr", "warmup_steps", "weight_decay", "beta1", "beta2", "eps", "grad_clip", "muon_momentum",
            "muon_ns_steps", "muon_adjust_lr_fn", "init_std", "rational_init", "post_rational_init",
            "rational_group_size", "rational_max_groups", "probe_batch_size", "matrix_spectrum_interval",
            "telemetry_rlb_stat_every", "sam_rho", "sam_adaptive", "tokenizer", "tokenizer_revision")
    out = {k: row[k] for k in keys}
    out.update(activation=row[f"{side}_activation"], optimizer=row[f"{side}_optimizer"],
               fairness_contract=contract(row), experiment_identity=experiment_identity(row),
               dataset_streaming=bool(row.get("dataset_streaming", True)), batch_size=batch, grad_accum=accum,
               grain_training_telemetry=row["phase"] != PRIMARY_PHASE)
    return out


def verify_args(args, row, arm: str, **kw) -> None:
    bad = {k: {"observed": getattr(args, k, None), "required": v}
           for k, v in expected_args(row, arm, **kw).items() if getattr(args, k, None) != v}
    if bad:
        raise RuntimeError(f"full-transfer argument mismatch: {bad}")
