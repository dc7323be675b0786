"""Run one activation x optimizer manifest row with the package's trainer
(behaviour of experiments/protocol/run_activation_row.py:1-305).

A row's trajectory goes to ``<output-root>/<phase>/<dataset>/<row_id>/<activation>.jsonl``
beside its process wall clock (``.wall_clock.json``, written by
:func:`.launch.run_timed`).  Before launching:

* a trajectory that already reached the row's endpoint is accepted (nothing
  runs) only when its config record carries this manifest's and this source
  freeze's identity (``RATIONALOPT_SOURCE_*``: manifest and row SHA-256, row id
  and index, freeze SHA-256), the row's activation / optimizer / data /
  tokenizer / geometry / hyper-parameters, ``experiment_identity == "none"``
  and a passed exact LR / weight-decay audit at the row's scalars;
* any other existing trajectory is an error unless ``--force``, which
  archives it (``<stem>.superseded-<sha12>.jsonl``, wall clock alongside).

The published rows were laid out for 4 GPUs; ``--gpus`` re-derives the
per-GPU batch and accumulation at the same global tokens per step
(:func:`.rows.rebalance`).  The trainer receives the row's flags unchanged
otherwise.

    python -m rational_optimizer_b200.protocol.sweep --manifest M.csv --row-index I \\
        --output-root runs/activation_optimizer [--gpus 8] [--force] [--dry-run]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shlex
import sys
from pathlib import Path

from . import launch as LA
from . import rows as R

EXACT_LR_WD_CONTRACT = R.EXACT_LR_WD_CONTRACT

# trainer flag <- manifest column, in the order the trainer documents them
VALUE_FLAGS = (
    ("--train-skip-documents", "train_skip_documents"), ("--validation-skip-documents", "validation_skip_documents"),
    ("--train-skip-tokens", "train_skip_tokens"), ("--validation-skip-tokens", "val_skip_tokens"),
    ("--max-train-tokens", "train_tokens"), ("--max-val-tokens", "val_tokens"), ("--steps", "steps"),
    ("--layers", "layers"), ("--d-model", "d_model"), ("--heads", "heads"), ("--ffn-dim", "ffn_dim"),
    ("--seq-len", "seq_len"), ("--batch-size", "batch_size"), ("--grad-accum", "grad_accum"),
    ("--eval-interval", "eval_interval"), ("--eval-batches", "eval_batches"), ("--log-interval", "log_interval"),
    ("--seed", "seed"), ("--lr", "lr"), ("--min-lr", "min_lr"), ("--warmup-steps", "warmup_steps"),
    ("--weight-decay", "weight_decay"), ("--beta1", "beta1"), ("--beta2", "beta2"), ("--eps", "eps"),
    ("--grad-clip", "grad_clip"), ("--muon-momentum", "muon_momentum"), ("--muon-ns-steps", "muon_ns_steps"),
    ("--muon-adjust-lr-fn", "muon_adjust_lr_fn"), ("--init-std", "init_std"), ("--rational-init", "rational_init"),
    ("--post-rational-init", "post_rational_init"), ("--rational-group-size", "rational_group_size"),
    ("--rational-max-groups", "rational_max_groups"), ("--probe-batch-size", "probe_batch_size"),
    ("--matrix-spectrum-interval", "matrix_spectrum_interval"),
    ("--telemetry-rlb-stat-every", "telemetry_rlb_stat_every"), ("--sam-rho", "sam_rho"),
    ("--tokenizer", "tokenizer"), ("--tokenizer-revision", "tokenizer_revision"),
)
EXACT_FIELDS = (("activation", "activation"), ("optimizer", "optimizer"), ("dataset", "dataset_name"),
                ("dataset_config", "dataset_config"), ("dataset_revision", "dataset_revision"),
                ("tokenizer", "tokenizer"), ("tokenizer_revision", "tokenizer_revision"))
INTEGER_FIELDS = (("train_tokens", "train_tokens"), ("val_tokens", "val_tokens"), ("steps", "steps"),
                  ("layers", "layers"), ("d_model", "d_model"), ("heads", "heads"), ("ffn_dim", "ffn_dim"),
                  ("global_tokens_per_step", "global_tokens_per_step"), ("warmup_steps", "warmup_steps"))
NUMBER_FIELDS = (("optimizer_lr", "lr"), ("optimizer_min_lr", "min_lr"),
                 ("optimizer_weight_decay", "weight_decay"), ("optimizer_beta1", "beta1"),
                 ("optimizer_beta2", "beta2"), ("optimizer_eps", "eps"), ("grad_clip", "grad_clip"),
                 ("init_std", "init_std"))


def sha256_file(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def row_sha256(row: dict) -> str:
    return hashlib.sha256(json.dumps(row, sort_keys=True, separators=(",", ":"),
                                     ensure_ascii=True).encode("utf-8")).hexdigest()


def source_identity(manifest, row: dict, freeze) -> dict[str, str]:
    """The identity a run of ``row`` records (environment ``RATIONALOPT_<KEY>``)."""
    if not Path(freeze).is_file():
        raise RuntimeError(f"source freeze is missing: {freeze}")
    return {"source_manifest_sha256": sha256_file(manifest), "source_manifest_row_sha256": row_sha256(row),
            "source_manifest_row_id": row["row_id"], "source_manifest_row_index": row["row_index"],
            "source_freeze_sha256": sha256_file(freeze)}


def trajectory_path(row: dict, output_root) -> Path:
    return Path(output_root) / row["phase"] / row["dataset"] / row["row_id"] / f"{row['activation']}.jsonl"


def training_argv(row: dict, output_root, *, gpus: int | None = None) -> list[str]:
    """Trainer flags of one manifest row (the per-GPU batch re-derived for ``gpus``)."""
    values = dict(row)
    if gpus is not None:
        values.update({k: str(v) for k, v in R.rebalance(row, gpus).items() if k != "world_size"})
    argv = ["--activation", row["activation"], "--optimizer", row["optimizer"],
            "--fairness-contract", EXACT_LR_WD_CONTRACT, "--run-name", row["row_id"],
            "--dataset-name", row["dataset_name"], "--dataset-config", row["dataset_config"],
            "--dataset-revision", row["dataset_revision"], "--dataset-text-column", row["text_column"],
            "--train-split", row["train_split"], "--validation-split", row["val_split"],
            "--cache-dir", row["cache_dir"],
            "--output-dir", str(Path(output_root) / row["phase"] / row["dataset"])]
    argv.append("--dataset-streaming" if row["dataset_streaming"].lower() == "true" else "--no-dataset-streaming")
    argv.append("--sam-adaptive" if row["sam_adaptive"].lower() == "true" else "--no-sam-adaptive")
    for flag, column in VALUE_FLAGS:
        argv += [flag, str(values[column])]
    return argv + shlex.split(row.get("extra_args", ""))


def _final_step(records) -> int | None:
    for r in reversed(records):
        if r.get("event") == "summary":
            return int(r.get("completed_steps", -1))
    return None


def matches(path, row: dict, identity: dict) -> bool:
    """True when ``path`` holds a finished trajectory of exactly this row and source."""
    from .results import read_jsonl
    recs = read_jsonl(path)
    if _final_step(recs) != int(row["steps"]):
        return False
    configs = [r for r in recs if r.get("event") == "config"]
    if len(configs) != 1:
        return False
    cfg = configs[0]
    if any(str(cfg.get(k, "")) != v for k, v in identity.items()) or cfg.get("experiment_identity") != "none":
        return False
    if any(str(cfg.get(k, "")) != row[c] for k, c in EXACT_FIELDS):
        return False
    try:
        if any(int(cfg.get(k, -1)) != int(row[c]) for k, c in INTEGER_FIELDS):
            return False
        if any(float(cfg.get(k, "nan")) != float(row[c]) for k, c in NUMBER_FIELDS):
            return False
        fair = cfg.get("optimizer_lr_wd_fairness")
        return (isinstance(fair, dict) and fair.get("contract") == EXACT_LR_WD_CONTRACT
                and fair.get("passed") is True
                and float(fair.get("base_lr", "nan")) == float(row["lr"])
                and float(fair.get("minimum_lr", "nan")) == float(row["min_lr"])
                and float(fair.get("base_weight_decay", "nan")) == float(row["weight_decay"]))
    except (TypeError, ValueError):
        return False


def archive(path) -> Path:
    """Move an existing trajectory (and its wall clock) aside; returns the new path."""
    path = Path(path)
    target = path.with_name(f"{path.stem}.superseded-{sha256_file(path)[:12]}{path.suffix}")
    if target.exists():
        raise RuntimeError(f"an archive already exists: {target}")
    path.rename(target)
    clock = path.with_suffix(".wall_clock.json")
    if clock.exists():
        clock.rename(target.with_suffix(".wall_clock.json"))
    return target


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--manifest", type=Path, required=True)
    ap.add_argument("--row-index", type=int, required=True)
    ap.add_argument("--output-root", type=Path, default=Path("runs/activation_optimizer"))
    ap.add_argument("--freeze", type=Path, help="SOURCE_FREEZE.sha256 (default: beside the manifest)")
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--port", type=int, default=29511)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--dry-run", action="store_true", help="print the command, run nothing")
    a = ap.parse_args(argv)
    row = R.load_manifest(a.manifest)[a.row_index]
    freeze = a.freeze or a.manifest.with_name("SOURCE_FREEZE.sha256")
    identity = source_identity(a.manifest, row, freeze)
    path = trajectory_path(row, a.output_root)
    if path.is_file():
        if matches(path, row, identity) and not a.force:
            print(json.dumps({"row": a.row_index, "status": "complete", "path": str(path)}))
            return 0
        if not a.force:
            raise RuntimeError(f"existing trajectory does not match the current row / source identity: {path}")
        archive(path)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={a.gpus}",
           "--master-addr=127.0.0.1", f"--master-port={a.port}", "-m", "rational_optimizer_b200.train",
           *training_argv(row, a.output_root, gpus=a.gpus)]
    if a.dry_run:
        print(json.dumps({"row": a.row_index, "command": cmd, "identity": identity}))
        return 0
    os.environ.update({f"RATIONALOPT_{k.upper()}": v for k, v in identity.items()})
    path.parent.mkdir(parents=True, exist_ok=True)
    rc = LA.run_timed(cmd, path.with_suffix(".wall_clock.json"), row["method"])
    if rc != 0:
        return rc
    from .results import read_jsonl
    if _final_step(read_jsonl(path)) != int(row["steps"]):
        raise RuntimeError(f"the row did not reach its endpoint: {path}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
