"""Evaluation matrix: paired control/candidate rows built from the activation x
optimizer manifest (behaviour of experiments/protocol/build_matrix.py:1-274;
same ``tiller_evaluation_matrix_v1`` payload, read by :mod:`.rows`).

The manifest (``activation_optimizer_manifest.csv``) lists one training
configuration per row.  The matrix takes the baseline row of every
(suite, dataset, seed) cell - ``silu_adamw`` in the 12-layer 100M suite,
``silu_muon`` in the 12-layer 300M and 18-layer 100M suites - and pairs it
with the TILLER candidate (``tiller_v1``); the 18-layer suite also gets the
two-stage TILLER -> Muon candidate.  A row's ``matched_control`` is the
published control run of the same cell from the results tables
(``<results>/<optimizer>/runs.csv``), or a ``pending`` stub.

    python -m rational_optimizer_b200.protocol.matrix --manifest M.csv --results RESULTS --output matrix.json
"""
from __future__ import annotations

import argparse
import csv
import hashlib
import json
from pathlib import Path

EXACT = "tiller_v1"
TWO_STAGE = "tiller_then_muon_v1"
SUITES = {
    # suite: (model, control optimizer folder, training tokens, steps)
    "12l_768d_100m_tokens_3050_steps": ("12l_768d", "adamw", 100_000_000, 3_050),
    "12l_768d_300m_tokens_9150_steps": ("12l_768d", "muon", 300_000_000, 9_150),
    "18l_1024d_100m_tokens_3050_steps": ("18l_1024d", "muon", 100_000_000, 3_050),
}
TWO_STAGE_SUITE = "18l_1024d_100m_tokens_3050_steps"
DATASETS = {"dclm", "fineweb_edu", "fineweb", "dolma_sample", "c4_en"}
SEEDS = {1337, 2027, 3407}
DEFAULT_TIMING = "exclusive allocation; one 8x B200 node (NVSwitch), NCCL plus in-kernel peer-memory collectives"


def _bool(text: str) -> bool:
    low = text.strip().lower()
    if low not in ("true", "false"):
        raise ValueError(f"expected true/false, found {text!r}")
    return low == "true"


def _opt_float(text: str):
    return None if text == "" else float(text)


# matrix key <- (manifest column, converter); the order is the payload's key order
FIELDS = (
    ("phase", "phase", str), ("model", "model", str), ("dataset", "dataset", str),
    ("dataset_name", "dataset_name", str), ("dataset_config", "dataset_config", str),
    ("dataset_revision", "dataset_revision", str), ("dataset_streaming", "dataset_streaming", _bool),
    ("dataset_text_column", "text_column", str), ("train_split", "train_split", str),
    ("validation_split", "val_split", str), ("train_skip_documents", "train_skip_documents", int),
    ("validation_skip_documents", "validation_skip_documents", int),
    ("train_skip_tokens", "train_skip_tokens", int), ("validation_skip_tokens", "val_skip_tokens", int),
    ("cache_dir", "cache_dir", str), ("max_train_tokens", "train_tokens", int),
    ("max_val_tokens", "val_tokens", int), ("steps", "steps", int), ("layers", "layers", int),
    ("d_model", "d_model", int), ("heads", "heads", int), ("ffn_dim", "ffn_dim", int),
    ("seq_len", "seq_len", int), ("batch_size", "batch_size", int), ("grad_accum", "grad_accum", int),
    ("global_tokens_per_step", "global_tokens_per_step", int), ("eval_interval", "eval_interval", int),
    ("eval_batches", "eval_batches", int), ("log_interval", "log_interval", int), ("seed", "seed", int),
    ("lr", "lr", float), ("min_lr", "min_lr", float), ("warmup_steps", "warmup_steps", int),
    ("weight_decay", "weight_decay", float), ("beta1", "beta1", float), ("beta2", "beta2", float),
    ("eps", "eps", float), ("grad_clip", "grad_clip", float), ("muon_momentum", "muon_momentum", float),
    ("muon_ns_steps", "muon_ns_steps", int), ("muon_adjust_lr_fn", "muon_adjust_lr_fn", str),
    ("init_std", "init_std", float), ("rational_init", "rational_init", str),
    ("post_rational_init", "post_rational_init", str), ("rational_group_size", "rational_group_size", int),
    ("rational_max_groups", "rational_max_groups", int), ("probe_batch_size", "probe_batch_size", int),
    ("matrix_spectrum_interval", "matrix_spectrum_interval", int),
    ("telemetry_rlb_stat_every", "telemetry_rlb_stat_every", int), ("sam_rho", "sam_rho", float),
    ("sam_adaptive", "sam_adaptive", _bool), ("tokenizer", "tokenizer", str),
    ("tokenizer_revision", "tokenizer_revision", str),
)


def file_sha256(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def read_manifest(path) -> list[dict[str, str]]:
    with Path(path).open(newline="") as fh:
        return list(csv.DictReader(fh))


def baseline_rows(manifest: list[dict[str, str]]) -> list[dict[str, str]]:
    """The control configuration of every (suite, dataset, seed) cell, in manifest order."""
    wanted = {suite: f"silu_{folder}" for suite, (_, folder, _, _) in SUITES.items()}
    picked = [r for r in manifest if wanted.get(r["phase"]) == r["method"]]
    for suite in SUITES:
        rows = [r for r in picked if r["phase"] == suite]
        cells = {(r["dataset"], int(r["seed"])) for r in rows}
        if {d for d, _ in cells} != DATASETS or {s for _, s in cells} != SEEDS or len(rows) != 15:
            raise ValueError(f"{suite}: expected the 5 datasets x 3 seeds, found {sorted(cells)}")
    return picked


def matched_controls(results_root) -> dict[tuple[str, str, int], dict]:
    """(suite, dataset, seed) -> the published control run (``<results>/<optimizer>/runs.csv``)."""
    out = {}
    root = Path(results_root)
    for suite, (model, folder, tokens, steps) in SUITES.items():
        table = root / folder / "runs.csv"
        with table.open(newline="") as fh:
            for r in csv.DictReader(fh):
                if (r["model_scale"], r["source_phase"], int(r["train_tokens"]), int(r["steps_required"]),
                        r["activation"], r["optimizer"]) != (model, suite, tokens, steps, "silu", folder):
                    continue
                key = (suite, r["dataset"], int(r["seed"]))
                if key in out:
                    raise ValueError(f"two published control runs for {key}")
                out[key] = {
                    "source_result": f"experiments/results/{folder}/runs.csv",
                    "source_run_index": int(r["run_index"]), "status": r["status"],
                    "endpoint_validation_loss": _opt_float(r["final_validation_loss"]),
                    "step1000_validation_loss": _opt_float(r["step1000_validation_loss"]),
                    "time_scope": r["time_scope"] or None, "total_seconds": _opt_float(r["total_seconds"]),
                }
    return out


def matrix_row(index: int, src: dict[str, str], controls, candidate: str, timing: str) -> dict:
    if candidate not in (EXACT, TWO_STAGE):
        raise ValueError(f"candidate optimizer {candidate!r} is not part of the matrix")
    if candidate == TWO_STAGE and src["phase"] != TWO_STAGE_SUITE:
        raise ValueError(f"the two-stage candidate runs only in {TWO_STAGE_SUITE}")
    control_opt = SUITES[src["phase"]][1]
    control = controls.get((src["phase"], src["dataset"], int(src["seed"]))) or {
        "source_result": f"experiments/results/{control_opt}/runs.csv", "source_run_index": None,
        "status": "pending", "endpoint_validation_loss": None, "step1000_validation_loss": None,
        "time_scope": None, "total_seconds": None}
    row = {"matrix_index": index, "source_manifest_row_index": int(src["row_index"]),
           "source_manifest_row_id": src["row_id"]}
    row.update({key: conv(src[col]) for key, col, conv in FIELDS})
    row.update({
        "control_activation": "silu", "control_optimizer": control_opt,
        "control_name": "SwiGLU+AdamW" if control_opt == "adamw" else "SwiGLU+Muon",
        "candidate_activation": "rlb_fused_global_rational", "candidate_optimizer": candidate,
        "candidate_name": "TILLER" if candidate == EXACT else "TILLER→Muon",
        "quality_action": "selected_method_endpoint", "timing_condition": timing,
        "matched_control": control,
    })
    if candidate == TWO_STAGE:
        row.update(switch_after_step=1_000, optimizer_state_transition="preserve_compatible_state",
                   learning_rate_schedule="single_full_horizon_cosine")
    return row


def build_matrix(manifest_path, results_root, *, timing=DEFAULT_TIMING,
                 manifest_name="experiments/protocol/activation_optimizer_manifest.csv") -> dict:
    controls = matched_controls(results_root)
    base = baseline_rows(read_manifest(manifest_path))
    rows = [matrix_row(i, r, controls, EXACT, timing) for i, r in enumerate(base)]
    rows += [matrix_row(len(rows) + k, r, controls, TWO_STAGE, timing)
             for k, r in enumerate(r for r in base if r["phase"] == TWO_STAGE_SUITE)]
    in_suite = lambda s: sum(r["phase"] == s for r in rows)  # noqa: E731
    return {
        "schema": "tiller_evaluation_matrix_v1",
        "objective": "TILLER and TILLER-to-Muon evaluation across the published model and token-budget suites",
        "source_manifest": manifest_name, "source_manifest_sha256": file_sha256(manifest_path),
        "matrix_rows": len(rows),
        "12l_100m_suite_rows": in_suite("12l_768d_100m_tokens_3050_steps"),
        "12l_300m_suite_rows": in_suite("12l_768d_300m_tokens_9150_steps"),
        "18l_100m_suite_rows": in_suite(TWO_STAGE_SUITE),
        "18l_100m_full_tiller_rows": sum(r["phase"] == TWO_STAGE_SUITE and r["candidate_optimizer"] == EXACT
                                         for r in rows),
        "18l_100m_tiller_then_muon_rows": sum(r["candidate_optimizer"] == TWO_STAGE for r in rows),
        "rows": rows,
    }


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--manifest", type=Path, required=True)
    ap.add_argument("--results", type=Path, required=True, help="root of <optimizer>/runs.csv tables")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--timing-condition", default=DEFAULT_TIMING)
    a = ap.parse_args(argv)
    payload = build_matrix(a.manifest, a.results, timing=a.timing_condition)
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n")
    print(f"wrote {a.output} ({payload['matrix_rows']} rows)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
