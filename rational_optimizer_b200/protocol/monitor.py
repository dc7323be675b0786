"""Step-1,000 paired screen: stop a candidate that trails its control.

    python -m rational_optimizer_b200.protocol.monitor --matrix PATH --index I \\
        --control CONTROL.jsonl --candidate CANDIDATE.jsonl --output SCREEN.json

Exit codes (reference experiments/protocol/monitor_step1000.py:94-138):
0 - the candidate's step-1,000 validation loss is not above the control's
(``pass_nonnegative``); 3 - the candidate has no config or no step-1,000
evaluation yet (keep training); 4 - the candidate trails
(``failed_negative_interrupted``).  Both trajectories must have exactly one
config record matching the row, and identical data and order fingerprints.
The screen is written atomically with a ``.sha256`` side file.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

from . import rows as R

SCREEN_STEP = 1000
FINGERPRINTS = ("train_token_sample_sha256", "val_token_sample_sha256", "first_batch_index_sha256",
                "validation_index_sha256")


class PendingCandidate(Exception):
    """The candidate has not reached the screen yet (exit 3)."""


def records(path: Path):
    return [json.loads(l) for l in Path(path).read_text(encoding="utf-8").splitlines() if l.strip()]


def evals(path: Path) -> dict:
    return {int(r["step"]): float(r["val_loss"]) for r in records(path) if r.get("event") == "eval"}


def audited_config(path: Path, row, arm: str) -> dict:
    configs = [r for r in records(path) if r.get("event") == "config"]
    if len(configs) != 1:
        if arm == "candidate" and not configs:
            raise PendingCandidate()
        raise RuntimeError(f"{arm} must contain exactly one config record")
    cfg = configs[0]
    side = "control" if arm == "control" else "candidate"
    expected = {"activation": row[f"{side}_activation"], "optimizer": row[f"{side}_optimizer"],
                "dataset": row["dataset_name"], "dataset_config": row["dataset_config"],
                "dataset_revision": row["dataset_revision"], "tokenizer": row["tokenizer"],
                "tokenizer_revision": row["tokenizer_revision"], "steps": row["steps"], "seed": row["seed"],
                "train_tokens": row["max_train_tokens"], "val_tokens": row["max_val_tokens"]}
    if arm == "candidate":
        expected["experiment_identity"] = R.experiment_identity(row)
    bad = {k: {"observed": cfg.get(k), "required": v} for k, v in expected.items() if cfg.get(k) != v}
    if arm == "candidate":
        ident = cfg.get("tiller_experiment_identity") or {}
        for k in ("matrix_index", "source_manifest_row_index", "source_manifest_row_id"):
            if ident.get(k) != row[k]:
                bad[f"matrix_identity.{k}"] = {"observed": ident.get(k), "required": row[k]}
        if ident.get("passed") is not True:
            bad["matrix_identity.passed"] = ident.get("passed")
    if bad:
        raise RuntimeError(f"{arm} configuration mismatch: {bad}")
    return cfg


def write_screen(path: Path, payload: dict) -> None:
    path = Path(path)
    text = json.dumps(payload, indent=2, sort_keys=True) + "\n"
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(text)
    tmp.replace(path)
    path.with_suffix(path.suffix + ".sha256").write_text(
        f"{hashlib.sha256(path.read_bytes()).hexdigest()}  {path.name}\n")


def screen(row, control: Path, candidate: Path, output: Path) -> int:
    control_cfg = audited_config(control, row, "control")
    c_evals = evals(control)
    if SCREEN_STEP not in c_evals:
        raise RuntimeError("paired control lacks step 1,000")
    try:
        cand_cfg = audited_config(candidate, row, "candidate")
    except PendingCandidate:
        return 3
    for key in FINGERPRINTS:
        if control_cfg.get(key) != cand_cfg.get(key):
            raise RuntimeError(f"paired data/order identity differs at {key}")
    k_evals = evals(candidate)
    if SCREEN_STEP not in k_evals:
        return 3
    lead = c_evals[SCREEN_STEP] - k_evals[SCREEN_STEP]
    payload = {
        "schema": "tiller_step1000_screen_v1", "matrix_index": row["matrix_index"], "phase": row["phase"],
        "model": row["model"], "dataset": row["dataset"], "seed": row["seed"], "control": row["control_name"],
        "candidate": row["candidate_name"], "candidate_optimizer": row["candidate_optimizer"],
        "control_step1000_loss": c_evals[SCREEN_STEP], "candidate_step1000_loss": k_evals[SCREEN_STEP],
        "candidate_step1000_lead": lead,
        "status": "pass_nonnegative" if lead >= 0.0 else "failed_negative_interrupted",
    }
    write_screen(output, payload)
    print(json.dumps(payload, sort_keys=True))
    return 0 if lead >= 0.0 else 4


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--matrix", required=True)
    ap.add_argument("--index", required=True, type=int)
    ap.add_argument("--control", required=True, type=Path)
    ap.add_argument("--candidate", required=True, type=Path)
    ap.add_argument("--output", required=True, type=Path)
    a = ap.parse_args(argv)
    return screen(R.row_at(R.load_matrix(a.matrix), a.index), a.control, a.candidate, a.output)


if __name__ == "__main__":
    sys.exit(main())
