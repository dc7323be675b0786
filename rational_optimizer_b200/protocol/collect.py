"""Per-row results of a matrix campaign from the arms' JSONL trajectories.

    python -m rational_optimizer_b200.protocol.collect --matrix PATH --output-root RUNS --out results.csv

For every matrix row: the control and candidate endpoint and step-1,000
validation losses, the candidate's lead (control minus candidate), both
runs' training-loop seconds and step times, and a status
(``complete`` / ``running`` / ``missing`` / ``failed_negative_step1000`` /
``retryable_execution_failure``, the last two from the launcher's failure
record), in the spirit of the reference's collect_results/analyze_row
(experiments/protocol/collect_results.py, analyze_row.py).  A matched
control published with the row (``matched_control``) is used when the
control arm was not re-run here.
"""
from __future__ import annotations

import argparse
import csv
import json
import sys
from pathlib import Path

from . import rows as R
from .monitor import SCREEN_STEP, records

COLUMNS = ("matrix_index", "phase", "model", "dataset", "seed", "candidate_optimizer", "status",
           "control_source", "control_final_val_loss", "control_step1000_val_loss",
           "candidate_final_val_loss", "candidate_step1000_val_loss", "candidate_final_lead",
           "candidate_step1000_lead", "control_total_seconds", "candidate_total_seconds",
           "control_mean_seconds_per_step", "candidate_mean_seconds_per_step", "candidate_completed_steps")


def _summary(path: Path):
    if not path.is_file():
        return None
    recs = records(path)
    evals = {int(r["step"]): float(r["val_loss"]) for r in recs if r.get("event") == "eval"}
    summary = next((r for r in reversed(recs) if r.get("event") == "summary"), None)
    stopped = next((r for r in recs if r.get("event") == "stopped_early"), None)
    final = evals[max(evals)] if evals else None
    return {"evals": evals, "summary": summary, "stopped": stopped, "final": final}


def collect_row(row, output_root: Path) -> dict:
    out = {k: row.get(k) for k in ("matrix_index", "phase", "model", "dataset", "seed", "candidate_optimizer")}
    ctl = _summary(R.jsonl_path(row, "control", output_root))
    cand = _summary(R.jsonl_path(row, "candidate", output_root))
    if ctl is not None and ctl["summary"] is not None:
        out.update(control_source="rerun", control_final_val_loss=ctl["final"],
                   control_step1000_val_loss=ctl["evals"].get(SCREEN_STEP),
                   control_total_seconds=ctl["summary"]["total_seconds"],
                   control_mean_seconds_per_step=ctl["summary"]["mean_seconds_per_step"])
    elif isinstance(row.get("matched_control"), dict):
        mc = row["matched_control"]
        out.update(control_source=mc.get("source_result"), control_final_val_loss=mc.get("endpoint_validation_loss"),
                   control_step1000_val_loss=mc.get("step1000_validation_loss"),
                   control_total_seconds=mc.get("total_seconds"))
    failure = Path(output_root) / f"{R.run_name(row, 'candidate')}.failure.json"
    if cand is None:
        out["status"] = "missing"
    elif cand["summary"] is None:
        out["status"] = "running"
    else:
        s = cand["summary"]
        out.update(status="complete" if not s.get("stopped_early") else f"stopped_{s.get('stop_reason')}",
                   candidate_final_val_loss=cand["final"],
                   candidate_step1000_val_loss=cand["evals"].get(SCREEN_STEP),
                   candidate_total_seconds=s["total_seconds"],
                   candidate_mean_seconds_per_step=s["mean_seconds_per_step"],
                   candidate_completed_steps=s["completed_steps"])
    if failure.is_file():
        out["status"] = json.loads(failure.read_text()).get("status", "retryable_execution_failure")
    for kind, a, b in (("final", "control_final_val_loss", "candidate_final_val_loss"),
                       ("step1000", "control_step1000_val_loss", "candidate_step1000_val_loss")):
        if out.get(a) is not None and out.get(b) is not None:
            out[f"candidate_{kind}_lead"] = float(out[a]) - float(out[b])
    return {k: out.get(k) for k in COLUMNS}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--matrix", required=True)
    ap.add_argument("--output-root", required=True, type=Path)
    ap.add_argument("--out", required=True, type=Path)
    a = ap.parse_args(argv)
    payload = R.load_matrix(a.matrix)
    table = [collect_row(row, a.output_root) for row in payload["rows"]]
    a.out.parent.mkdir(parents=True, exist_ok=True)
    with a.out.open("w", newline="", encoding="utf-8") as fh:
        w = csv.DictWriter(fh, fieldnames=list(COLUMNS), lineterminator="\n")
        w.writeheader()
        w.writerows(table)
    print(json.dumps({"rows": len(table), "complete": sum(r["status"] == "complete" for r in table)}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
