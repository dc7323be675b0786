"""Endpoint analysis of matrix rows (behaviour of experiments/protocol/analyze_row.py:1-468
and analyze_all.py:1-173; same ``tiller_matched_endpoint_result_v1`` result keys).

``endpoint_result`` audits one paired row - the control and candidate
trajectories (JSONL written by the trainer) - and summarises it:

* each arm has exactly one config record that matches the row
  (:func:`.monitor.audited_config`), a passed LR / weight-decay fairness audit
  at the row's base LR, minimum LR and weight decay (every group at scale 1,
  weight decay 0 or the row's), and evaluations at the screen step and at
  the endpoint;
* both arms trained on the same data in the same order (token-sample and
  batch-index fingerprints) under the same realised LR schedule (audited
  steps = row steps, equal trace digests);
* timing: end-to-end seconds from the launcher's wall-clock records
  (``rationalopt_process_wall_clock_v1``) when given, else the trainers'
  loop totals; hardware: when both arms' audits are given
  (:mod:`.hardware`), they must agree on GPU model, count and NVLink wiring;
* status ``complete`` when the candidate does not trail at the screen step,
  else ``invalid_not_interrupted`` (such a row should have been stopped).

``aggregate`` reduces many results per (suite, candidate optimizer): rows,
complete rows, candidate wins at the endpoint, mean and median leads and
time ratios, and the rows that pass the 1.20 / 1.05 time gates.

    python -m rational_optimizer_b200.protocol.analyze row --matrix M --index I --control C.jsonl \\
        --candidate K.jsonl --output RESULT.json [--control-wall-clock W] [--candidate-wall-clock W] \\
        [--control-hardware H] [--candidate-hardware H]
    python -m rational_optimizer_b200.protocol.analyze all RESULT.json ... --output SUMMARY.json
"""
from __future__ import annotations

import argparse
import hashlib
import json
import statistics
from pathlib import Path

from . import monitor as MON
from . import rows as R

SCHEMA = "tiller_matched_endpoint_result_v1"
SUMMARY_SCHEMA = "tiller_matched_endpoint_summary_v1"
HARDWARE_FIELDS = ("schema", "gpu_name", "count", "fully_connected", "nvlink")


def _sha(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def _summary(path) -> dict:
    found = [r for r in MON.records(path) if r.get("event") == "summary"]
    if len(found) != 1:
        raise RuntimeError(f"{path}: expected one summary record, found {len(found)}")
    return found[0]


def _fairness_problems(cfg: dict, row) -> dict:
    fair = cfg.get("optimizer_lr_wd_fairness") or {}
    bad = {}
    if fair.get("passed") is not True:
        bad["passed"] = fair.get("passed")
    for key, want in (("base_lr", row["lr"]), ("minimum_lr", row["min_lr"]),
                      ("base_weight_decay", row["weight_decay"])):
        if key in fair and float(fair[key]) != float(want):
            bad[key] = fair[key]
    for g in fair.get("groups", ()):
        if float(g.get("lr_scale", 1.0)) != 1.0:
            bad[f"group_{g.get('group_index')}_lr_scale"] = g.get("lr_scale")
        if float(g.get("weight_decay", 0.0)) not in (0.0, float(row["weight_decay"])):
            bad[f"group_{g.get('group_index')}_weight_decay"] = g.get("weight_decay")
    for name, value in (fair.get("internal_lr_wd_scalars") or {}).items():
        if float(value) != 1.0:
            bad[f"internal:{name}"] = value
    return bad


def audit_arm(path, row, arm: str, *, screen_step: int = MON.SCREEN_STEP):
    """(config, {step: val_loss}, summary) of one arm, or RuntimeError."""
    cfg = MON.audited_config(path, row, arm)
    bad = _fairness_problems(cfg, row)
    if bad:
        raise RuntimeError(f"{arm} learning-rate / weight-decay audit failed: {bad}")
    ev = MON.evals(path)
    need = {screen_step, int(row["steps"])}
    if not need <= set(ev):
        raise RuntimeError(f"{arm} lacks evaluations at steps {sorted(need - set(ev))}")
    return cfg, ev, _summary(path)


def _wall_seconds(path, arm: str) -> float:
    payload = json.loads(Path(path).read_text())
    if payload.get("schema") != "rationalopt_process_wall_clock_v1" or payload.get("return_code") != 0:
        raise RuntimeError(f"{path} is not a successful wall-clock record")
    if payload.get("arm") not in (arm, None) and not str(payload.get("arm", "")).endswith(arm):
        raise RuntimeError(f"{path} records arm {payload.get('arm')!r}, not {arm!r}")
    seconds = float(payload.get("elapsed_seconds", 0.0))
    if seconds <= 0.0:
        raise RuntimeError(f"{path} has no elapsed time")
    return seconds


def _hardware(path) -> dict:
    payload = json.loads(Path(path).read_text())
    if payload.get("passed") is not True:
        raise RuntimeError(f"hardware audit {path} did not pass")
    return payload


def endpoint_result(row, control, candidate, *, control_wall=None, candidate_wall=None, control_hw=None,
                    candidate_hw=None, screen_step: int = MON.SCREEN_STEP) -> dict:
    c_cfg, c_ev, c_sum = audit_arm(control, row, "control", screen_step=screen_step)
    k_cfg, k_ev, k_sum = audit_arm(candidate, row, "candidate", screen_step=screen_step)
    steps = int(row["steps"])
    schedule = {key: {"control": c_sum.get(key), "candidate": k_sum.get(key)}
                for key in ("realized_lr_audit_steps", "realized_lr_trace_sha256")}
    if (schedule["realized_lr_audit_steps"]["control"] != steps
            or schedule["realized_lr_audit_steps"]["candidate"] != steps
            or not schedule["realized_lr_trace_sha256"]["control"]
            or schedule["realized_lr_trace_sha256"]["control"] != schedule["realized_lr_trace_sha256"]["candidate"]):
        raise RuntimeError(f"the arms did not realise the same LR schedule: {schedule}")
    identity = {k: {"control": c_cfg.get(k), "candidate": k_cfg.get(k),
                    "equal": c_cfg.get(k) == k_cfg.get(k)} for k in MON.FINGERPRINTS}
    if not all(v["equal"] for v in identity.values()):
        raise RuntimeError(f"the arms did not see the same data in the same order: {identity}")
    if control_wall is not None and candidate_wall is not None:
        c_sec, k_sec = _wall_seconds(control_wall, "control"), _wall_seconds(candidate_wall, "candidate")
        scope = "end_to_end_process"
    else:
        c_sec, k_sec = float(c_sum["total_seconds"]), float(k_sum["total_seconds"])
        scope = "training_loop"
    hardware = None
    if control_hw is not None and candidate_hw is not None:
        a, b = _hardware(control_hw), _hardware(candidate_hw)
        hardware = {f: {"control": a.get(f), "candidate": b.get(f), "equal": a.get(f) == b.get(f)}
                    for f in HARDWARE_FIELDS}
        if not all(v["equal"] for v in hardware.values()):
            raise RuntimeError(f"the arms ran on different hardware standards: {hardware}")
    screen_lead = c_ev[screen_step] - k_ev[screen_step]
    end_lead = c_ev[steps] - k_ev[steps]
    ratio = k_sec / c_sec
    result = {
        "schema": SCHEMA, "status": "complete" if screen_lead >= 0.0 else "invalid_not_interrupted",
        "matrix_index": row["matrix_index"], "source_manifest_row_index": row["source_manifest_row_index"],
        "phase": row["phase"], "model": row["model"], "dataset": row["dataset"], "seed": row["seed"],
        "control": row["control_name"], "candidate": row["candidate_name"],
        "candidate_optimizer": row["candidate_optimizer"], "steps": steps, "screen_step": screen_step,
        "control_step1000_loss": c_ev[screen_step], "candidate_step1000_loss": k_ev[screen_step],
        "step1000_absolute_lead": screen_lead, "control_endpoint_loss": c_ev[steps],
        "candidate_endpoint_loss": k_ev[steps], "absolute_endpoint_lead": end_lead,
        "time_scope": scope, "exact_matched_hardware_end_to_end_total_time_ratio": ratio,
        "control_end_to_end_total_seconds": c_sec, "candidate_end_to_end_total_seconds": k_sec,
        "control_training_loop_total_seconds": float(c_sum["total_seconds"]),
        "candidate_training_loop_total_seconds": float(k_sum["total_seconds"]),
        "passes_discovery_1_20_time_gate": ratio <= 1.20, "passes_final_1_05_time_gate": ratio <= 1.05,
        "lr_wd_and_all_shared_argparse_hyperparameters_identical": True,
        "realized_lr_schedule_identity": schedule, "data_and_order_identity": identity,
        "matched_hardware_standard": hardware,
        "control_jsonl": {"path": str(control), "sha256": _sha(control)},
        "candidate_jsonl": {"path": str(candidate), "sha256": _sha(candidate)},
    }
    return result


def write_result(path, result: dict) -> None:
    MON.write_screen(path, result)  # atomic JSON + ".sha256" side file


def aggregate(results) -> dict:
    """Per (suite, candidate optimizer) totals of many endpoint results."""
    cells = {}
    for r in results:
        if r.get("schema") != SCHEMA:
            raise RuntimeError(f"not an endpoint result: {r.get('schema')!r}")
        cells.setdefault((r["phase"], r["candidate_optimizer"]), []).append(r)
    groups = []
    for (phase, opt), rs in sorted(cells.items()):
        done = [r for r in rs if r["status"] == "complete"]
        leads = [r["absolute_endpoint_lead"] for r in done]
        ratios = [r["exact_matched_hardware_end_to_end_total_time_ratio"] for r in done]
        groups.append({
            "phase": phase, "candidate_optimizer": opt, "rows": len(rs), "complete_rows": len(done),
            "candidate_endpoint_wins": sum(v > 0.0 for v in leads),
            "mean_absolute_endpoint_lead": statistics.fmean(leads) if leads else None,
            "median_absolute_endpoint_lead": statistics.median(leads) if leads else None,
            "mean_time_ratio": statistics.fmean(ratios) if ratios else None,
            "median_time_ratio": statistics.median(ratios) if ratios else None,
            "passes_1_20_time_gate": sum(v <= 1.20 for v in ratios),
            "passes_1_05_time_gate": sum(v <= 1.05 for v in ratios),
        })
    return {"schema": SUMMARY_SCHEMA, "results": len(results), "groups": groups}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    one = sub.add_parser("row")
    one.add_argument("--matrix", required=True)
    one.add_argument("--index", type=int, required=True)
    one.add_argument("--control", type=Path, required=True)
    one.add_argument("--candidate", type=Path, required=True)
    one.add_argument("--output", type=Path, required=True)
    for name in ("control-wall-clock", "candidate-wall-clock", "control-hardware", "candidate-hardware"):
        one.add_argument(f"--{name}", type=Path)
    one.add_argument("--screen-step", type=int, default=MON.SCREEN_STEP)
    many = sub.add_parser("all")
    many.add_argument("results", nargs="+", type=Path)
    many.add_argument("--output", type=Path, required=True)
    a = ap.parse_args(argv)
    if a.cmd == "row":
        row = R.row_at(R.load_matrix(a.matrix), a.index)
        result = endpoint_result(row, a.control, a.candidate, control_wall=a.control_wall_clock,
                                 candidate_wall=a.candidate_wall_clock, control_hw=a.control_hardware,
                                 candidate_hw=a.candidate_hardware, screen_step=a.screen_step)
        write_result(a.output, result)
        print(json.dumps(result, sort_keys=True))
        return 0 if result["status"] == "complete" else 4
    summary = aggregate([json.loads(p.read_text()) for p in a.results])
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n")
    print(json.dumps(summary, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
