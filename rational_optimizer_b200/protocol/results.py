"""Published result tables of a campaign: ``runs.csv``, ``summary.csv`` and
``checkpoints.csv`` per optimizer (behaviour of
experiments/protocol/collect_results.py:20-146 for the column sets, :166-358 for
one run's record, :359-393 for control pairing, :705-808 for the per-cell
summary; the tables under experiments/results/ are the published format).

Sources:

* the activation x optimizer manifest (one CSV line per run) with each run's
  trainer JSONL at ``<runs>/<phase>/<dataset>/<row_id>/<activation>.jsonl``;
* the TILLER matrix (``matrix.json``) with each candidate's JSONL at
  ``<runs>/<phase>-<dataset>-seed<seed>-<method>/<activation>.jsonl`` and, when
  analysed, ``<analysis>/row-NN/RESULT.json`` (an endpoint result,
  ``tiller_matched_endpoint_result_v1``) and a step-1,000 screen.

A run is ``pending`` (no JSONL), ``incomplete``, ``stopped_early``,
``non_finite`` (endpoint evaluated, loss not finite) or ``complete``.  Time is
the launcher's process wall clock (``rationalopt_process_wall_clock_v1``
beside the JSONL or under the run root) when it records a successful exit,
else the trainer's loop total; ``time_scope`` says which.  A candidate with a
GRAIN activation is paired with the SwiGLU run of the same suite, dataset,
seed and optimizer, a TILLER candidate with the manifest run its matrix row
names (or the control published with the row): lead = control loss minus
candidate loss; the time ratio only when both times are process times.

The summary groups runs by (model, dataset, tokens, steps, activation,
optimizer, method) and reports seed means and sample standard deviations of
endpoint loss, matched-control loss, lead, time ratio, seconds and
throughput, with a cell status (``non_finite`` > ``stopped_early`` >
``pending`` / ``incomplete`` > ``endpoint_loss_unavailable`` > ``complete``).

    python -m rational_optimizer_b200.protocol.results --manifest M.csv --runs RUNS \\
        [--matrix matrix.json --tiller-runs R --tiller-analysis A] --output-root results/ [--include-pending]
"""
from __future__ import annotations

import argparse
import csv
import hashlib
import json
import math
import statistics
from collections import defaultdict
from pathlib import Path
from typing import Any, Iterable

from . import rows as R

GRAIN = "rlb_fused_global_rational"
SWIGLU = "silu"
PREFLIGHT = "12l_768d_preflight_2621440_tokens_80_steps"
SCREEN_STEP = 1000
WALL_CLOCK_SCHEMA = "rationalopt_process_wall_clock_v1"

ACTIVATION_NAMES = {SWIGLU: "SwiGLU", GRAIN: "GRAIN"}
OPTIMIZER_NAMES = {
    "adamw": "AdamW", "muon": "Muon", "lion": "Lion", "soap_adamw": "SOAP", "ademamix": "ADeMaMix",
    "adafactor_came": "CAME", "schedule_free_adamw": "Schedule-Free AdamW", "tiller_v1": "TILLER",
    "tiller_then_muon_v1": "TILLER→Muon",
}
# optimizer key -> directory of its tables
TABLE_DIRS = {
    "adamw": "adamw", "muon": "muon", "soap_adamw": "soap", "ademamix": "ademamix", "adafactor_came": "came",
    "schedule_free_adamw": "schedule_free_adamw", "tiller_v1": "tiller", "tiller_then_muon_v1": "tiller_then_muon",
}
CANDIDATE_METHODS = {"tiller_v1": "tiller", "tiller_then_muon_v1": "tiller_then_muon"}

RUN_FIELDS = (
    "run_index", "model_scale", "dataset", "seed", "train_tokens", "steps_required", "steps_completed", "status",
    "activation", "activation_display_name", "optimizer", "optimizer_display_name", "method",
    "method_display_name", "step1000_validation_loss", "final_validation_loss", "final_validation_perplexity",
    "matched_control_step1000_validation_loss", "matched_control_validation_loss",
    "lead_at_step1000_vs_matched_control", "lead_vs_matched_control", "time_scope", "total_seconds",
    "matched_control_total_seconds", "total_time_ratio_vs_matched_control", "training_loop_total_seconds",
    "mean_seconds_per_step", "tokens_per_second", "stopped_early", "lr_wd_fairness_passed",
    "realized_lr_trace_sha256", "slurm_job_id", "slurm_restart_count", "slurm_node", "timing_attempt_id",
    "source_phase", "source_row_index", "source_row_id", "source_jsonl", "source_jsonl_sha256",
)
GROUP_FIELDS = ("model_scale", "dataset", "train_tokens", "steps_required", "activation",
                "activation_display_name", "optimizer", "optimizer_display_name", "method", "method_display_name")
SUMMARY_FIELDS = GROUP_FIELDS + (
    "runs_total", "runs_reached_required_step", "runs_stopped_early", "runs_non_finite", "endpoint_seed_count",
    "validation_loss_mean", "validation_loss_sample_std", "matched_control_seed_count",
    "matched_control_validation_loss_mean", "lead_vs_matched_control_mean", "lead_vs_matched_control_sample_std",
    "exact_time_ratio_seed_count", "exact_total_time_ratio_mean", "exact_total_time_ratio_sample_std",
    "total_seconds_mean", "total_seconds_sample_std", "mean_seconds_per_step", "tokens_per_second_mean", "status",
)
CHECKPOINT_FIELDS = (
    "run_index", "model_scale", "dataset", "seed", "activation", "activation_display_name", "optimizer",
    "optimizer_display_name", "method", "method_display_name", "step", "validation_loss", "validation_perplexity",
    "active_seconds_at_validation",
)
_INT_GROUP = {"train_tokens", "steps_required"}


class ResultsError(RuntimeError):
    pass


def number(value: Any) -> float | None:
    """A finite float, or None for blanks, text and inf/nan."""
    if value is None or value == "":
        return None
    try:
        x = float(value)
    except (TypeError, ValueError):
        return None
    return x if math.isfinite(x) else None


def _blank(value):
    return "" if value is None else value


def read_jsonl(path: Path) -> list[dict]:
    """Records of a trainer JSONL; a torn LAST line (a run still writing) is dropped,
    any other unreadable line is an error."""
    lines = Path(path).read_text(encoding="utf-8").splitlines()
    out = []
    last = max((i for i, line in enumerate(lines) if line.strip()), default=-1)
    for i, line in enumerate(lines):
        if not line.strip():
            continue
        try:
            rec = json.loads(line)
        except json.JSONDecodeError:
            if i == last:
                break
            raise ResultsError(f"{path}: line {i + 1} is not JSON")
        if not isinstance(rec, dict):
            raise ResultsError(f"{path}: line {i + 1} is not an object")
        out.append(rec)
    return out


def _only(recs: Iterable[dict], event: str) -> dict | None:
    found = [r for r in recs if r.get("event") == event]
    if len(found) > 1:
        raise ResultsError(f"{len(found)} {event!r} records in one run")
    return found[0] if found else None


def _evals(recs: Iterable[dict]) -> dict[int, dict]:
    out: dict[int, dict] = {}
    for r in recs:
        if r.get("event") == "eval":
            step = int(r["step"])
            if step in out:
                raise ResultsError(f"two evaluations at step {step}")
            out[step] = r
    return out


def wall_clock(candidates: Iterable[Path]) -> tuple[dict | None, Path | None]:
    """The first existing process wall-clock record among ``candidates``."""
    for p in candidates:
        if p is not None and Path(p).is_file():
            payload = json.loads(Path(p).read_text())
            if payload.get("schema") != WALL_CLOCK_SCHEMA:
                raise ResultsError(f"{p} is not a process wall-clock record")
            if payload.get("return_code") == 0 and number(payload.get("elapsed_seconds")) is None:
                raise ResultsError(f"{p} records a clean exit without an elapsed time")
            return payload, Path(p)
    return None, None


def method_display(activation: str, optimizer: str) -> str:
    if optimizer in CANDIDATE_METHODS:
        return OPTIMIZER_NAMES[optimizer]
    return f"{ACTIVATION_NAMES[activation]} + {OPTIMIZER_NAMES[optimizer]}"


def run_record(spec: dict, path: Path, *, clock_paths: Iterable[Path] = (), display_root: Path | None = None):
    """(runs.csv row, checkpoints.csv rows) of one run.  ``spec`` holds run_index,
    model, dataset, seed, train_tokens, steps, activation, optimizer, method, phase,
    source_row_index, source_row_id."""
    activation, optimizer, steps = spec["activation"], spec["optimizer"], int(spec["steps"])
    row = dict.fromkeys(RUN_FIELDS, "")
    row.update(run_index=int(spec["run_index"]), model_scale=spec["model"], dataset=spec["dataset"],
               seed=int(spec["seed"]), train_tokens=int(spec["train_tokens"]), steps_required=steps,
               steps_completed=0, status="pending", activation=activation,
               activation_display_name=ACTIVATION_NAMES[activation], optimizer=optimizer,
               optimizer_display_name=OPTIMIZER_NAMES[optimizer], method=spec["method"],
               method_display_name=method_display(activation, optimizer), source_phase=spec["phase"],
               source_row_index=int(spec["source_row_index"]), source_row_id=spec["source_row_id"])
    path = Path(path)
    if not path.is_file():
        return row, []
    recs = read_jsonl(path)
    cfg, summ = _only(recs, "config"), _only(recs, "summary")
    ev = _evals(recs)
    if summ is not None:
        completed = int(summ.get("completed_steps", 0))
        stopped = bool(summ.get("stopped_early"))
    else:
        completed = max((int(r["step"]) for r in recs if isinstance(r.get("step"), (int, float))), default=0)
        stopped = any(r.get("event") == "stopped_early" for r in recs)
    end = ev.get(steps)
    end_loss = number(end.get("val_loss")) if end else None
    end_ppl = number(end.get("val_ppl")) if end else None
    loop = number(summ.get("total_seconds")) if summ else None
    clock, _ = wall_clock([path.with_suffix(".wall_clock.json"), *clock_paths])
    process = float(clock["elapsed_seconds"]) if clock is not None and clock.get("return_code") == 0 else None
    total = process if process is not None else loop
    if stopped:
        status = "stopped_early"
    elif summ is not None and completed == steps and end is not None:
        status = "complete" if end_loss is not None else "non_finite"
    else:
        status = "incomplete"
    if status == "complete" and clock is not None and clock.get("return_code") != 0:
        # the trainer finished but the process did not exit cleanly
        status, end_loss, end_ppl = "incomplete", None, None
    ident = summ or cfg or {}
    fair = (cfg or {}).get("optimizer_lr_wd_fairness", {})
    shown = path
    if display_root is not None:
        try:
            shown = path.resolve().relative_to(Path(display_root).resolve())
        except ValueError:
            shown = path.resolve()
    row.update(
        steps_completed=completed, status=status,
        step1000_validation_loss=_blank(number(ev[SCREEN_STEP].get("val_loss"))) if SCREEN_STEP in ev else "",
        final_validation_loss=_blank(end_loss), final_validation_perplexity=_blank(end_ppl),
        time_scope=("end_to_end_process" if process is not None else "training_loop") if total is not None else "",
        total_seconds=_blank(total), training_loop_total_seconds=_blank(loop),
        mean_seconds_per_step=_blank(number(summ.get("mean_seconds_per_step"))) if summ else "",
        tokens_per_second=_blank(number(summ.get("tokens_per_second"))) if summ else "",
        stopped_early=stopped, lr_wd_fairness_passed=fair.get("passed", ""),
        realized_lr_trace_sha256=summ.get("realized_lr_trace_sha256", "") if summ else "",
        slurm_job_id=_blank(ident.get("slurm_job_id")), slurm_restart_count=_blank(ident.get("slurm_restart_count")),
        slurm_node=_blank(ident.get("slurm_node")), timing_attempt_id=_blank(ident.get("timing_attempt_id")),
        source_jsonl=str(shown), source_jsonl_sha256=hashlib.sha256(path.read_bytes()).hexdigest())
    points = []
    for step, r in sorted(ev.items()):
        points.append({
            "run_index": row["run_index"], "model_scale": row["model_scale"], "dataset": row["dataset"],
            "seed": row["seed"], "activation": activation, "activation_display_name": row["activation_display_name"],
            "optimizer": optimizer, "optimizer_display_name": row["optimizer_display_name"],
            "method": row["method"], "method_display_name": row["method_display_name"], "step": step,
            "validation_loss": _blank(number(r.get("val_loss"))),
            "validation_perplexity": _blank(number(r.get("val_ppl"))),
            "active_seconds_at_validation": _blank(number(r.get("active_seconds_at_val_loss"))),
        })
    return row, points


def pair(candidate: dict, control: dict) -> None:
    """Fill the candidate's matched-control columns from ``control``."""
    c1000, k1000 = number(control["step1000_validation_loss"]), number(candidate["step1000_validation_loss"])
    if c1000 is not None:
        candidate["matched_control_step1000_validation_loss"] = c1000
        if k1000 is not None:
            candidate["lead_at_step1000_vs_matched_control"] = c1000 - k1000
    if control["status"] != "complete":
        return
    candidate["matched_control_validation_loss"] = control["final_validation_loss"]
    c_sec = number(control["total_seconds"])
    if c_sec is not None:
        candidate["matched_control_total_seconds"] = c_sec
    if candidate["status"] != "complete":
        return
    candidate["lead_vs_matched_control"] = float(control["final_validation_loss"]) - float(
        candidate["final_validation_loss"])
    k_sec = number(candidate["total_seconds"])
    if (k_sec is not None and c_sec is not None
            and candidate["time_scope"] == control["time_scope"] == "end_to_end_process"):
        candidate["total_time_ratio_vs_matched_control"] = k_sec / c_sec


def _mean(xs):
    return statistics.fmean(xs) if xs else ""


def _std(xs):
    return statistics.stdev(xs) if len(xs) > 1 else ""


def _finite_column(rows, field, keep=lambda r: True):
    return [x for r in rows if keep(r) and (x := number(r[field])) is not None]


def summarize(runs: Iterable[dict]) -> list[dict]:
    """summary.csv rows: one per cell of ``GROUP_FIELDS``, sorted by cell."""
    cells: dict[tuple, list[dict]] = defaultdict(list)
    for r in runs:
        cells[tuple(int(r[f]) if f in _INT_GROUP else str(r[f]) for f in GROUP_FIELDS)].append(r)
    out = []
    for key in sorted(cells):
        group = cells[key]
        ends = _finite_column(group, "final_validation_loss", lambda r: r["status"] == "complete")
        controls = _finite_column(group, "matched_control_validation_loss")
        leads = _finite_column(group, "lead_vs_matched_control")
        ratios = _finite_column(group, "total_time_ratio_vs_matched_control")
        seconds = _finite_column(group, "total_seconds")
        reached = sum(int(r["steps_completed"]) >= int(r["steps_required"]) for r in group)
        stopped = sum(str(r["stopped_early"]).strip().lower() == "true" for r in group)
        bad = sum(r["status"] == "non_finite" for r in group)
        if bad:
            status = "non_finite"
        elif stopped:
            status = "stopped_early"
        elif reached < len(group):
            status = "pending" if all(r["status"] == "pending" for r in group) else "incomplete"
        elif len(ends) < len(group):
            status = "endpoint_loss_unavailable"
        else:
            status = "complete"
        cell = dict(zip(GROUP_FIELDS, key))
        cell.update(
            runs_total=len(group), runs_reached_required_step=reached, runs_stopped_early=stopped,
            runs_non_finite=bad, endpoint_seed_count=len(ends), validation_loss_mean=_mean(ends),
            validation_loss_sample_std=_std(ends), matched_control_seed_count=len(controls),
            matched_control_validation_loss_mean=_mean(controls), lead_vs_matched_control_mean=_mean(leads),
            lead_vs_matched_control_sample_std=_std(leads), exact_time_ratio_seed_count=len(ratios),
            exact_total_time_ratio_mean=_mean(ratios), exact_total_time_ratio_sample_std=_std(ratios),
            total_seconds_mean=_mean(seconds), total_seconds_sample_std=_std(seconds),
            mean_seconds_per_step=_mean(_finite_column(group, "mean_seconds_per_step")),
            tokens_per_second_mean=_mean(_finite_column(group, "tokens_per_second")), status=status)
        out.append(cell)
    return out


def manifest_tables(manifest_rows: Iterable[dict], run_root: Path, *, display_root=None):
    """Runs and checkpoints per optimizer for the manifest's baseline runs, GRAIN
    arms paired with their SwiGLU control."""
    runs: dict[str, list] = defaultdict(list)
    points: dict[str, list] = defaultdict(list)
    arms: dict[tuple, dict] = defaultdict(dict)
    for m in manifest_rows:
        if m["phase"] == PREFLIGHT or m["optimizer"] not in TABLE_DIRS:
            continue
        spec = dict(run_index=m["row_index"], model=m["model"], dataset=m["dataset"], seed=m["seed"],
                    train_tokens=m["train_tokens"], steps=m["steps"], activation=m["activation"],
                    optimizer=m["optimizer"], method=m["method"], phase=m["phase"],
                    source_row_index=m["row_index"], source_row_id=m["row_id"])
        path = Path(run_root) / m["phase"] / m["dataset"] / m["row_id"] / f"{m['activation']}.jsonl"
        run, pts = run_record(spec, path, display_root=display_root)
        runs[m["optimizer"]].append(run)
        points[m["optimizer"]].extend(pts)
        key = tuple(m[k] for k in ("phase", "model", "dataset", "seed", "train_tokens", "steps", "optimizer"))
        arms[key][m["activation"]] = run
    for both in arms.values():
        if SWIGLU in both and GRAIN in both:
            pair(both[GRAIN], both[SWIGLU])
    return runs, points


def _screen(row, run_root: Path, result_dir: Path) -> dict | None:
    for p in (result_dir / "STEP1000_SCREEN.json", Path(run_root) / f"{R.run_name(row, 'candidate')}.step1000.json"):
        if p.is_file():
            screen = json.loads(p.read_text())
            if screen.get("matrix_index") != row["matrix_index"]:
                raise ResultsError(f"{p} belongs to matrix row {screen.get('matrix_index')}")
            return screen
    return None


def _published_control(row) -> dict | None:
    """The matched control published with a matrix row, as a runs.csv-like row."""
    mc = row.get("matched_control")
    if not isinstance(mc, dict) or mc.get("status") != "complete":
        return None
    return {"status": "complete", "final_validation_loss": mc.get("endpoint_validation_loss"),
            "step1000_validation_loss": _blank(mc.get("step1000_validation_loss")),
            "total_seconds": _blank(mc.get("total_seconds")), "time_scope": mc.get("time_scope", "")}


def matrix_tables(matrix: dict, run_root: Path, analysis_root: Path, *, controls=None, display_root=None):
    """Runs and checkpoints of the matrix's candidate arms.  An endpoint result
    (``row-NN/RESULT.json``) supplies the paired columns and process times;
    without one the candidate is paired with its control run (``controls``:
    manifest row id -> runs.csv row) or the control published with the row.  A
    negative step-1,000 screen marks the run stopped."""
    controls = controls or {}
    runs, points = [], []
    for row in matrix["rows"]:
        index, optimizer = int(row["matrix_index"]), row["candidate_optimizer"]
        spec = dict(run_index=index, model=row["model"], dataset=row["dataset"], seed=row["seed"],
                    train_tokens=row["max_train_tokens"], steps=row["steps"], activation=row["candidate_activation"],
                    optimizer=optimizer, method=CANDIDATE_METHODS[optimizer], phase=row["phase"],
                    source_row_index=row["source_manifest_row_index"], source_row_id=row["source_manifest_row_id"])
        path = R.jsonl_path(row, "candidate", run_root)
        clock = Path(run_root) / f"{R.run_name(row, 'candidate')}.wall_clock.json"
        run, pts = run_record(spec, path, clock_paths=[clock], display_root=display_root)
        result_dir = Path(analysis_root) / f"row-{index:02d}"
        screen = _screen(row, run_root, result_dir)
        if screen is not None and screen.get("status") == "failed_negative_interrupted":
            seen = number(_evals(read_jsonl(path)).get(SCREEN_STEP, {}).get("val_loss")) if path.is_file() else None
            if path.is_file() and (seen is None or screen.get("candidate_step1000_loss") != seen):
                raise ResultsError(f"the step-1,000 screen of row {index} disagrees with the candidate's JSONL")
            run.update(status="stopped_early", stopped_early=True, final_validation_loss="",
                       final_validation_perplexity="")
        result_path = result_dir / "RESULT.json"
        if result_path.is_file():
            res = json.loads(result_path.read_text())
            want = {"schema": "tiller_matched_endpoint_result_v1", "status": "complete", "matrix_index": index,
                    "model": row["model"], "dataset": row["dataset"], "seed": int(row["seed"]),
                    "steps": int(row["steps"])}
            wrong = {k: (res.get(k), v) for k, v in want.items() if res.get(k) != v}
            if wrong:
                raise ResultsError(f"{result_path} does not match its matrix row: {wrong}")
            if run["status"] == "stopped_early":
                raise ResultsError(f"row {index} was stopped at step 1,000 but has a complete endpoint result")
            run.update(
                step1000_validation_loss=res["candidate_step1000_loss"],
                final_validation_loss=res["candidate_endpoint_loss"],
                matched_control_step1000_validation_loss=res["control_step1000_loss"],
                matched_control_validation_loss=res["control_endpoint_loss"],
                lead_at_step1000_vs_matched_control=res["step1000_absolute_lead"],
                lead_vs_matched_control=res["absolute_endpoint_lead"],
                time_scope=res.get("time_scope", "end_to_end_process"),
                total_seconds=res["candidate_end_to_end_total_seconds"],
                matched_control_total_seconds=res["control_end_to_end_total_seconds"],
                total_time_ratio_vs_matched_control=(
                    res["exact_matched_hardware_end_to_end_total_time_ratio"]
                    if res.get("time_scope", "end_to_end_process") == "end_to_end_process" else ""),
                training_loop_total_seconds=res["candidate_training_loop_total_seconds"], status="complete")
        else:
            ctl = controls.get(row["source_manifest_row_id"]) or _published_control(row)
            if ctl is not None:
                pair(run, ctl)
        runs.append(run)
        points.extend(pts)
    return runs, points


def write_csv(path: Path, fields, rows) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("w", newline="", encoding="utf-8") as fh:
        w = csv.DictWriter(fh, fieldnames=list(fields), extrasaction="raise", lineterminator="\n")
        w.writeheader()
        w.writerows(rows)
    tmp.replace(path)


def publish(output_root: Path, optimizer: str, runs: list, points: list) -> Path:
    """Write one optimizer's three tables (sorted like the published ones)."""
    d = Path(output_root) / TABLE_DIRS[optimizer]
    runs = sorted(runs, key=lambda r: (str(r["model_scale"]), int(r["train_tokens"]), str(r["dataset"]),
                                       int(r["seed"]), str(r["activation"]), int(r["run_index"])))
    points = sorted(points, key=lambda r: (str(r["model_scale"]), str(r["dataset"]), int(r["seed"]),
                                           str(r["activation"]), int(r["step"])))
    write_csv(d / "runs.csv", RUN_FIELDS, runs)
    write_csv(d / "summary.csv", SUMMARY_FIELDS, summarize(runs))
    write_csv(d / "checkpoints.csv", CHECKPOINT_FIELDS, points)
    return d


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--manifest", type=Path, required=True)
    ap.add_argument("--runs", type=Path, required=True, help="root of the manifest runs' JSONL")
    ap.add_argument("--matrix", type=Path)
    ap.add_argument("--tiller-runs", type=Path)
    ap.add_argument("--tiller-analysis", type=Path)
    ap.add_argument("--output-root", type=Path, required=True)
    ap.add_argument("--only-optimizer", action="append", choices=tuple(TABLE_DIRS))
    ap.add_argument("--include-pending", action="store_true")
    a = ap.parse_args(argv)
    by_opt, pts = manifest_tables(R.load_manifest(a.manifest), a.runs)
    if a.matrix is not None:
        controls = {r["source_row_id"]: r for rows in by_opt.values() for r in rows if r["status"] != "pending"}
        mruns, mpts = matrix_tables(R.load_matrix(a.matrix), a.tiller_runs or a.runs,
                                    a.tiller_analysis or (a.tiller_runs or a.runs), controls=controls)
        for optimizer in CANDIDATE_METHODS:
            by_opt[optimizer] = [r for r in mruns if r["optimizer"] == optimizer]
            pts[optimizer] = [p for p in mpts if p["optimizer"] == optimizer]
    written = 0
    for optimizer in TABLE_DIRS:
        if a.only_optimizer and optimizer not in a.only_optimizer:
            continue
        runs = [r for r in by_opt.get(optimizer, []) if a.include_pending or r["status"] != "pending"]
        if not runs:
            continue
        keep = {int(r["run_index"]) for r in runs}
        points = [p for p in pts.get(optimizer, []) if int(p["run_index"]) in keep]
        d = publish(a.output_root, optimizer, runs, points)
        written += 1
        print(json.dumps({"tables": str(d), "runs": len(runs), "checkpoints": len(points)}))
    if not written:
        print(json.dumps({"error": "no run produced a JSONL; nothing written"}))
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
