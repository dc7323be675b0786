"""Aggregate trainer JSONL trajectories by (optimizer, activation, seed).

    python -m rational_optimizer_b200.train.aggregate --run-dir RUNS --out-dir OUT \\
        [--baseline silu] [--baseline-optimizer ""] [--classic-optimizer adamw]

Writes ``per_seed.csv``, ``aggregate.csv``, ``summary.json`` and a Markdown
``README.md``.  Column names and gap definitions are those of the reference
tool (training/aggregate_results.py:27-337) so result tables from either
framework compare directly: for every complete run (a final ``eval`` and a
``summary`` record) the validation-loss / perplexity gaps and the step-time
ratio are taken against the external baseline activation (same seed, the
row's optimizer unless ``--baseline-optimizer`` is given) and against the
classic optimizer with the same activation; per (optimizer, activation) the
seed mean and sample standard deviation are reported.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import statistics
from datetime import datetime, timezone
from pathlib import Path

GAP_KINDS = ("external_baseline", "classic_same_activation")


def parse_run_dir(run_dir: Path) -> dict:
    """(optimizer, activation, seed) -> {config fields, final_eval, summary}."""
    runs = {}
    for path in sorted(Path(run_dir).glob("*.jsonl")):
        key = None
        for line in path.read_text(encoding="utf-8").splitlines():
            if not line.strip():
                continue
            ev = json.loads(line)
            kind = ev.get("event")
            if kind == "config":
                key = (str(ev.get("optimizer", "adamw")), str(ev["activation"]), int(ev["seed"]))
                runs[key] = {"optimizer": key[0], "activation": key[1], "seed": key[2],
                             "params": int(ev["params"]), "steps": int(ev["steps"]), "config": ev,
                             "final_eval": None, "summary": None}
            elif key is not None and kind == "eval":
                prev = runs[key]["final_eval"]
                if prev is None or int(ev["step"]) >= int(prev["step"]):
                    runs[key]["final_eval"] = ev
            elif key is not None and kind == "summary":
                runs[key]["summary"] = ev
    return runs


def sample_std(values) -> float:
    finite = [float(v) for v in values if math.isfinite(float(v))]
    if not finite:
        return math.nan
    return statistics.stdev(finite) if len(finite) > 1 else 0.0


def _metrics(run):
    if run is None:
        return math.nan, math.nan, math.nan
    return (float(run["final_eval"]["val_loss"]), float(run["final_eval"]["val_ppl"]),
            float(run["summary"]["mean_seconds_per_step"]))


def build_rows(runs, baseline, baseline_optimizer, classic_optimizer):
    done = {k: r for k, r in runs.items() if r.get("final_eval") is not None and r.get("summary") is not None}
    optimizers = sorted({k[0] for k in done})
    activations = sorted({k[1] for k in done})
    seeds = sorted({k[2] for k in done})
    per_seed = []
    for opt in optimizers:
        ext_opt = baseline_optimizer or opt
        for seed in seeds:
            b_loss, b_ppl, b_sec = _metrics(done.get((ext_opt, baseline, seed)))
            for act in activations:
                run = done.get((opt, act, seed))
                if run is None:
                    continue
                c_loss, c_ppl, c_sec = _metrics(done.get((classic_optimizer, act, seed)))
                loss, ppl, sec = _metrics(run)
                row = {
                    "optimizer": opt, "seed": seed, "activation": act, "params": int(run["params"]),
                    "val_loss": loss, "val_ppl": ppl, "mean_seconds_per_step": sec,
                    "tokens_per_second": float(run["summary"]["tokens_per_second"]),
                    "total_seconds": float(run["summary"]["total_seconds"]),
                    "external_baseline_optimizer": ext_opt, "external_baseline_activation": baseline,
                    "classic_optimizer": classic_optimizer,
                }
                for kind, (rl, rp, rs) in zip(GAP_KINDS, ((b_loss, b_ppl, b_sec), (c_loss, c_ppl, c_sec))):
                    row[f"loss_gap_vs_{kind}"] = loss - rl
                    row[f"ppl_gap_vs_{kind}"] = ppl - rp
                    row[f"time_ratio_vs_{kind}"] = sec / rs if rs == rs and rs != 0 else math.nan
                # legacy column names: the external baseline is SiLU in every published table
                row["loss_gap_vs_silu"] = row["loss_gap_vs_external_baseline"]
                row["ppl_gap_vs_silu"] = row["ppl_gap_vs_external_baseline"]
                row["time_ratio_vs_silu"] = row["time_ratio_vs_external_baseline"]
                per_seed.append(row)
    aggregate = []
    for opt in optimizers:
        for act in activations:
            rows = [r for r in per_seed if r["optimizer"] == opt and r["activation"] == act]
            if not rows:
                continue
            col = lambda k: [float(r[k]) for r in rows]
            agg = {"optimizer": opt, "activation": act, "seeds": len(rows), "params": int(rows[0]["params"]),
                   "mean_val_loss": statistics.mean(col("val_loss")), "std_val_loss": sample_std(col("val_loss")),
                   "mean_val_ppl": statistics.mean(col("val_ppl")), "std_val_ppl": sample_std(col("val_ppl")),
                   "mean_seconds_per_step": statistics.mean(col("mean_seconds_per_step"))}
            for kind in GAP_KINDS:
                agg[f"mean_loss_gap_vs_{kind}"] = statistics.mean(col(f"loss_gap_vs_{kind}"))
                agg[f"std_loss_gap_vs_{kind}"] = sample_std(col(f"loss_gap_vs_{kind}"))
                agg[f"mean_ppl_gap_vs_{kind}"] = statistics.mean(col(f"ppl_gap_vs_{kind}"))
                agg[f"mean_time_ratio_vs_{kind}"] = statistics.mean(col(f"time_ratio_vs_{kind}"))
            agg["mean_loss_gap_vs_silu"] = agg["mean_loss_gap_vs_external_baseline"]
            agg["std_loss_gap_vs_silu"] = agg["std_loss_gap_vs_external_baseline"]
            agg["mean_ppl_gap_vs_silu"] = agg["mean_ppl_gap_vs_external_baseline"]
            agg["mean_time_ratio_vs_silu"] = agg["mean_time_ratio_vs_external_baseline"]
            aggregate.append(agg)
    return per_seed, aggregate


def write_csv(path: Path, rows) -> None:
    if not rows:
        path.write_text("", encoding="utf-8")
        return
    with path.open("w", encoding="utf-8", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=list(rows[0].keys()), lineterminator="\n")
        w.writeheader()
        w.writerows(rows)


def _table(rows, headers):
    out = ["| " + " | ".join(headers) + " |", "|" + "|".join(["---"] * len(headers)) + "|"]
    out += ["| " + " | ".join(r) + " |" for r in rows]
    return "\n".join(out)


def write_readme(out_dir: Path, run_dir, job_id, log_path, per_seed, aggregate) -> None:
    f6 = lambda v: f"{float(v):.6f}"
    seed_rows = [[str(r["optimizer"]), str(r["seed"]), str(r["activation"]), f"{int(r['params']):,}",
                  f6(r["val_loss"]), f6(r["loss_gap_vs_external_baseline"]),
                  f6(r["loss_gap_vs_classic_same_activation"]), f"{float(r['val_ppl']):.3f}",
                  f6(r["mean_seconds_per_step"]), f"{float(r['time_ratio_vs_external_baseline']):.3f}x",
                  f"{float(r['time_ratio_vs_classic_same_activation']):.3f}x"]
                 for r in sorted(per_seed, key=lambda r: (r["optimizer"], r["seed"], r["activation"]))]
    agg_rows = [[str(r["optimizer"]), str(r["activation"]), str(r["seeds"]), f"{int(r['params']):,}",
                 f6(r["mean_val_loss"]), f6(r["std_val_loss"]), f6(r["mean_loss_gap_vs_external_baseline"]),
                 f6(r["std_loss_gap_vs_external_baseline"]), f6(r["mean_loss_gap_vs_classic_same_activation"]),
                 f6(r["std_loss_gap_vs_classic_same_activation"]), f"{float(r['mean_val_ppl']):.3f}",
                 f6(r["mean_seconds_per_step"]), f"{float(r['mean_time_ratio_vs_external_baseline']):.3f}x",
                 f"{float(r['mean_time_ratio_vs_classic_same_activation']):.3f}x"]
                for r in sorted(aggregate, key=lambda r: (r["optimizer"], r["activation"]))]
    stamp = datetime.now(timezone.utc).strftime("%Y-%m-%d %H:%M:%S UTC")
    text = (f"# Language-Model Benchmark Summary\n\nGenerated: {stamp}\n\nRaw run directory:\n\n```text\n{run_dir}\n```\n\n"
            f"Job:\n\n```text\n{job_id or 'unknown'}\n```\n\nLog:\n\n```text\n{log_path or 'unknown'}\n```\n\n"
            "This result folder is an organized summary only. The raw JSONL logs remain in\nthe run directory above.\n\n"
            "## Per-Seed Results\n\n"
            + _table(seed_rows, ["Optimizer", "Seed", "Activation", "Params", "Val loss", "Gap vs external",
                                 "Gap vs classic", "PPL", "Sec/step", "Time vs external", "Time vs classic"])
            + "\n\n## Aggregate Results\n\n"
            + _table(agg_rows, ["Optimizer", "Activation", "Seeds", "Params", "Mean loss", "Std loss",
                                "Mean gap vs external", "Std gap vs external", "Mean gap vs classic",
                                "Std gap vs classic", "Mean PPL", "Mean sec/step", "Mean time vs external",
                                "Mean time vs classic"]) + "\n")
    (Path(out_dir) / "README.md").write_text(text, encoding="utf-8")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--run-dir", required=True, type=Path)
    ap.add_argument("--out-dir", required=True, type=Path)
    ap.add_argument("--baseline", default="silu", help="external baseline activation")
    ap.add_argument("--baseline-optimizer", default="",
                    help="optimizer of the external baseline; defaults to each row's optimizer")
    ap.add_argument("--classic-optimizer", default="adamw")
    ap.add_argument("--job-id", default="")
    ap.add_argument("--log-path", default="")
    a = ap.parse_args(argv)
    runs = parse_run_dir(a.run_dir)
    per_seed, aggregate = build_rows(runs, a.baseline, a.baseline_optimizer, a.classic_optimizer)
    a.out_dir.mkdir(parents=True, exist_ok=True)
    write_csv(a.out_dir / "per_seed.csv", per_seed)
    write_csv(a.out_dir / "aggregate.csv", aggregate)
    (a.out_dir / "summary.json").write_text(json.dumps(
        {"run_dir": str(a.run_dir), "job_id": a.job_id, "log_path": a.log_path, "per_seed": per_seed,
         "aggregate": aggregate}, indent=2, sort_keys=True), encoding="utf-8")
    write_readme(a.out_dir, a.run_dir, a.job_id, a.log_path, per_seed, aggregate)


if __name__ == "__main__":
    main()
