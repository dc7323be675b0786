"""Verification of a published experiment package: manifest, matrix, token
fingerprints, result tables and source freeze (behaviour of
experiments/protocol/verify_repository.py:328-1672, checked by regeneration
instead of by restating every rule).

* manifest - equal, line for line, to the one :mod:`.manifest` builds from
  the experiment design, and every matched cell differs only in its
  activation arm (:func:`.manifest.check_matched_arms`);
* matrix - equal to the one :mod:`.matrix` derives from that manifest and
  the published result tables (the hardware ``timing_condition`` aside), its
  ``source_manifest_sha256`` the manifest's hash;
* token fingerprints - ``rationalopt_token_fingerprints_v2``, one cell per
  (dataset, 100M / 300M budget), four 64-hex digests each;
* result tables - per optimizer directory: published headers, unique cells,
  identity columns (display names, method keys), every lead equal to the
  control loss minus the candidate loss, run statuses consistent with their
  numbers, ``summary.csv`` byte-equal to :func:`.results.summarize` of
  ``runs.csv``, checkpoints belonging to listed runs with unique steps;
* source freeze - :func:`.freeze.check` reports nothing added, removed or
  changed (full mode only).

    python -m rational_optimizer_b200.protocol.verify --package experiments/protocol \\
        --results experiments/results [--root .] [--quick]

Exit status 0 with one ``PASS <check>: <count>`` line per check, 1 with
``FAIL <reason>``.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import re
import sys
from pathlib import Path

from . import freeze as FZ
from . import manifest as MF
from . import matrix as MX
from . import results as RS

HEX64 = re.compile(r"[0-9a-f]{64}")
FINGERPRINT_SCHEMA = "rationalopt_token_fingerprints_v2"
BUDGETS = ((100_000_000, 4_000_000), (300_000_000, 8_000_000))
LEADS = (("final_validation_loss", "matched_control_validation_loss", "lead_vs_matched_control"),
         ("step1000_validation_loss", "matched_control_step1000_validation_loss",
          "lead_at_step1000_vs_matched_control"))


class VerificationError(RuntimeError):
    pass


def require(ok: bool, message: str) -> None:
    if not ok:
        raise VerificationError(message)


def _csv(path: Path, fields) -> list[dict]:
    require(path.is_file(), f"{path} is missing")
    with path.open(newline="", encoding="utf-8") as fh:
        reader = csv.DictReader(fh)
        require(tuple(reader.fieldnames or ()) == tuple(fields), f"{path}: the header changed")
        return list(reader)


def _float(text: str, where: str) -> float | None:
    if text == "":
        return None
    try:
        return float(text)
    except ValueError:
        raise VerificationError(f"{where}: {text!r} is not a number") from None


def verify_manifest(path: Path) -> list[dict]:
    rows = MX.read_manifest(path)
    built = MF.build_rows()
    require(len(rows) == len(built), f"the manifest holds {len(rows)} rows, the design {len(built)}")
    for have, want in zip(rows, built):
        diff = {k: (have.get(k), v) for k, v in want.items() if have.get(k) != v}
        require(not diff, f"manifest row {want['row_index']} differs from the design: {diff}")
    MF.check_matched_arms(rows)
    return rows


def verify_matrix(path: Path, manifest_path: Path, results_root: Path) -> dict:
    payload = json.loads(path.read_text(encoding="utf-8"))
    require(payload.get("schema") == "tiller_evaluation_matrix_v1", "matrix schema changed")
    require(payload.get("source_manifest_sha256") == MX.file_sha256(manifest_path),
            "the matrix was built from another manifest")
    built = MX.build_matrix(manifest_path, results_root, manifest_name=payload.get("source_manifest"))
    require({k: v for k, v in payload.items() if k != "rows"} == {k: v for k, v in built.items() if k != "rows"},
            "matrix header differs from the one the manifest and results give")
    require(len(payload["rows"]) == len(built["rows"]), "matrix row count differs")
    for have, want in zip(payload["rows"], built["rows"]):
        want = dict(want, timing_condition=have.get("timing_condition"))
        diff = sorted(k for k in set(have) | set(want) if have.get(k) != want.get(k))
        require(not diff, f"matrix row {have.get('matrix_index')} differs in {diff}")
    return payload


def verify_fingerprints(path: Path, datasets) -> dict:
    payload = json.loads(path.read_text(encoding="utf-8"))
    require(payload.get("schema") == FINGERPRINT_SCHEMA, "token-fingerprint schema changed")
    require(payload.get("tokenizer") == MF.TOKENIZER[0] and payload.get("tokenizer_revision") == MF.TOKENIZER[1],
            "token-fingerprint tokenizer changed")
    want = {(d, t, v) for d in datasets for t, v in BUDGETS}
    seen = set()
    for i, cell in enumerate(payload.get("cells", ())):
        key = (cell.get("dataset"), cell.get("train_tokens"), cell.get("validation_tokens"))
        require(key in want and key not in seen, f"token-fingerprint cell {i} {key} is unexpected or repeated")
        seen.add(key)
        for f in ("train_token_content_sha256", "validation_token_content_sha256", "train_token_sample_sha256",
                  "validation_token_sample_sha256"):
            require(HEX64.fullmatch(str(cell.get(f, ""))) is not None, f"cell {key}: malformed {f}")
    require(seen == want, f"token-fingerprint cells missing: {sorted(want - seen)}")
    return payload


def _run_checks(folder: str, runs: list[dict]) -> None:
    optimizer = next(k for k, v in RS.TABLE_DIRS.items() if v == folder)
    keys = set()
    for i, r in enumerate(runs):
        where = f"{folder}/runs.csv row {i + 2}"
        require(r["optimizer"] == optimizer and r["optimizer_display_name"] == RS.OPTIMIZER_NAMES[optimizer],
                f"{where}: optimizer identity")
        require(r["activation"] in RS.ACTIVATION_NAMES
                and r["activation_display_name"] == RS.ACTIVATION_NAMES[r["activation"]], f"{where}: activation")
        require(r["method_display_name"] == RS.method_display(r["activation"], optimizer), f"{where}: method name")
        if optimizer in RS.CANDIDATE_METHODS:
            require(r["activation"] == RS.GRAIN and r["method"] == RS.CANDIDATE_METHODS[optimizer],
                    f"{where}: a TILLER row must be GRAIN with its method key")
        key = (r["model_scale"], r["dataset"], r["seed"], r["train_tokens"], r["activation"])
        require(key not in keys, f"{where}: duplicate run cell {key}")
        keys.add(key)
        for cand, ctl, lead in LEADS:
            c, k, d = (_float(r[f], f"{where}/{f}") for f in (ctl, cand, lead))
            if c is None or k is None or not (math.isfinite(c) and math.isfinite(k)):
                require(d is None, f"{where}: {lead} without two finite losses")
            else:
                require(d is not None and math.isclose(d, c - k, rel_tol=1e-12, abs_tol=1e-12),
                        f"{where}: {lead} is not control minus candidate")
        status, final = r["status"], _float(r["final_validation_loss"], f"{where}/final")
        done = int(r["steps_completed"]) >= int(r["steps_required"])
        if status == "complete":
            require(done and final is not None and math.isfinite(final), f"{where}: complete without an endpoint")
        elif status == "pending":
            require(final is None and int(r["steps_completed"]) == 0, f"{where}: pending with results")
        elif status == "non_finite":
            require(final is None or not math.isfinite(final), f"{where}: non_finite with a finite endpoint")
        elif status == "stopped_early":
            require(r["stopped_early"].strip().lower() == "true", f"{where}: stopped_early flag")
        else:
            require(status == "incomplete", f"{where}: unknown status {status!r}")
        if r["time_scope"]:
            require(r["time_scope"] in ("end_to_end_process", "training_loop"), f"{where}: time scope")
        ratio = _float(r["total_time_ratio_vs_matched_control"], f"{where}/ratio")
        if ratio is not None:
            require(r["time_scope"] == "end_to_end_process", f"{where}: a time ratio needs process times")


def verify_results(root: Path) -> dict:
    root = Path(root)
    out = {}
    for folder in RS.TABLE_DIRS.values():
        d = root / folder
        if not d.is_dir():
            continue
        runs = _csv(d / "runs.csv", RS.RUN_FIELDS)
        _run_checks(folder, runs)
        buf = io.StringIO()
        w = csv.DictWriter(buf, fieldnames=list(RS.SUMMARY_FIELDS), lineterminator="\n")
        w.writeheader()
        w.writerows(RS.summarize(runs))
        _csv(d / "summary.csv", RS.SUMMARY_FIELDS)
        require((d / "summary.csv").read_text(encoding="utf-8") == buf.getvalue(),
                f"{folder}/summary.csv is not the summary of its runs.csv")
        points = _csv(d / "checkpoints.csv", RS.CHECKPOINT_FIELDS)
        listed = {r["run_index"] for r in runs}
        steps = set()
        for i, p in enumerate(points):
            require(p["run_index"] in listed, f"{folder}/checkpoints.csv row {i + 2}: run {p['run_index']} not listed")
            key = (p["run_index"], p["step"])
            require(key not in steps, f"{folder}/checkpoints.csv row {i + 2}: repeated step")
            steps.add(key)
        out[folder] = {"runs": len(runs), "checkpoints": len(points)}
    require(out, f"no result tables under {root}")
    return out


def verify_package(package: Path, results: Path, *, root: Path | None = None, quick: bool = False):
    package, results = Path(package), Path(results)
    manifest_path = package / "activation_optimizer_manifest.csv"
    manifest = verify_manifest(manifest_path)
    matrix = verify_matrix(package / "matrix.json", manifest_path, results)
    fp = verify_fingerprints(package / "token_fingerprints.json", MF.DATASET_ORDER)
    checks = [("activation/optimizer manifest", len(manifest)), ("TILLER matrix", len(matrix["rows"])),
              ("token fingerprint cells", len(fp["cells"]))]
    if quick:
        return checks
    tables = verify_results(results)
    checks.append(("optimizer result directories", len(tables)))
    freeze_path = package / "SOURCE_FREEZE.sha256"
    if root is not None and freeze_path.is_file():
        diff = FZ.check(freeze_path, root, manifests=(), required=())
        require(not any(diff.values()), f"the source freeze is stale: {diff}")
        checks.append(("frozen source files", len(FZ.Freeze.parse(freeze_path.read_text()))))
    return checks


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--package", type=Path, required=True, help="directory with the manifest, matrix, fingerprints")
    ap.add_argument("--results", type=Path, required=True, help="directory of the per-optimizer tables")
    ap.add_argument("--root", type=Path, help="repository root for the source-freeze check")
    ap.add_argument("--quick", action="store_true", help="skip result tables and the freeze")
    a = ap.parse_args(argv)
    try:
        checks = verify_package(a.package, a.results, root=a.root, quick=a.quick)
    except (VerificationError, FZ.FreezeError, RuntimeError, ValueError) as exc:
        print(f"FAIL {exc}", file=sys.stderr)
        return 1
    for label, count in checks:
        print(f"PASS {label}: {count}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
