"""Protocol tooling against the reference's own data and tools (CPU)."""
import json
import os

import pytest

from reference_oracle import REF, require_reference
from rational_optimizer_b200.protocol import matrix as MX

PROTO = os.path.join(REF, "experiments", "protocol")
RESULTS = os.path.join(REF, "experiments", "results")


def _need_data():
    require_reference()
    if not os.path.isfile(os.path.join(PROTO, "activation_optimizer_manifest.csv")):
        pytest.skip("the reference's protocol data files are not beside the installed package")


def test_matrix_rebuilds_the_reference_matrix():
    _need_data()
    ours = MX.build_matrix(os.path.join(PROTO, "activation_optimizer_manifest.csv"), RESULTS)
    with open(os.path.join(PROTO, "matrix.json")) as fh:
        theirs = json.load(fh)
    assert {k: v for k, v in ours.items() if k != "rows"} == {k: v for k, v in theirs.items() if k != "rows"}
    assert len(ours["rows"]) == len(theirs["rows"]) == 60
    for a, b in zip(ours["rows"], theirs["rows"]):
        # the timing condition names the hardware the matrix is run on
        assert a["timing_condition"] == MX.DEFAULT_TIMING
        a = dict(a, timing_condition=b["timing_condition"])
        assert a == b


def test_matrix_rejects_incomplete_cells(tmp_path):
    _need_data()
    rows = MX.read_manifest(os.path.join(PROTO, "activation_optimizer_manifest.csv"))
    keep = [r for r in rows if not (r["phase"] == MX.TWO_STAGE_SUITE and r["seed"] == "2027")]
    path = tmp_path / "m.csv"
    import csv
    with path.open("w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=list(rows[0]))
        w.writeheader()
        w.writerows(keep)
    with pytest.raises(ValueError, match="5 datasets x 3 seeds"):
        MX.build_matrix(path, RESULTS)


def test_manifest_reproduces_the_reference_csv(tmp_path):
    _need_data()
    from rational_optimizer_b200.protocol import manifest as MF
    rows = MF.build_rows()
    MF.check_matched_arms(rows)
    out = tmp_path / "m.csv"
    MF.write(rows, out)
    with open(os.path.join(PROTO, "activation_optimizer_manifest.csv"), "rb") as fh:
        assert out.read_bytes() == fh.read()


def test_manifest_check_rejects_unpaired_arms():
    from rational_optimizer_b200.protocol import manifest as MF
    rows = MF.build_rows()
    broken = [dict(r) for r in rows]
    victim = next(r for r in broken if r["method"] == "rlb_muon" and r["phase"] == MF.L100)
    victim["lr"] = "0.001"
    with pytest.raises(ValueError, match="differ beyond the activation"):
        MF.check_matched_arms(broken)
    with pytest.raises(ValueError, match="lacks"):
        MF.check_matched_arms([r for r in rows if r["method"] != "silu_came"])


def _git_repo(tmp_path):
    import subprocess
    root = tmp_path / "repo"
    (root / "pkg").mkdir(parents=True)
    (root / "pkg" / "a.py").write_text("x = 1\n")
    (root / "pkg" / "k.cu").write_text("// kernel\n")
    (root / "setup.py").write_text("print()\n")
    (root / "notes.txt").write_text("not a source\n")
    (root / "weights.pt").write_bytes(b"\0" * 8)
    (root / "experiments" / "results").mkdir(parents=True)
    (root / "experiments" / "results" / "r.py").write_text("# results are never frozen\n")
    (root / ".gitignore").write_text("ignored.py\n")
    (root / "ignored.py").write_text("x = 2\n")
    subprocess.run(["git", "init", "-q", str(root)], check=True)
    return root


def test_source_freeze_matches_sha256sum_format_and_detects_drift(tmp_path):
    import hashlib
    from rational_optimizer_b200.protocol import freeze as FZ
    root = _git_repo(tmp_path)
    out = root / "SOURCE_FREEZE.sha256"
    assert FZ.main(["--root", str(root), "--output", str(out)]) == 0
    text = out.read_text()
    listed = [line.split("  ", 1)[1] for line in text.splitlines()]
    assert listed == ["pkg/a.py", "pkg/k.cu", "setup.py"]
    for line in text.splitlines():
        digest, rel = line.split("  ", 1)
        assert digest == hashlib.sha256((root / rel).read_bytes()).hexdigest()
    assert FZ.main(["--root", str(root), "--output", str(out), "--check"]) == 0
    (root / "pkg" / "a.py").write_text("x = 3\n")
    (root / "pkg" / "b.py").write_text("y = 1\n")
    assert FZ.check(out, root) == {"added": ["pkg/b.py"], "removed": [], "changed": ["pkg/a.py"]}
    assert FZ.main(["--root", str(root), "--output", str(out), "--check"]) == 1


def test_source_freeze_agrees_with_the_reference_tool(tmp_path, monkeypatch):
    """The reference tool's selection rules on the same tree give the same lines
    (its required-file list is satisfied by creating those files)."""
    import importlib
    _need_data()
    ref = importlib.import_module("experiments.protocol.build_source_freeze")
    root = _git_repo(tmp_path)
    for rel in sorted(ref.MANIFESTS) + ["experiments/protocol/build_source_freeze.py",
                                        "experiments/protocol/test_suite.py",
                                        "experiments/protocol/verify_repository.py",
                                        "optimizer_design/tiller.py", "training/train.py"]:
        (root / rel).parent.mkdir(parents=True, exist_ok=True)
        (root / rel).write_text(f"# {rel}\n")
    monkeypatch.setattr(ref, "ROOT", root)
    monkeypatch.setattr(ref, "OUTPUT", root / "experiments" / "protocol" / "SOURCE_FREEZE.sha256")
    theirs = ref.render_freeze(root)
    from rational_optimizer_b200.protocol import freeze as FZ
    ours = FZ.Freeze.collect(root, manifests=ref.MANIFESTS,
                             output="experiments/protocol/SOURCE_FREEZE.sha256").render()
    assert ours == theirs


def _arm_records(row, arm, losses, *, lr_digest="d" * 64, fingerprint="f" * 64, seconds=100.0):
    from rational_optimizer_b200.protocol import rows as R
    side = "control" if arm == "control" else "candidate"
    cfg = {"event": "config", "activation": row[f"{side}_activation"], "optimizer": row[f"{side}_optimizer"],
           "dataset": row["dataset_name"], "dataset_config": row["dataset_config"],
           "dataset_revision": row["dataset_revision"], "tokenizer": row["tokenizer"],
           "tokenizer_revision": row["tokenizer_revision"], "steps": row["steps"], "seed": row["seed"],
           "train_tokens": row["max_train_tokens"], "val_tokens": row["max_val_tokens"],
           "optimizer_lr_wd_fairness": {"passed": True, "base_lr": row["lr"], "minimum_lr": row["min_lr"],
                                        "base_weight_decay": row["weight_decay"],
                                        "groups": [{"group_index": 0, "lr_scale": 1.0, "weight_decay": 0.1}]},
           "train_token_sample_sha256": fingerprint, "val_token_sample_sha256": "v" * 64,
           "first_batch_index_sha256": "b" * 64, "validation_index_sha256": "i" * 64}
    if arm == "candidate":
        cfg["experiment_identity"] = R.experiment_identity(row)
        cfg["tiller_experiment_identity"] = {"passed": True, "matrix_index": row["matrix_index"],
                                             "source_manifest_row_index": row["source_manifest_row_index"],
                                             "source_manifest_row_id": row["source_manifest_row_id"]}
    recs = [cfg] + [{"event": "eval", "step": s, "val_loss": v} for s, v in losses.items()]
    recs.append({"event": "summary", "realized_lr_audit_steps": row["steps"],
                 "realized_lr_trace_sha256": lr_digest, "total_seconds": seconds})
    return recs


def _write_jsonl(path, recs):
    path.write_text("".join(json.dumps(r) + "\n" for r in recs))
    return path


def test_endpoint_analysis_and_aggregate(tmp_path):
    from test_protocol import _row
    from rational_optimizer_b200.protocol import analyze as AN
    row = _row()
    ctrl = _write_jsonl(tmp_path / "c.jsonl", _arm_records(row, "control", {1000: 4.5, 3050: 4.29}, seconds=100.0))
    cand = _write_jsonl(tmp_path / "k.jsonl", _arm_records(row, "candidate", {1000: 4.4, 3050: 4.22}, seconds=104.0))
    res = AN.endpoint_result(row, ctrl, cand)
    assert res["status"] == "complete" and res["schema"] == AN.SCHEMA
    assert abs(res["absolute_endpoint_lead"] - 0.07) < 1e-12 and abs(res["step1000_absolute_lead"] - 0.1) < 1e-12
    assert abs(res["exact_matched_hardware_end_to_end_total_time_ratio"] - 1.04) < 1e-12
    assert res["passes_final_1_05_time_gate"] and res["time_scope"] == "training_loop"
    AN.write_result(tmp_path / "r.json", res)
    assert (tmp_path / "r.json.sha256").read_text().split()[0] == AN._sha(tmp_path / "r.json")
    # a candidate that trails at the screen step is an invalid (uninterrupted) row
    bad = _write_jsonl(tmp_path / "k2.jsonl", _arm_records(row, "candidate", {1000: 4.6, 3050: 4.2}))
    assert AN.endpoint_result(row, ctrl, bad)["status"] == "invalid_not_interrupted"
    summary = AN.aggregate([res, AN.endpoint_result(row, ctrl, bad)])
    g = summary["groups"][0]
    assert g["rows"] == 2 and g["complete_rows"] == 1 and g["candidate_endpoint_wins"] == 1
    # different data order or LR schedule between the arms is rejected
    other = _write_jsonl(tmp_path / "k3.jsonl", _arm_records(row, "candidate", {1000: 4.4, 3050: 4.2},
                                                              fingerprint="0" * 64))
    with pytest.raises(RuntimeError, match="same data"):
        AN.endpoint_result(row, ctrl, other)
    sched = _write_jsonl(tmp_path / "k4.jsonl", _arm_records(row, "candidate", {1000: 4.4, 3050: 4.2},
                                                              lr_digest="e" * 64))
    with pytest.raises(RuntimeError, match="LR schedule"):
        AN.endpoint_result(row, ctrl, sched)
    missing = _write_jsonl(tmp_path / "k5.jsonl", _arm_records(row, "candidate", {1000: 4.4}))
    with pytest.raises(RuntimeError, match="lacks evaluations"):
        AN.endpoint_result(row, ctrl, missing)


def test_fairness_audit_of_both_arms():
    from test_protocol import _row
    from rational_optimizer_b200.protocol import fairness as FA
    row = _row()
    row.update(layers=2, d_model=128, heads=4, ffn_dim=256)  # the audit logic, not the size, is under test
    payload = FA.audit_rows([row])
    assert payload["schema"] == FA.SCHEMA and payload["passed"] is True
    arms = {r["arm"]: r for r in payload["reports"]}
    assert arms["control"]["optimizer"] == "muon" and arms["candidate"]["optimizer"] == "tiller_v1"
    assert all(r["covered_parameter_elements"] == r["trainable_parameter_elements"] for r in payload["reports"])


def test_results_summary_reproduces_every_published_summary_table():
    """summary.csv of each optimizer, recomputed from its published runs.csv, byte for byte."""
    import csv
    import io
    from rational_optimizer_b200.protocol import results as RS
    _need_data()
    tables = [d for d in sorted(os.listdir(RESULTS)) if os.path.isfile(os.path.join(RESULTS, d, "runs.csv"))]
    assert set(tables) == set(RS.TABLE_DIRS.values())
    for d in tables:
        with open(os.path.join(RESULTS, d, "runs.csv"), newline="") as fh:
            reader = csv.DictReader(fh)
            assert tuple(reader.fieldnames) == RS.RUN_FIELDS
            runs = list(reader)
        buf = io.StringIO()
        w = csv.DictWriter(buf, fieldnames=list(RS.SUMMARY_FIELDS), lineterminator="\n")
        w.writeheader()
        w.writerows(RS.summarize(runs))
        with open(os.path.join(RESULTS, d, "summary.csv"), newline="") as fh:
            assert buf.getvalue() == fh.read(), d
        with open(os.path.join(RESULTS, d, "checkpoints.csv"), newline="") as fh:
            assert tuple(csv.DictReader(fh).fieldnames) == RS.CHECKPOINT_FIELDS


def _write_run(path, *, steps, losses, summary=True, stopped=False, torn=False, tps=1000.0):
    import json
    path.parent.mkdir(parents=True, exist_ok=True)
    recs = [{"event": "config", "optimizer_lr_wd_fairness": {"passed": True}, "slurm_job_id": "7"}]
    recs += [{"event": "eval", "step": s, "val_loss": v, "val_ppl": 2.0 ** v, "active_seconds_at_val_loss": s / 10}
             for s, v in losses.items()]
    if stopped:
        recs.append({"event": "stopped_early", "step": max(losses)})
    if summary:
        recs.append({"event": "summary", "completed_steps": max(losses), "stopped_early": stopped,
                     "total_seconds": 50.0, "mean_seconds_per_step": 0.01, "tokens_per_second": tps,
                     "realized_lr_trace_sha256": "ab" * 32, "slurm_job_id": "7"})
    text = "".join(json.dumps(r) + "\n" for r in recs)
    if torn:
        text += '{"event": "train", "st'
    path.write_text(text)


def test_results_tables_from_trainer_jsonl(tmp_path):
    import csv
    import json
    from rational_optimizer_b200.protocol import results as RS
    manifest = []
    for i, (act, loss) in enumerate((("silu", 4.0), ("rlb_fused_global_rational", 3.9))):
        manifest.append({"row_index": str(i), "row_id": f"r{i}", "phase": "12l_768d_100m_tokens_3050_steps",
                         "model": "12l_768d", "dataset": "c4_en", "seed": "1337", "train_tokens": "100",
                         "steps": "20", "activation": act, "optimizer": "muon", "method": f"{act}_muon"})
    runs = tmp_path / "runs"
    for m, loss in zip(manifest, (4.0, 3.9)):
        _write_run(runs / m["phase"] / m["dataset"] / m["row_id"] / f"{m['activation']}.jsonl",
                   steps=20, losses={10: loss + 1, 20: loss}, torn=m["activation"] == "silu")
    # the GRAIN arm's launcher recorded its process time
    grain = runs / manifest[1]["phase"] / "c4_en" / "r1" / "rlb_fused_global_rational.wall_clock.json"
    grain.write_text(json.dumps({"schema": "rationalopt_process_wall_clock_v1", "return_code": 0,
                                 "elapsed_seconds": 60.0}))
    by_opt, points = RS.manifest_tables(manifest, runs)
    silu, g = by_opt["muon"]
    assert silu["status"] == g["status"] == "complete"
    assert silu["time_scope"] == "training_loop" and g["time_scope"] == "end_to_end_process"
    assert g["total_seconds"] == 60.0 and g["training_loop_total_seconds"] == 50.0
    assert abs(g["lead_vs_matched_control"] - 0.1) < 1e-12 and g["matched_control_total_seconds"] == 50.0
    assert g["total_time_ratio_vs_matched_control"] == ""  # the control has no process time
    assert g["method_display_name"] == "GRAIN + Muon" and len(points["muon"]) == 4
    out = RS.publish(tmp_path / "tables", "muon", by_opt["muon"], points["muon"])
    with (out / "summary.csv").open() as fh:
        cells = list(csv.DictReader(fh))
    assert [c["status"] for c in cells] == ["complete", "complete"]
    assert cells[0]["activation"] == "rlb_fused_global_rational" and cells[0]["lead_vs_matched_control_mean"]


def test_results_run_states(tmp_path):
    from rational_optimizer_b200.protocol import results as RS
    spec = dict(run_index=3, model="18l_1024d", dataset="dclm", seed=1337, train_tokens=10, steps=20,
                activation="rlb_fused_global_rational", optimizer="tiller_v1", method="tiller",
                phase="p", source_row_index=3, source_row_id="x")
    assert RS.run_record(spec, tmp_path / "none.jsonl")[0]["status"] == "pending"
    p = tmp_path / "a.jsonl"
    _write_run(p, steps=20, losses={10: 5.0}, summary=False)
    row, _ = RS.run_record(spec, p)
    assert row["status"] == "incomplete" and row["steps_completed"] == 10
    _write_run(p, steps=20, losses={10: 5.0, 20: float("nan")})
    assert RS.run_record(spec, p)[0]["status"] == "non_finite"
    _write_run(p, steps=20, losses={10: 5.0}, stopped=True)
    assert RS.run_record(spec, p)[0]["status"] == "stopped_early"
    _write_run(p, steps=20, losses={10: 5.0, 20: 4.0})
    (tmp_path / "a.wall_clock.json").write_text('{"schema": "rationalopt_process_wall_clock_v1", '
                                                 '"return_code": 1, "elapsed_seconds": 9.0}')
    row, _ = RS.run_record(spec, p)
    assert row["status"] == "incomplete" and row["final_validation_loss"] == ""
    p.write_text('{"event": "config"}\nnot json\n{"event": "summary"}\n')
    with pytest.raises(RS.ResultsError):
        RS.run_record(spec, p)
    cells = RS.summarize([dict(RS.run_record(spec, tmp_path / "none.jsonl")[0])])
    assert cells[0]["status"] == "pending" and cells[0]["validation_loss_mean"] == ""


def test_results_matrix_candidates_pair_with_their_control(tmp_path):
    import json
    from rational_optimizer_b200.protocol import results as RS
    from rational_optimizer_b200.protocol import rows as R
    _need_data()
    matrix = R.load_matrix(os.path.join(PROTO, "matrix.json"))
    row = matrix["rows"][0]
    steps = int(row["steps"])
    small = {"rows": [row]}
    runs, analysis = tmp_path / "runs", tmp_path / "analysis"
    got, _ = RS.matrix_tables(small, runs, analysis)
    assert got[0]["status"] == "pending" and got[0]["optimizer"] == row["candidate_optimizer"]
    _write_run(R.jsonl_path(row, "candidate", runs), steps=steps, losses={1000: 5.0, steps: 4.0})
    got, pts = RS.matrix_tables(small, runs, analysis)
    published = row["matched_control"]["endpoint_validation_loss"]
    assert got[0]["status"] == "complete" and len(pts) == 2
    assert abs(got[0]["lead_vs_matched_control"] - (published - 4.0)) < 1e-12
    # a negative step-1,000 screen stops the run
    screen = runs / f"{R.run_name(row, 'candidate')}.step1000.json"
    screen.write_text(json.dumps({"matrix_index": row["matrix_index"], "status": "failed_negative_interrupted",
                                  "candidate_step1000_loss": 5.0}))
    got, _ = RS.matrix_tables(small, runs, analysis)
    assert got[0]["status"] == "stopped_early" and got[0]["final_validation_loss"] == ""
    # an endpoint result beside a stopped screen is a contradiction
    (analysis / f"row-{row['matrix_index']:02d}").mkdir(parents=True)
    (analysis / f"row-{row['matrix_index']:02d}" / "RESULT.json").write_text(json.dumps({
        "schema": "tiller_matched_endpoint_result_v1", "status": "complete", "matrix_index": row["matrix_index"],
        "model": row["model"], "dataset": row["dataset"], "seed": int(row["seed"]), "steps": steps}))
    with pytest.raises(RS.ResultsError):
        RS.matrix_tables(small, runs, analysis)


def test_verify_passes_on_the_published_package_and_catches_edits(tmp_path):
    import shutil
    from rational_optimizer_b200.protocol import verify as V
    _need_data()
    checks = dict(V.verify_package(PROTO, RESULTS))
    assert checks["activation/optimizer manifest"] == 640 and checks["TILLER matrix"] == 60
    assert checks["optimizer result directories"] == 8
    results = tmp_path / "results"
    shutil.copytree(RESULTS, results)
    runs = results / "tiller" / "runs.csv"
    original = runs.read_text()
    lines = original.splitlines(keepends=True)
    cells = lines[1].split(",")
    i = lines[0].split(",").index("lead_vs_matched_control")
    cells[i] = str(float(cells[i]) + 1e-3)
    runs.write_text(lines[0] + ",".join(cells) + "".join(lines[2:]))
    with pytest.raises(V.VerificationError, match="control minus candidate"):
        V.verify_results(results)
    runs.write_text(original)
    summary = results / "muon" / "summary.csv"
    summary.write_text(summary.read_text().replace("complete", "pending", 1))
    with pytest.raises(V.VerificationError, match="summary of its runs"):
        V.verify_results(results)
    package = tmp_path / "package"
    shutil.copytree(PROTO, package)
    manifest = package / "activation_optimizer_manifest.csv"
    manifest.write_text(manifest.read_text().replace("3407", "3408", 1))
    with pytest.raises(V.VerificationError):
        V.verify_package(package, RESULTS, quick=True)


def _flag_map(argv):
    out, i = {}, 0
    while i < len(argv):
        a = argv[i]
        if i + 1 < len(argv) and not argv[i + 1].startswith("--"):
            out[a] = argv[i + 1]
            i += 2
        else:
            out[a] = True
            i += 1
    return out


def test_sweep_row_argv_matches_the_reference_row_runner(tmp_path):
    import importlib
    from rational_optimizer_b200.protocol import rows as R
    from rational_optimizer_b200.protocol import sweep as SW
    _need_data()
    ref = importlib.import_module("experiments.protocol.run_activation_row")
    manifest = R.load_manifest(os.path.join(PROTO, "activation_optimizer_manifest.csv"))
    for row in manifest[::53]:
        theirs = _flag_map(ref.training_arguments(row, tmp_path)[1:])
        theirs.pop("--hf-cache")
        assert _flag_map(SW.training_argv(row, tmp_path)) == theirs, row["row_id"]
        assert SW.trajectory_path(row, tmp_path) == ref.result_path(row, tmp_path)
        assert SW.row_sha256(row) == ref.row_sha256(row)
    # re-derived for 8 GPUs at the same global tokens per step
    row = manifest[12]
    flags = _flag_map(SW.training_argv(row, tmp_path, gpus=8))
    assert int(flags["--batch-size"]) * int(flags["--grad-accum"]) * 8 * int(row["seq_len"]) == int(
        row["global_tokens_per_step"])


def test_sweep_accepts_only_a_matching_finished_trajectory(tmp_path):
    import json
    from rational_optimizer_b200.protocol import rows as R
    from rational_optimizer_b200.protocol import sweep as SW
    _need_data()
    manifest_path = os.path.join(PROTO, "activation_optimizer_manifest.csv")
    row = R.load_manifest(manifest_path)[12]
    identity = SW.source_identity(manifest_path, row, os.path.join(PROTO, "SOURCE_FREEZE.sha256"))
    cfg = {"event": "config", **identity, "experiment_identity": "none",
           "optimizer_lr_wd_fairness": {"contract": "exact_lr_wd_v1", "passed": True, "base_lr": float(row["lr"]),
                                        "minimum_lr": float(row["min_lr"]),
                                        "base_weight_decay": float(row["weight_decay"])}}
    cfg.update({k: row[c] for k, c in SW.EXACT_FIELDS})
    cfg.update({k: int(row[c]) for k, c in SW.INTEGER_FIELDS})
    cfg.update({k: float(row[c]) for k, c in SW.NUMBER_FIELDS})
    path = SW.trajectory_path(row, tmp_path)
    path.parent.mkdir(parents=True)

    def write(config, steps):
        path.write_text(json.dumps(config) + "\n" + json.dumps({"event": "summary", "completed_steps": steps}) + "\n")

    write(cfg, int(row["steps"]))
    assert SW.matches(path, row, identity)
    write(cfg, int(row["steps"]) - 1)
    assert not SW.matches(path, row, identity)
    write(dict(cfg, optimizer_lr=1e-3), int(row["steps"]))
    assert not SW.matches(path, row, identity)
    write(dict(cfg, source_freeze_sha256="0" * 64), int(row["steps"]))
    assert not SW.matches(path, row, identity)
    moved = SW.archive(path)
    assert moved.name.startswith(f"{row['activation']}.superseded-") and not path.exists()
