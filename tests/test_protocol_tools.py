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
