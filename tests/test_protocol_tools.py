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
