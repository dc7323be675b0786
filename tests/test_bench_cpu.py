"""bench.py helpers that run without a GPU: the reference arm's self-install."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_present_needs_no_install(tmp_path, monkeypatch):
    ref = tmp_path / "_ref"
    (ref / "training").mkdir(parents=True)
    monkeypatch.setattr(bench, "REF_DIR", str(ref))
    monkeypatch.setattr(bench, "REF_SRC", str(tmp_path / "no-such-source"))
    assert bench.ensure_reference() is None


def test_reference_missing_without_source_reports_why(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "REF_DIR", str(tmp_path / "baseline" / "_ref"))
    monkeypatch.setattr(bench, "REF_SRC", str(tmp_path / "no-such-source"))
    reason = bench.ensure_reference()
    assert reason is not None and "no reference source" in reason
    assert not os.path.exists(tmp_path / "baseline" / "_ref" / "training")


def test_reference_install_failure_is_reported(tmp_path, monkeypatch):
    """A source tree pip cannot install gives a one-line reason, not an exception."""
    src = tmp_path / "src"
    src.mkdir()
    (src / "README").write_text("not a Python project\n")
    monkeypatch.setattr(bench, "REF_DIR", str(tmp_path / "baseline" / "_ref"))
    monkeypatch.setattr(bench, "REF_SRC", str(src))
    reason = bench.ensure_reference()
    assert reason is not None and reason.startswith("reference install failed")
    assert "\n" not in reason
