"""Trainer CLI, token cache, JSONL records and exact resume (CPU)."""
import importlib
import json
import sys

import pytest
import torch

from rational_optimizer_b200.train import resume, tokens, trainer
from rational_optimizer_b200.train.integrity import Manifest, tensor_content_sha256
from reference_oracle import require_reference


def _tiny_args(tmp_path, run_name, *extra):
    return [
        "--allow-cpu", "--dataset-name", "synthetic/zipf", "--dataset-config", "none",
        "--vocab-size", "256", "--max-train-tokens", "20000", "--max-val-tokens", "4000",
        "--cache-dir", str(tmp_path / "cache"), "--output-dir", str(tmp_path / "runs"),
        "--run-name", run_name, "--layers", "2", "--d-model", "64", "--heads", "16",
        "--ffn-dim", "128", "--seq-len", "32", "--batch-size", "4", "--steps", "6",
        "--warmup-steps", "2", "--log-interval", "1", "--eval-interval", "3", "--eval-batches", "2",
        "--probe-batch-size", "2", "--matrix-spectrum-interval", "3", "--seed", "7", *extra,
    ]


def _records(path):
    return [json.loads(line) for line in path.read_text().splitlines()]


def test_parser_defaults_match_reference(monkeypatch):
    refs = require_reference()
    monkeypatch.setattr(sys, "argv", ["train.py"])
    ref = vars(refs["train"].parse_args())
    ours = vars(trainer.reference_namespace(trainer.parse_args([])))
    assert ours == ref


def test_synthetic_corpora_match_reference():
    refs = require_reference()
    ref = refs["train"]
    for name, fn in tokens.TEXT_CORPORA.items():
        for i in list(range(0, 300)) + [50_000_000 + k for k in range(60)]:
            assert fn(i) == ref.synthetic_text_for_dataset(name, i), (name, i)


def test_cache_path_matches_reference(monkeypatch, tmp_path):
    refs = require_reference()
    argv = ["--cache-dir", str(tmp_path), "--train-skip-tokens", "5", "--dataset-revision", "abc"]
    monkeypatch.setattr(sys, "argv", ["train.py", *argv])
    ref_args = refs["train"].parse_args()
    ours = trainer.parse_args(argv)
    for split, n in (("train", 1000), ("validation", None)):
        assert tokens.token_cache_path(ours, split, n) == refs["train"].token_cache_path(ref_args, split, n)
    assert tokens.cache_metadata(ours, "train") == refs["train"]._cache_metadata(ref_args, "train")


def test_token_cache_roundtrip_and_rejections(tmp_path):
    args = trainer.parse_args(["--dataset-name", "synthetic/arithmetic", "--tokenizer", "bytes",
                               "--cache-dir", str(tmp_path), "--seq-len", "16"])
    t = tokens.load_or_tokenize(args, "train", 5000)
    assert t.dtype == torch.int32 and t.numel() == 5000 and int(t.max()) <= 256
    again = tokens.load_or_tokenize(args, "train", 5000)
    assert torch.equal(t, again)
    path = tokens.token_cache_path(args, "train", 5000)
    payload = torch.load(path, weights_only=False)
    assert payload["token_content_sha256"] == tensor_content_sha256(t)
    payload["token_content_sha256"] = "not-a-hash"
    torch.save(payload, path)
    with pytest.raises(RuntimeError, match="token_content_sha256"):
        tokens.load_cached_tokens(path, args, "train", 5000)
    other = trainer.parse_args(["--dataset-name", "synthetic/arithmetic", "--tokenizer", "gpt2",
                                "--cache-dir", str(tmp_path), "--seq-len", "16"])
    with pytest.raises(RuntimeError, match="tokenizer"):
        tokens.load_cached_tokens(path, other, "train", 5000)


def test_protocol_validation():
    bad = [
        (["--optimizer", "tiller_v1"], "requires the GRAIN activation"),
        (["--sam-rho", "0.1"], "SAM"),
        (["--experiment-identity", "tiller_matrix_v1"], "exact LR/WD contract"),
        (["--fairness-contract", "exact_lr_wd_v1", "--min-lr", "1", "--lr", "0.1"], "min_lr"),
    ]
    for argv, message in bad:
        with pytest.raises(ValueError, match=message):
            trainer.validate_optimizer_protocol(trainer.parse_args(argv))


@pytest.mark.parametrize("optimizer,activation", [("adamw", "silu"), ("tiller_v1", "grain"),
                                                  ("lion", "grain")])
def test_cpu_run_writes_reference_records(tmp_path, optimizer, activation):
    argv = _tiny_args(tmp_path, "r", "--optimizer", optimizer, "--activation", activation,
                      "--fairness-contract", "exact_lr_wd_v1")
    if optimizer == "tiller_v1":
        argv += ["--lr", "3e-4"]
    assert trainer.main(argv) == 0
    recs = _records(tmp_path / "runs" / "r" / f"{activation}.jsonl")
    events = [r["event"] for r in recs]
    assert events[0] == "config" and events[-1] == "summary"
    assert events.count("train") == 6 and events.count("eval") == 3
    cfg = recs[0]
    assert cfg["optimizer_lr_wd_fairness"]["passed"] is True
    assert cfg["global_tokens_per_step"] == 4 * 32
    train = [r for r in recs if r["event"] == "train"]
    assert all(torch.isfinite(torch.tensor(r["loss"])) for r in train)
    summary = recs[-1]
    assert summary["completed_steps"] == 6 and summary["realized_lr_audit_steps"] == 6
    ev = [r for r in recs if r["event"] == "eval"][-1]
    assert "probe_kl_since_step1" in ev and "svd_entropy_attn_q" in ev


def test_exact_resume_is_bitwise(tmp_path):
    ck = tmp_path / "ck" / "state.pt"
    common = ["--optimizer", "tiller_v1", "--activation", "grain", "--lr", "3e-4",
              "--resume-checkpoint", str(ck), "--resume-checkpoint-interval", "3"]
    assert trainer.main(_tiny_args(tmp_path, "full", *common)) == 0
    full = [r for r in _records(tmp_path / "runs" / "full" / "grain.jsonl") if r["event"] == "train"]
    assert ck.is_file() and Manifest.path_for(ck).is_file()
    assert torch.load(ck, weights_only=False)["completed_step"] == 3
    assert trainer.main(_tiny_args(tmp_path, "resumed", *common)) == 0
    recs = _records(tmp_path / "runs" / "resumed" / "grain.jsonl")
    assert recs[0]["event"] == "resumed" and recs[0]["step"] == 3
    tail = [r for r in recs if r["event"] == "train"]
    assert [r["step"] for r in tail] == [4, 5, 6]
    for a, b in zip(full[3:], tail):
        assert a["loss"] == b["loss"] and a["grad_global_norm_before_clip"] == b["grad_global_norm_before_clip"]


def test_crash_between_promotion_and_manifest_still_resumes(tmp_path, monkeypatch):
    """A save that stops after its files are promoted but before the new manifest
    is written leaves no stale manifest behind, so the run resumes from it."""
    from rational_optimizer_b200.utils import faults
    ck = tmp_path / "ck" / "state.pt"
    common = ["--optimizer", "adamw", "--resume-checkpoint", str(ck), "--resume-checkpoint-interval", "2",
              "--eval-interval", "2"]  # checkpoints are written at evaluation steps 2 and 4
    monkeypatch.setenv(faults.ENV, "checkpoint_promoted:0:4:raise")
    with pytest.raises(faults.InjectedFault):
        trainer.main(_tiny_args(tmp_path, "a", *common))
    monkeypatch.delenv(faults.ENV)
    assert torch.load(ck, weights_only=False)["completed_step"] == 4
    assert not Manifest.path_for(ck).is_file()  # the step-2 manifest is gone, not stale
    assert trainer.main(_tiny_args(tmp_path, "b", *common)) == 0
    recs = _records(tmp_path / "runs" / "b" / "silu.jsonl")
    assert recs[0]["event"] == "resumed" and recs[0]["step"] == 4


def test_resume_rejects_changed_contract_and_corruption(tmp_path):
    ck = tmp_path / "ck" / "state.pt"
    common = ["--optimizer", "adamw", "--resume-checkpoint", str(ck), "--resume-checkpoint-interval", "3"]
    assert trainer.main(_tiny_args(tmp_path, "a", *common)) == 0
    with pytest.raises(RuntimeError, match="contract differs"):
        trainer.main(_tiny_args(tmp_path, "b", *common, "--lr", "1e-3"))
    raw = bytearray(ck.read_bytes())
    raw[len(raw) // 2] ^= 0xFF
    ck.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="differs from its manifest"):
        trainer.main(_tiny_args(tmp_path, "c", *common))


def test_recover_interrupted_commit_and_trajectory(tmp_path):
    path = tmp_path / "state.pt"
    for step, suffix in ((3, ""), (6, ".tmp")):
        torch.save({"schema": resume.MAIN_SCHEMA, "completed_step": step}, f"{path}{suffix}")
        for r in range(2):
            torch.save({"schema": resume.RANK_SCHEMA, "completed_step": step, "rank": r},
                       f"{path}.rank{r}.pt{suffix}")
    # rank 1's step-6 payload never reached disk: generation 6 is incomplete
    (tmp_path / "state.pt.rank1.pt.tmp").unlink()
    assert resume.recover_interrupted_commit(path, 2) == 3
    torch.save({"schema": resume.RANK_SCHEMA, "completed_step": 6, "rank": 1}, f"{path}.rank1.pt.tmp")
    assert resume.recover_interrupted_commit(path, 2) == 6
    assert torch.load(path, weights_only=False)["completed_step"] == 6
    traj = tmp_path / "run.jsonl"
    lines = [{"event": "config"}] + [{"event": "train", "step": s} for s in range(1, 9)] + [{"event": "summary"}]
    traj.write_text("\n".join(json.dumps(l) for l in lines) + "\n")
    out = resume.prepare_trajectory(path, traj, 2)
    assert out["mode"] == "resume" and out["completed_step"] == 6 and out["removed_records"] == 3
    kept = [json.loads(l) for l in traj.read_text().splitlines()]
    assert [r.get("step") for r in kept] == [None, 1, 2, 3, 4, 5, 6]


def test_strict_resume_path_and_interval(tmp_path):
    argv = ["--output-dir", str(tmp_path), "--run-name", "x", "--eval-interval", "5",
            "--resume-checkpoint-interval", "5", "--strict-exact-resume"]
    good = trainer.parse_args(argv + ["--resume-checkpoint",
                                      str(tmp_path / "x" / ".exact_resume" / "trainer_state.pt")])
    trainer.validate_optimizer_protocol(good)
    with pytest.raises(ValueError, match="run-local checkpoint"):
        trainer.validate_optimizer_protocol(trainer.parse_args(argv + ["--resume-checkpoint", str(tmp_path / "y.pt")]))


def test_lr_trace_digest_matches_reference():
    refs = require_reference()
    er = importlib.import_module("training.exact_resume")
    args = trainer.parse_args(["--steps", "50", "--warmup-steps", "7", "--lr", "0.01", "--min-lr", "0.001"])
    assert resume.full_lr_trace_digest(args) == er.full_lr_trace_digest(args)
    ref_ns = trainer.reference_namespace(args)
    assert resume.complete_argument_digest(ref_ns) == er.complete_argument_digest(ref_ns)


def test_aggregate_matches_reference(tmp_path):
    refs = require_reference()
    agg_ref = importlib.import_module("training.aggregate_results")
    from rational_optimizer_b200.train import aggregate
    for act, opt in (("silu", "adamw"), ("grain", "adamw"), ("grain", "lion")):
        assert trainer.main(_tiny_args(tmp_path, "agg", "--activation", act, "--optimizer", opt,
                                       "--steps", "3")) == 0
    run_dir = tmp_path / "runs" / "agg"
    ours = aggregate.build_rows(aggregate.parse_run_dir(run_dir), "silu", "", "adamw")
    ref = agg_ref.build_rows(agg_ref.parse_run_dir(run_dir), "silu", "", "adamw")
    import math as _m
    for a_rows, b_rows in zip(ours, ref):
        assert len(a_rows) == len(b_rows) > 0
        for a, b in zip(a_rows, b_rows):
            assert list(a) == list(b)
            for k in a:
                if isinstance(a[k], float) and _m.isnan(a[k]):
                    assert _m.isnan(b[k])
                else:
                    assert a[k] == b[k], k
    out = tmp_path / "out"
    aggregate.main(["--run-dir", str(run_dir), "--out-dir", str(out)])
    assert (out / "per_seed.csv").is_file() and (out / "README.md").is_file()
