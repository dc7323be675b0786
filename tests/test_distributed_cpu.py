"""Two-rank CPU (gloo) runs of the trainer: replica equality, failure
detection with host-side fault injection, crash-consistent checkpoints."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from rational_optimizer_b200.train import resume

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _args(tmp_path, run, *extra):
    return ["--allow-cpu", "--dataset-name", "synthetic/zipf", "--dataset-config", "none", "--vocab-size", "256",
            "--max-train-tokens", "20000", "--max-val-tokens", "4000", "--cache-dir", str(tmp_path / "cache"),
            "--output-dir", str(tmp_path / "runs"), "--run-name", run, "--layers", "2", "--d-model", "64",
            "--heads", "16", "--ffn-dim", "128", "--seq-len", "32", "--batch-size", "4", "--steps", "4",
            "--warmup-steps", "1", "--log-interval", "1", "--eval-interval", "2", "--eval-batches", "1",
            "--probe-batch-size", "1", "--matrix-spectrum-interval", "0", "--activation", "grain",
            "--optimizer", "tiller_v1", "--lr", "3e-4", "--dist-timeout-s", "20", "--seed", "11", *extra]


def _launch(tmp_path, run, nproc, *extra, env=None, timeout=240):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(ROOT, "tests", "dist_worker.py"),
           str(tmp_path / run), *_args(tmp_path, run, *extra)]
    e = dict(os.environ, OMP_NUM_THREADS="1")
    e.pop("RO_INJECT_FAULT", None)
    e.update(env or {})
    return subprocess.run(cmd, cwd=ROOT, env=e, capture_output=True, text=True, timeout=timeout)


def _records(tmp_path, run):
    path = tmp_path / "runs" / run / "grain.jsonl"
    return [json.loads(l) for l in path.read_text().splitlines()] if path.exists() else []


def test_two_rank_training_keeps_replicas_identical(tmp_path):
    res = _launch(tmp_path, "dp2", 2)
    assert res.returncode == 0, res.stderr[-3000:]
    digests = [json.loads((tmp_path / f"dp2.rank{r}.json").read_text()) for r in range(2)]
    assert digests[0]["world"] == 2 and digests[0]["digest"] == digests[1]["digest"]
    recs = _records(tmp_path, "dp2")
    assert recs[0]["world_size"] == 2 and recs[0]["global_tokens_per_step"] == 2 * 4 * 32
    assert recs[-1]["event"] == "summary" and recs[-1]["completed_steps"] == 4


def test_failed_rank_stops_the_job(tmp_path):
    res = _launch(tmp_path, "fail", 2, env={"RO_INJECT_FAULT": "train_step:1:3:raise"})
    assert res.returncode != 0
    assert "injected fault" in res.stderr
    recs = _records(tmp_path, "fail")
    assert [r["step"] for r in recs if r["event"] == "train"] == [1, 2]
    assert not any(r["event"] == "summary" for r in recs)


def test_crash_during_checkpoint_commit_recovers(tmp_path):
    ck = tmp_path / "runs" / "crash" / ".exact_resume" / "trainer_state.pt"
    common = ["--resume-checkpoint", str(ck), "--resume-checkpoint-interval", "2", "--strict-exact-resume"]
    res = _launch(tmp_path, "crash", 2, *common, env={"RO_INJECT_FAULT": "checkpoint_written:1:2:exit"})
    assert res.returncode != 0
    assert not ck.exists() and (ck.parent / "trainer_state.pt.tmp").exists()
    traj = tmp_path / "runs" / "crash" / "grain.jsonl"
    out = resume.prepare_trajectory(ck, traj, 2)
    assert out["completed_step"] == 2 and ck.exists()
    res = _launch(tmp_path, "crash", 2, *common)
    assert res.returncode == 0, res.stderr[-3000:]
    recs = _records(tmp_path, "crash")
    assert sum(r["event"] == "resumed" for r in recs) == 1
    assert [r["step"] for r in recs if r["event"] == "train"] == [1, 2, 3, 4]
    ref = _launch(tmp_path, "straight", 2)
    assert ref.returncode == 0
    straight = [r["loss"] for r in _records(tmp_path, "straight") if r["event"] == "train"]
    assert [r["loss"] for r in recs if r["event"] == "train"] == straight


def test_resume_with_another_world_size_is_rejected(tmp_path):
    ck = tmp_path / "ck" / "state.pt"
    common = ["--resume-checkpoint", str(ck), "--resume-checkpoint-interval", "2"]
    assert _launch(tmp_path, "ws", 2, *common).returncode == 0
    assert torch.load(ck, weights_only=False)["contract"]["world_size"] == 2
    res = _launch(tmp_path, "ws1", 1, *common)
    assert res.returncode != 0 and "contract differs" in res.stderr


def test_sharded_muon_ownership_and_state_replication():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(ROOT, "tests", "muon_shard_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=dict(os.environ, OMP_NUM_THREADS="1"), capture_output=True, text=True,
                         timeout=240)
    assert res.returncode == 0, res.stderr[-3000:]
    assert "MUON_STATE_OK 2" in res.stdout
