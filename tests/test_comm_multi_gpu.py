"""Peer-memory all-reduce across GPUs (one process per GPU, torchrun)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs at least two GPUs")
def test_p2p_allreduce_matches_nccl():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29517",
           os.path.join(ROOT, "tests", "comm_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert f"COMM_OK {n}" in res.stdout


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs at least two GPUs")
def test_overlapped_sharded_training_matches_replicated():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29518",
           os.path.join(ROOT, "tests", "train_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert f"TRAIN_OK {n}" in res.stdout
    assert "OWNER_OK" in res.stdout
    assert "PULL_OK" in res.stdout
    assert "MUON_SHARD_OK" in res.stdout
    assert "INT8_OK" in res.stdout
    assert "FUSED_WGRAD_OK" in res.stdout
    assert "COPY_ENGINE_OK" in res.stdout


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs at least two GPUs")
def test_transport_smoke():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29519",
           "-m", "rational_optimizer_b200.protocol.smoke"]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    line = [l for l in res.stdout.splitlines() if l.startswith("{")][-1]
    import json
    out = json.loads(line)
    assert out["passed"] is True and out["world_size"] == n
