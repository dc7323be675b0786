"""Run one arm of a matrix row on this node and record its wall clock.

    python -m rational_optimizer_b200.protocol.launch --matrix PATH --index I --arm candidate \\
        --output-root RUNS [--gpus 8] [--max-batch-per-gpu B] [--timeout-s S]

One process per GPU through ``torch.distributed.run`` on 127.0.0.1; the row's
batch and accumulation are re-derived for ``--gpus`` at the row's global
tokens per step.  Each child installs the row's identity auditor before the
trainer parses its flags.  The launcher writes a
``rationalopt_process_wall_clock_v1`` record (reference
experiments/protocol/run_timed.py:29-74) and, on a non-zero exit, a
``tiller_row_failure_v1`` record (reference record_failure.py:12-53) that
separates a negative step-1,000 screen from retryable execution failures.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import signal
import subprocess
import sys
import time
from datetime import datetime, timezone
from pathlib import Path

from . import rows as R


def utc_now() -> str:
    return datetime.now(timezone.utc).isoformat()


def write_atomic(path: Path, payload: dict) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n")
    os.replace(tmp, path)


def run_timed(command, output: Path, arm: str, *, timeout_s: float | None = None) -> int:
    """Run ``command``, forward SIGINT/SIGTERM to it, record its wall time."""
    if not command:
        raise ValueError("a command is required")
    if not str(arm).strip():
        raise ValueError("arm must be non-empty")
    started_utc, t0 = utc_now(), time.monotonic_ns()
    proc = subprocess.Popen(list(command))

    def forward(signum, _frame):
        if proc.poll() is None:
            proc.send_signal(signum)

    previous = {s: signal.signal(s, forward) for s in (signal.SIGINT, signal.SIGTERM)}
    try:
        try:
            rc = proc.wait(timeout=timeout_s)
        except subprocess.TimeoutExpired:
            proc.terminate()
            try:
                rc = proc.wait(timeout=60)
            except subprocess.TimeoutExpired:
                proc.kill()
                rc = proc.wait()
    finally:
        for s, h in previous.items():
            signal.signal(s, h)
    write_atomic(output, {
        "schema": "rationalopt_process_wall_clock_v1", "arm": arm, "command": list(command),
        "started_utc": started_utc, "ended_utc": utc_now(),
        "elapsed_seconds": (time.monotonic_ns() - t0) / 1e9, "return_code": int(rc),
        "hostname": platform.node(), "slurm_job_id": os.environ.get("SLURM_JOB_ID"),
        "slurm_restart_count": int(os.environ.get("SLURM_RESTART_COUNT", "0") or 0),
    })
    return int(rc)


def failure_record(row, *, stage: str, exit_code: int, screen_path: Path | None, output: Path) -> dict:
    screen = None
    if screen_path is not None and Path(screen_path).is_file():
        try:
            screen = json.loads(Path(screen_path).read_text())
        except Exception as error:  # the record must still be written
            screen = {"parse_error": repr(error)}
    negative = isinstance(screen, dict) and screen.get("status") == "failed_negative_interrupted"
    payload = {
        "schema": "tiller_row_failure_v1", "matrix_index": row["matrix_index"], "model": row["model"],
        "dataset": row["dataset"], "seed": row["seed"], "stage": stage, "exit_code": int(exit_code),
        "status": "failed_negative_step1000" if negative else "retryable_execution_failure",
        "scientific_terminal": bool(negative), "step1000_screen": screen,
    }
    write_atomic(output, payload)
    return payload


def child_main(argv=None) -> int:
    """Entry of each rank: install the row's auditor, then run the trainer."""
    ap = argparse.ArgumentParser(add_help=False)
    ap.add_argument("--matrix", required=True)
    ap.add_argument("--index", required=True, type=int)
    ap.add_argument("--arm", required=True)
    ap.add_argument("--world", required=True, type=int)
    ap.add_argument("--vocab-size", type=int, default=None)
    ap.add_argument("--max-batch-per-gpu", type=int, default=None)
    known, trainer_argv = ap.parse_known_args(argv)
    from . import identity
    from ..train import trainer
    from ..train.tokens import vocab_size_for
    row = R.row_at(R.load_matrix(known.matrix), known.index)
    targs = trainer.parse_args(trainer_argv)
    vocab = known.vocab_size or vocab_size_for(targs)
    identity.install(row, known.arm, world_size=known.world, vocab_size=vocab,
                     max_batch_per_gpu=known.max_batch_per_gpu)
    return trainer.main(trainer_argv)


def command_for(matrix, index: int, arm: str, output_root, *, gpus: int, port: int = 29511,
                max_batch_per_gpu=None, extra=()) -> list[str]:
    row = R.row_at(R.load_matrix(matrix), index)
    targv = R.training_argv(row, arm, output_root, world_size=gpus, max_batch_per_gpu=max_batch_per_gpu)
    child = [f"--matrix={matrix}", f"--index={index}", f"--arm={arm}", f"--world={gpus}"]
    if max_batch_per_gpu is not None:
        child.append(f"--max-batch-per-gpu={max_batch_per_gpu}")
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "rational_optimizer_b200.protocol.launch",
            "--child", *child, *targv, *extra]


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "--child":
        return child_main(argv[1:])
    ap = argparse.ArgumentParser()
    ap.add_argument("--matrix", required=True)
    ap.add_argument("--index", required=True, type=int)
    ap.add_argument("--arm", required=True, choices=R.ARMS)
    ap.add_argument("--output-root", required=True, type=Path)
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--port", type=int, default=29511)
    ap.add_argument("--max-batch-per-gpu", type=int, default=None)
    ap.add_argument("--timeout-s", type=float, default=None)
    a = ap.parse_args(argv)
    row = R.row_at(R.load_matrix(a.matrix), a.index)
    cmd = command_for(a.matrix, a.index, a.arm, a.output_root, gpus=a.gpus, port=a.port,
                      max_batch_per_gpu=a.max_batch_per_gpu)
    name = R.run_name(row, a.arm)
    rc = run_timed(cmd, a.output_root / f"{name}.wall_clock.json", a.arm, timeout_s=a.timeout_s)
    if rc != 0:
        failure_record(row, stage=a.arm, exit_code=rc, screen_path=a.output_root / f"{name}.step1000.json",
                       output=a.output_root / f"{name}.failure.json")
    return rc


if __name__ == "__main__":
    sys.exit(main())
