"""Protocol layer: matrix rows -> trainer flags, identity audit, screen, hardware audit (CPU)."""
import importlib
import json

import pytest

from rational_optimizer_b200.protocol import collect, hardware, identity, launch, monitor, rows as R
from rational_optimizer_b200.train import trainer
from reference_oracle import require_reference


def _row(index=0, phase="18l_1024d_100m_tokens_3050_steps", candidate="tiller_v1"):
    return {
        "matrix_index": index, "phase": phase, "model": "18l_1024d", "dataset": "dclm",
        "dataset_name": "mlfoundations/dclm-baseline-1.0", "dataset_config": "none",
        "dataset_revision": "abc", "dataset_streaming": True, "dataset_text_column": "text",
        "train_split": "train", "validation_split": "train", "train_skip_documents": 0,
        "validation_skip_documents": 0, "train_skip_tokens": 0, "validation_skip_tokens": 210000000,
        "cache_dir": "cache", "max_train_tokens": 100000000, "max_val_tokens": 4000000, "steps": 3050,
        "layers": 18, "d_model": 1024, "heads": 16, "ffn_dim": 3072, "seq_len": 256, "batch_size": 16,
        "grad_accum": 2, "global_tokens_per_step": 32768, "eval_interval": 50, "eval_batches": 10,
        "log_interval": 10, "seed": 1337, "lr": 0.0003, "min_lr": 3e-05, "warmup_steps": 200,
        "weight_decay": 0.1, "beta1": 0.9, "beta2": 0.95, "eps": 1e-08, "grad_clip": 1.0,
        "muon_momentum": 0.95, "muon_ns_steps": 5, "muon_adjust_lr_fn": "match_rms_adamw",
        "init_std": 0.02, "rational_init": "silu", "post_rational_init": "identity",
        "rational_group_size": 256, "rational_max_groups": 32, "probe_batch_size": 1,
        "matrix_spectrum_interval": 250, "telemetry_rlb_stat_every": 4, "sam_rho": 0.0, "sam_adaptive": False,
        "tokenizer": "gpt2", "tokenizer_revision": "607a", "control_activation": "silu",
        "control_optimizer": "muon", "candidate_activation": "rlb_fused_global_rational",
        "candidate_optimizer": candidate, "control_name": "SwiGLU+Muon", "candidate_name": "TILLER",
        "source_manifest_row_id": "row-x", "source_manifest_row_index": 7,
    }


@pytest.mark.parametrize("arm", ["control", "candidate"])
def test_training_argv_matches_reference(arm, tmp_path):
    require_reference()
    suite = importlib.import_module("experiments.protocol.suite")
    row = _row()
    ref = suite.training_argv(row, arm, tmp_path)
    ours = R.training_argv(row, arm, tmp_path)
    assert ours == [str(a) for a in ref[1:]]
    assert R.run_name(row, arm) == suite.run_name(row, arm)
    assert R.jsonl_path(row, arm, tmp_path) == suite.jsonl_path(row, arm, tmp_path)
    # the trainer accepts every flag and reproduces the expected values
    args = trainer.parse_args(ours)
    R.verify_args(args, row, arm)


def test_rebalance_keeps_global_tokens():
    row = _row()
    for world in (1, 2, 4, 8):
        plan = R.rebalance(row, world)
        assert plan["batch_size"] * plan["grad_accum"] * world * row["seq_len"] == row["global_tokens_per_step"]
    assert R.rebalance(row, 8, max_batch_per_gpu=8) == {"batch_size": 8, "grad_accum": 2, "world_size": 8}
    with pytest.raises(ValueError):
        R.rebalance(dict(row, global_tokens_per_step=1000), 3)


@pytest.mark.parametrize("arm,act,expected", [("control", "silu", 296_867_840),
                                               ("candidate", "rlb_fused_global_rational", 296_871_080)])
def test_expected_parameter_counts(arm, act, expected):
    assert identity.expected_parameter_count(_row(), arm, 50257) == expected


def test_identity_auditor(tmp_path):
    row = _row()
    argv = R.training_argv(row, "candidate", tmp_path, world_size=8)
    args = trainer.parse_args(argv)
    audit = identity.make_auditor(row, "candidate", world_size=8, vocab_size=50257)
    rec = audit(args, world_size=8, global_tokens=32768, train_token_count=100000000,
                val_token_count=4000000, parameter_count=296_871_080)
    assert rec["passed"] and rec["matrix_index"] == 0
    with pytest.raises(RuntimeError, match="identity mismatch"):
        audit(args, world_size=8, global_tokens=32768, train_token_count=5, val_token_count=4000000,
              parameter_count=296_871_080)
    with pytest.raises(RuntimeError, match="argument mismatch"):
        audit(trainer.parse_args(argv + ["--lr", "0.001"]), world_size=8, global_tokens=32768,
              train_token_count=100000000, val_token_count=4000000, parameter_count=296_871_080)


def _write(path, records):
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text("\n".join(json.dumps(r) for r in records) + "\n")


def test_step1000_screen(tmp_path):
    row = _row()
    fp = {k: "h" for k in monitor.FINGERPRINTS}
    cfg = {"event": "config", "dataset": row["dataset_name"], "dataset_config": "none", "dataset_revision": "abc",
           "tokenizer": "gpt2", "tokenizer_revision": "607a", "steps": 3050, "seed": 1337,
           "train_tokens": 100000000, "val_tokens": 4000000, **fp}
    ctl = tmp_path / "c.jsonl"
    _write(ctl, [dict(cfg, activation="silu", optimizer="muon"), {"event": "eval", "step": 1000, "val_loss": 4.0}])
    cand = tmp_path / "k.jsonl"
    ident = {"passed": True, "matrix_index": 0, "source_manifest_row_index": 7, "source_manifest_row_id": "row-x"}
    kcfg = dict(cfg, activation="rlb_fused_global_rational", optimizer="tiller_v1",
                experiment_identity="tiller_matrix_v1", tiller_experiment_identity=ident)
    _write(cand, [kcfg])
    assert monitor.screen(row, ctl, cand, tmp_path / "s.json") == 3
    _write(cand, [kcfg, {"event": "eval", "step": 1000, "val_loss": 3.9}])
    assert monitor.screen(row, ctl, cand, tmp_path / "s.json") == 0
    assert json.loads((tmp_path / "s.json").read_text())["status"] == "pass_nonnegative"
    _write(cand, [kcfg, {"event": "eval", "step": 1000, "val_loss": 4.1}])
    assert monitor.screen(row, ctl, cand, tmp_path / "s.json") == 4
    rec = launch.failure_record(row, stage="candidate", exit_code=4, screen_path=tmp_path / "s.json",
                                output=tmp_path / "f.json")
    assert rec["status"] == "failed_negative_step1000" and rec["scientific_terminal"]
    _write(cand, [dict(kcfg, train_token_sample_sha256="other"), {"event": "eval", "step": 1000, "val_loss": 3.0}])
    with pytest.raises(RuntimeError, match="identity differs"):
        monitor.screen(row, ctl, cand, tmp_path / "s.json")


def test_run_timed_records_wall_clock(tmp_path):
    import sys
    rc = launch.run_timed([sys.executable, "-c", "import sys; sys.exit(3)"], tmp_path / "w.json", "control")
    rec = json.loads((tmp_path / "w.json").read_text())
    assert rc == 3 and rec["return_code"] == 3 and rec["schema"] == "rationalopt_process_wall_clock_v1"


class FakeNvml:
    """Eight B200s; GPU 3 is busy, GPU 5 is throttled."""

    def __init__(self):
        self.devs = [{"index": i, "uuid": f"GPU-{i}", "name": "NVIDIA B200", "memory_used_mib": 10,
                      "processes": 0, "clock_reasons": 0} for i in range(8)]
        self.devs[3]["processes"] = 1
        self.devs[5]["clock_reasons"] = 0x40

    def count(self):
        return len(self.devs)

    def info(self, i):
        return dict(self.devs[i])


TOPO = "\n".join(["\tGPU0\tGPU1\tGPU2\tGPU3\tGPU4\tGPU5\tGPU6\tGPU7\tCPU Affinity"] + [
    f"GPU{i}\t" + "\t".join("X" if j == i else "NV18" for j in range(8)) + "\t0-55" for i in range(8)])


def test_hardware_selection_with_fake_nvml():
    rec = hardware.select(FakeNvml(), TOPO, 4)
    assert rec["passed"] and rec["cuda_visible_devices"] == "0,1,2,4"
    bad = hardware.audit(FakeNvml(), TOPO, [3, 5])
    assert not bad["passed"] and len(bad["problems"]) == 2
    pcie = TOPO.replace("NV18", "SYS")
    assert not hardware.audit(FakeNvml(), pcie, [0, 1])["passed"]
    with pytest.raises(RuntimeError):
        hardware.select(FakeNvml(), TOPO, 7)


def test_collect_reports_rows(tmp_path):
    row = _row()
    payload = {"schema": "tiller_evaluation_matrix_v1", "rows": [row]}
    (tmp_path / "m.json").write_text(json.dumps(payload))
    cand = R.jsonl_path(row, "candidate", tmp_path / "runs")
    _write(cand, [{"event": "config"}, {"event": "eval", "step": 1000, "val_loss": 3.5},
                  {"event": "eval", "step": 3050, "val_loss": 3.2},
                  {"event": "summary", "total_seconds": 10.0, "mean_seconds_per_step": 0.1, "completed_steps": 3050,
                   "stopped_early": False}])
    ctl = R.jsonl_path(row, "control", tmp_path / "runs")
    _write(ctl, [{"event": "config"}, {"event": "eval", "step": 1000, "val_loss": 3.6},
                 {"event": "eval", "step": 3050, "val_loss": 3.3},
                 {"event": "summary", "total_seconds": 9.0, "mean_seconds_per_step": 0.09, "completed_steps": 3050}])
    out = collect.collect_row(row, tmp_path / "runs")
    assert out["status"] == "complete" and abs(out["candidate_final_lead"] - 0.1) < 1e-9
    assert collect.main(["--matrix", str(tmp_path / "m.json"), "--output-root", str(tmp_path / "runs"),
                         "--out", str(tmp_path / "r.csv")]) == 0
