"""MHA study: model parity with the reference graph, packed data, switch, bitwise resume (CPU)."""
import importlib
import json

import numpy as np
import pytest
import torch

from rational_optimizer_b200.mha import config as C
from rational_optimizer_b200.mha import train as T
from rational_optimizer_b200.mha.data import PackedBatches, digest, write_cache
from rational_optimizer_b200.mha.model import ModernMHADecoder
from reference_oracle import require_reference


def tiny_config():
    cfg = C.default_config()
    cfg["model"].update(hidden_size=64, head_dim=4, intermediate_size=128, num_hidden_layers=2, vocab_size=256)
    cfg["grain"] = {"group_width": 64, "groups": 3, "intermediate_size": 192}
    cfg.update(context=16, microbatch=2, accumulation=2, world_size=1, loss_tokens_per_update=64, updates=6,
               loss_tokens_per_condition=384, schedule_horizon_updates=10, warmup_updates=2,
               validation_every=3, checkpoint_every=2, checkpoint_keep_recent=2, small_validation_tokens=64)
    return cfg


def write_data(tmp_path):
    rng = np.random.default_rng(0)
    train = rng.integers(0, 256, 64 * 8 + 64, dtype=np.int64)
    val = rng.integers(0, 256, 200, dtype=np.int64)
    splits = {}
    for name, ids in (("train", train), ("validation", val)):
        m = write_cache(tmp_path / f"{name}.u32", ids, vocab_size=256)
        splits[name] = {"path": f"{name}.u32", "sha256": m["sha256"], "tokens": m["tokens"]}
    (tmp_path / "manifest.json").write_text(json.dumps({"dtype": "<u4", "splits": splits}))
    cfg_path = tmp_path / "config.json"
    cfg_path.write_text(json.dumps(tiny_config()))
    return tmp_path / "manifest.json", cfg_path


def test_model_matches_reference_graph():
    require_reference()
    try:
        ref = importlib.import_module("experiments.mha_1b_tokens.model")
    except ModuleNotFoundError:
        pytest.skip("the reference MHA study is not part of the installed reference package")
    cfg = tiny_config()["model"]
    torch.manual_seed(3)
    ours = ModernMHADecoder(cfg, grain=True, groups=3)
    torch.manual_seed(3)
    theirs = ref.ModernMHADecoder(cfg, grain=True, groups=3)
    assert [n for n, _ in ours.named_parameters()] == [n for n, _ in theirs.named_parameters()]
    theirs.load_state_dict(ours.state_dict())
    ids = torch.randint(0, 256, (2, 16))
    torch.testing.assert_close(ours(ids), theirs(ids), rtol=1e-4, atol=1e-4)


def test_packed_batches_are_disjoint(tmp_path):
    write_cache(tmp_path / "t.u32", np.arange(2000), vocab_size=4096)
    data = PackedBatches(tmp_path / "t.u32", world_size=2, microbatch=2, accumulation=2, context=8)
    seen = set()
    for u in range(3):
        for m in range(2):
            for r in range(2):
                x, y, mask = data.batch(u, m, r)
                assert mask.all() and (y[:, :-1] == x[:, 1:]).all()
                for row in y:
                    assert not (set(row.tolist()) & seen)
                    seen.update(row.tolist())
    with pytest.raises(FileExistsError):
        write_cache(tmp_path / "t.u32", np.arange(10), vocab_size=4096)


def _metrics(out):
    return [json.loads(l) for l in (out / "metrics.jsonl").read_text().splitlines()]


@pytest.mark.parametrize("condition", ["swiglu_adamw", "swiglu_muon", "grain_tiller"])
def test_conditions_train_and_resume_bitwise(tmp_path, condition):
    manifest, cfg = write_data(tmp_path)
    full = tmp_path / "full"
    assert T.main(["--condition", condition, "--data", str(manifest), "--output", str(full), "--config", str(cfg),
                   "--device", "cpu"]) == 0
    part = tmp_path / "part"
    assert T.main(["--condition", condition, "--data", str(manifest), "--output", str(part), "--config", str(cfg),
                   "--device", "cpu", "--stop-after", "3"]) == 0
    assert json.loads((part / "result.json").read_text())["update"] == 3
    assert T.main(["--condition", condition, "--data", str(manifest), "--output", str(part), "--config", str(cfg),
                   "--device", "cpu", "--resume", "latest"]) == 0
    a, b = _metrics(full), _metrics(part)
    assert [r["step"] for r in b] == [1, 2, 3, 4, 5, 6]
    assert [r["loss"] for r in a] == [r["loss"] for r in b]
    assert a[-1]["validation_loss"] == b[-1]["validation_loss"]
    assert len(list(full.glob("checkpoint-*-periodic"))) <= 2


def test_switch_hands_momentum_to_muon(tmp_path, monkeypatch):
    monkeypatch.setattr(C, "SWITCH_UPDATE", 2)
    manifest, cfg = write_data(tmp_path)
    out = tmp_path / "switch"
    assert T.main(["--condition", "grain_tiller100_muon", "--data", str(manifest), "--output", str(out),
                   "--config", str(cfg), "--device", "cpu"]) == 0
    phases = [r["phase"] for r in _metrics(out)]
    assert phases[:2] == ["tiller", "tiller"] and phases[2:] == ["muon"] * 4
    assert (out / "checkpoint-000002-switch").is_dir() and (out / "checkpoint-000003-switch").is_dir()


@pytest.mark.gpu
@pytest.mark.parametrize("condition", ["grain_tiller", "swiglu_muon"])
def test_conditions_train_on_gpu(tmp_path, condition):
    manifest, cfg = write_data(tmp_path)
    out = tmp_path / condition
    assert T.main(["--condition", condition, "--data", str(manifest), "--output", str(out), "--config", str(cfg),
                   "--device", "cuda"]) == 0
    recs = _metrics(out)
    assert len(recs) == 6 and all(np.isfinite(r["loss"]) for r in recs)
    assert np.isfinite(recs[-1]["validation_loss"])
