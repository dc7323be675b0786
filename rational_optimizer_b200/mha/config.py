"""Study configuration and its invariants (reference experiments/mha_1b_tokens/config.json,
conditions.py, switch_contract.py, train.py:39-56)."""
from __future__ import annotations

import copy

MHA_MUON = "swiglu_muon"
MHA_ADAMW = "swiglu_adamw"
MHA_TILLER = "grain_tiller"
MHA_SWITCH = "grain_tiller100_muon"
CONDITIONS = (MHA_MUON, MHA_ADAMW, MHA_TILLER, MHA_SWITCH)
SWITCH_CONDITIONS = (MHA_SWITCH,)
GRAIN_CONDITIONS = (MHA_TILLER, MHA_SWITCH)
SWITCH_UPDATE = 100

DEFAULT_CONFIG = {
    "accumulation": 4, "checkpoint_every": 250, "checkpoint_keep_recent": 2,
    "conditions": {c: {"lr": 0.0003} for c in CONDITIONS},
    "context": 2048, "dataset_config": "sample-100BT", "dataset_id": "HuggingFaceFW/fineweb-edu",
    "grain": {"group_width": 256, "groups": 18, "intermediate_size": 4608},
    "loss_tokens_per_condition": 1000079360, "loss_tokens_per_update": 262144, "microbatch": 8,
    "min_lr_ratio": 0.1,
    "model": {"attention_bias": False, "head_dim": 64, "hidden_size": 1024, "initializer_range": 0.02,
              "intermediate_size": 3072, "num_attention_heads": 16, "num_hidden_layers": 28,
              "num_key_value_heads": 16, "rms_norm_eps": 1e-06, "rope_scaling": None, "rope_theta": 1000000,
              "tie_word_embeddings": True, "use_sliding_window": False, "vocab_size": 151936},
    "schedule_horizon_updates": 45776, "seed": 1337, "small_validation_tokens": 131072,
    "updates": 3815, "validation_every": 100, "warmup_updates": 200, "world_size": 4,
}


def default_config():
    return copy.deepcopy(DEFAULT_CONFIG)


def validate_config(cfg):
    c = cfg["model"]
    if c["num_attention_heads"] != 16 or c["num_key_value_heads"] != 16 or 16 * c["head_dim"] != c["hidden_size"]:
        raise ValueError("TILLER attention requires 16 equal heads and a square output projection")
    g = cfg["grain"]
    if g["intermediate_size"] * 2 != c["intermediate_size"] * 3 or g["intermediate_size"] != g["groups"] * g["group_width"]:
        raise ValueError("GRAIN/SwiGLU width matching differs")
    if set(cfg["conditions"]) != set(CONDITIONS):
        raise ValueError("condition inventory changed")
    if cfg["world_size"] * cfg["microbatch"] * cfg["accumulation"] * cfg["context"] != cfg["loss_tokens_per_update"]:
        raise ValueError("global loss-bearing token batch mismatch")
    if cfg["updates"] * cfg["loss_tokens_per_update"] != cfg["loss_tokens_per_condition"]:
        raise ValueError("target tokens/updates mismatch")
    if not 0 <= cfg["warmup_updates"] < cfg["schedule_horizon_updates"] or cfg["updates"] > cfg["schedule_horizon_updates"]:
        raise ValueError("invalid schedule horizon")


def schedule(completed, cfg, base_lr):
    """LR of update ``completed + 1``: linear warm-up, cosine to ``min_lr_ratio`` at the horizon."""
    import math
    step = completed + 1
    if step <= cfg["warmup_updates"]:
        return base_lr * step / cfg["warmup_updates"]
    progress = (step - cfg["warmup_updates"]) / (cfg["schedule_horizon_updates"] - cfg["warmup_updates"])
    return base_lr * (cfg["min_lr_ratio"] + (1 - cfg["min_lr_ratio"]) * 0.5 * (1 + math.cos(math.pi * progress)))
