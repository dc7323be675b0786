"""Identity auditor for ``--experiment-identity`` runs (reference
experiments/protocol/suite.py:257-333).

:func:`install` registers with the trainer a check that the parsed arguments
are exactly the row's (:func:`rows.verify_args`), and that world size,
global tokens per step, token counts and parameter count match the row; the
returned record is written into the run's ``config`` event.
"""
from __future__ import annotations

import torch

from ..models.transformer import CausalTransformer, model_args
from ..train import audit
from . import rows as R


def expected_parameter_count(row, arm: str, vocab_size: int) -> int:
    """Parameters of the row's model for ``arm`` (counted on the meta device)."""
    side = "control" if arm == "control" else "candidate"
    args = model_args(layers=int(row["layers"]), d_model=int(row["d_model"]), heads=int(row["heads"]),
                      ffn_dim=int(row["ffn_dim"]), seq_len=int(row["seq_len"]),
                      activation=row[f"{side}_activation"], rational_init=row["rational_init"],
                      rational_group_size=int(row["rational_group_size"]),
                      rational_max_groups=int(row["rational_max_groups"]), init_std=float(row["init_std"]))
    with torch.device("meta"):
        model = CausalTransformer(args, int(vocab_size))
    seen, total = set(), 0
    for p in model.parameters():
        if id(p) not in seen:
            seen.add(id(p))
            total += p.numel()
    return total


def make_auditor(row, arm: str, *, world_size: int, vocab_size: int, max_batch_per_gpu=None):
    required_contract = R.contract(row)
    required_params = expected_parameter_count(row, arm, vocab_size)

    def auditor(args, *, world_size: int, global_tokens: int, train_token_count: int, val_token_count: int,
                parameter_count: int):
        if args.fairness_contract != required_contract or args.experiment_identity != R.experiment_identity(row):
            return None
        R.verify_args(args, row, arm, world_size=expected_world, max_batch_per_gpu=max_batch_per_gpu)
        required = {
            "world_size": (int(world_size), expected_world),
            "global_tokens_per_step": (int(global_tokens), int(row["global_tokens_per_step"])),
            "train_tokens": (int(train_token_count), int(row["max_train_tokens"])),
            "val_tokens": (int(val_token_count), int(row["max_val_tokens"])),
            "parameter_count": (int(parameter_count), required_params),
        }
        bad = {k: {"observed": o, "required": e} for k, (o, e) in required.items() if o != e}
        if bad:
            raise RuntimeError(f"full-transfer runtime identity mismatch: {bad}")
        return {"passed": True, "matrix_index": int(row["matrix_index"]),
                "source_manifest_row_index": int(row["source_manifest_row_index"]),
                "source_manifest_row_id": row["source_manifest_row_id"], "model": row["model"],
                "dataset": row["dataset"], "seed": int(row["seed"]), "arm": arm,
                "parameter_count": int(parameter_count), "train_token_count": int(train_token_count),
                "val_token_count": int(val_token_count)}

    expected_world = int(world_size)
    return auditor


def install(row, arm: str, *, world_size: int, vocab_size: int, max_batch_per_gpu=None) -> None:
    audit.install_tiller_identity_auditor(
        make_auditor(row, arm, world_size=world_size, vocab_size=vocab_size, max_batch_per_gpu=max_batch_per_gpu))
