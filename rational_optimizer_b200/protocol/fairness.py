"""Full-model learning-rate / weight-decay fairness audit of the matrix suites
(behaviour of experiments/protocol/audit_full_model_fairness.py:1-127; same
``tiller_full_model_fairness_v1`` payload).

For one representative row of each suite, both arms are constructed exactly
as a run would construct them - the trainer's own argument parser on the
row's command line (:func:`.rows.training_argv`), the model, and the arm's
optimizer - and :func:`~rational_optimizer_b200.train.audit.audit_optimizer_lr_wd_fairness`
reports every parameter group's LR scale and weight decay and every internal
LR/WD scalar.  The audit passes when both arms run at base LR 3e-4, minimum
LR 3e-5 and weight decay 0.1, every scale is one, and the optimizer covers
every trainable element.

    python -m rational_optimizer_b200.protocol.fairness --matrix matrix.json [--output F.json]
"""
from __future__ import annotations

import argparse
import gc
import json
import tempfile
from pathlib import Path

from . import rows as R

SCHEMA = "tiller_full_model_fairness_v1"
SUITES = ("12l_768d_100m_tokens_3050_steps", "12l_768d_300m_tokens_9150_steps", "18l_1024d_100m_tokens_3050_steps")
VOCAB = 50_257


def audit_arm(row, arm: str) -> dict:
    from ..models.transformer import CausalTransformer
    from ..optim.composite import configure_optimizer
    from ..train import audit
    from ..train.trainer import parse_args

    with tempfile.TemporaryDirectory() as tmp:
        args = parse_args(R.training_argv(row, arm, Path(tmp)))
    model = CausalTransformer(args, VOCAB)
    count = sum(p.numel() for p in model.parameters())
    optimizer = configure_optimizer(model, args)
    fair = audit.audit_optimizer_lr_wd_fairness(model, optimizer, args)
    report = {
        "suite": row["phase"], "model": row["model"], "arm": arm, "optimizer": args.optimizer,
        "parameter_count": count, "base_lr": fair["base_lr"], "minimum_lr": fair["minimum_lr"],
        "base_weight_decay": fair["base_weight_decay"],
        "all_group_lr_scales_are_one": all(g["lr_scale"] == 1.0 for g in fair["groups"]),
        "all_internal_lr_wd_scalars_are_one": all(v == 1.0 for v in fair["internal_lr_wd_scalars"].values()),
        "covered_parameter_elements": fair["covered_parameter_elements"],
        "trainable_parameter_elements": fair["trainable_parameter_elements"],
    }
    del optimizer, model
    gc.collect()
    return report


def passes(report: dict) -> bool:
    return (report["base_lr"] == 3e-4 and report["minimum_lr"] == 3e-5 and report["base_weight_decay"] == 0.1
            and report["all_group_lr_scales_are_one"] and report["all_internal_lr_wd_scalars_are_one"]
            and report["covered_parameter_elements"] == report["trainable_parameter_elements"])


def audit_rows(rows) -> dict:
    reports = [audit_arm(row, arm) for row in rows for arm in ("control", "candidate")]
    return {"schema": SCHEMA, "passed": all(passes(r) for r in reports), "reports": reports}


def representative_rows(matrix: dict, suites=SUITES) -> list:
    first = {}
    for row in matrix["rows"]:
        first.setdefault(row["phase"], row)
    missing = [s for s in suites if s not in first]
    if missing:
        raise ValueError(f"the matrix has no row for {missing}")
    return [first[s] for s in suites]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--matrix", required=True)
    ap.add_argument("--output", type=Path)
    a = ap.parse_args(argv)
    payload = audit_rows(representative_rows(R.load_matrix(a.matrix)))
    if a.output is not None:
        a.output.parent.mkdir(parents=True, exist_ok=True)
        a.output.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n")
    print(json.dumps(payload, sort_keys=True))
    return 0 if payload["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
