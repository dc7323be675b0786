"""Activation x optimizer experiment manifest (behaviour of
experiments/protocol/build_activation_optimizer_manifest.py:1-361; the CSV it
writes is the same file, byte for byte).

One row per (suite, dataset, seed, method).  The dataset revisions, model
shapes, method hyper-parameters and suite budgets below define the published
experiments and are kept exactly (they are the experiment design, not code).
Rows are generated suite by suite as the product dataset x seed x method;
:func:`check_matched_arms` then requires every (suite, dataset, model,
budget, seed) cell to hold each method of its suite, and the SiLU and GRAIN
arms of one optimizer to differ only in their activation.

    python -m rational_optimizer_b200.protocol.manifest --output activation_optimizer_manifest.csv
"""
from __future__ import annotations

import argparse
import csv
import itertools
from collections import Counter, defaultdict
from pathlib import Path

GRAIN = "rlb_fused_global_rational"
SMALL, LARGE = "12l_768d", "18l_1024d"
PREFLIGHT = "12l_768d_preflight_2621440_tokens_80_steps"
S100, S300, L100 = ("12l_768d_100m_tokens_3050_steps", "12l_768d_300m_tokens_9150_steps",
                    "18l_1024d_100m_tokens_3050_steps")

# name: (hub id, config, revision, validation split, validation skip at 100M / 300M tokens)
DATASETS = {
    "dclm": ("mlfoundations/dclm-baseline-1.0", "none", "a3b142c183aebe5af344955ae20836eb34dcf69b", "train",
             210_000_000, 610_000_000),
    "fineweb_edu": ("HuggingFaceFW/fineweb-edu", "sample-10BT", "87f09149ef4734204d70ed1d046ddc9ca3f2b8f9", "train",
                    210_000_000, 610_000_000),
    "fineweb": ("HuggingFaceFW/fineweb", "sample-10BT", "9bb295ddab0e05d785b879661af7260fed5140fc", "train",
                210_000_000, 610_000_000),
    "dolma_sample": ("allenai/dolma", "v1_6-sample", "7f48140530a023e9ea4c5cfb141160922727d4d3", "train",
                     210_000_000, 610_000_000),
    "c4_en": ("allenai/c4", "en", "1588ec454efa1a09f29cd18ddd04fe05fc8653a2", "validation", 0, 0),
}
DATASET_ORDER = ("dclm", "fineweb_edu", "fineweb", "dolma_sample", "c4_en")
SEEDS = (1337, 2027, 3407)
# model: layers, d_model, heads, ffn_dim, batch_size, grad_accum
MODELS = {SMALL: (12, 768, 12, 2048, 16, 2), LARGE: (18, 1024, 16, 3072, 8, 4)}
_MUON = "--muon-momentum 0.95 --muon-ns-steps 5 --muon-adjust-lr-fn match_rms_adamw"
# optimizer family: (manifest optimizer id, lr, min_lr, extra trainer flags); each
# family runs once with SiLU ("silu_<family>") and once with GRAIN ("rlb_<family>")
FAMILIES = (
    ("adamw", "adamw", "0.0003", "0.00003", ""),
    ("muon", "muon", "0.0003", "0.00003", _MUON),
    ("lion", "lion", "0.0001", "0.00001", ""),
    ("soap", "soap_adamw", "0.0003", "0.00003", "--soap-precondition-frequency 50 --no-soap-one-sided"),
    ("ademamix", "ademamix", "0.0003", "0.00003", "--ademamix-alpha 5.0 --ademamix-beta3 0.9999"),
    ("came", "adafactor_came", "0.0003", "0.00003", "--came-confidence-scale 1.0"),
    ("schedulefree", "schedule_free_adamw", "0.0003", "0.00003",
     "--schedule-free-beta1 0.90 --schedule-free-warmup-steps 0"),
)
TOKENIZER = ("gpt2", "607a30d783dfa663caf39e06633721c8d4cfcd7e")
COLUMNS = (
    "row_index", "row_id", "phase", "dataset", "dataset_name", "dataset_config", "dataset_revision",
    "dataset_streaming", "text_column", "train_split", "val_split", "train_skip_documents",
    "validation_skip_documents", "train_skip_tokens", "val_skip_tokens", "cache_dir", "model", "layers",
    "d_model", "heads", "ffn_dim", "seq_len", "batch_size", "grad_accum", "global_tokens_per_step",
    "train_tokens", "val_tokens", "steps", "eval_interval", "eval_batches", "log_interval", "seed", "method",
    "activation", "optimizer", "lr", "min_lr", "weight_decay", "warmup_steps", "beta1", "beta2", "eps",
    "grad_clip", "muon_momentum", "muon_ns_steps", "muon_adjust_lr_fn", "init_std", "rational_init",
    "post_rational_init", "rational_group_size", "rational_max_groups", "probe_batch_size",
    "matrix_spectrum_interval", "telemetry_rlb_stat_every", "sam_rho", "sam_adaptive", "tokenizer",
    "tokenizer_revision", "extra_args",
)


def methods():
    """Every method row fragment, SiLU then GRAIN within each optimizer family."""
    out = []
    for family, optimizer, lr, min_lr, extra in FAMILIES:
        for prefix, activation in (("silu", "silu"), ("rlb", GRAIN)):
            out.append({"method": f"{prefix}_{family}", "activation": activation, "optimizer": optimizer,
                        "lr": lr, "min_lr": min_lr, "weight_decay": "0.10", "extra_args": extra})
    return out


# suite: (model, training tokens, seeds, method names or None for all, overrides)
SUITES = (
    (PREFLIGHT, SMALL, 100_000_000, (1337,), ("silu_adamw", "rlb_adamw"),
     {"steps": "80", "train_tokens": "2621440", "val_tokens": "200000", "eval_interval": "40",
      "eval_batches": "2"}),
    (S100, SMALL, 100_000_000, SEEDS, None, {}),
    (S300, SMALL, 300_000_000, SEEDS, None, {}),
    (L100, LARGE, 100_000_000, SEEDS, None, {}),
)


def _budget(tokens: int):
    """(steps, validation tokens, eval interval) of a training-token budget."""
    return {100_000_000: (3_050, 4_000_000, 50), 300_000_000: (9_150, 8_000_000, 50)}[tokens]


def _row(suite, dataset, model, tokens, seed, method) -> dict[str, str]:
    hub, config, revision, val_split, skip100, skip300 = DATASETS[dataset]
    layers, d_model, heads, ffn, batch, accum = MODELS[model]
    steps, val_tokens, eval_interval = _budget(tokens)
    small = model == SMALL
    row = {
        "row_id": f"{suite}_{dataset}_seed{seed}_{method['method']}", "phase": suite, "dataset": dataset,
        "dataset_name": hub, "dataset_config": config, "dataset_revision": revision,
        "dataset_streaming": "true", "text_column": "text", "train_split": "train", "val_split": val_split,
        "train_skip_documents": "0", "validation_skip_documents": "0", "train_skip_tokens": "0",
        "val_skip_tokens": str(skip300 if tokens == 300_000_000 else skip100),
        "cache_dir": f"experiments/cache/tokens_iclr26_main/{dataset}", "model": model, "layers": str(layers),
        "d_model": str(d_model), "heads": str(heads), "ffn_dim": str(ffn), "seq_len": "256",
        "batch_size": str(batch), "grad_accum": str(accum), "global_tokens_per_step": str(256 * 4 * batch * accum),
        "train_tokens": str(tokens), "val_tokens": str(val_tokens), "steps": str(steps),
        "eval_interval": str(eval_interval), "eval_batches": "10", "log_interval": "10", "seed": str(seed),
        "warmup_steps": "200", "beta1": "0.90", "beta2": "0.95", "eps": "0.00000001", "grad_clip": "1.0",
        "muon_momentum": "0.95", "muon_ns_steps": "5", "muon_adjust_lr_fn": "match_rms_adamw",
        "init_std": "0.02", "rational_init": "silu", "post_rational_init": "identity",
        "rational_group_size": "256", "rational_max_groups": "32", "probe_batch_size": "1" if small else "0",
        "matrix_spectrum_interval": "250" if small else "0", "telemetry_rlb_stat_every": "4", "sam_rho": "0.0",
        "sam_adaptive": "false", "tokenizer": TOKENIZER[0], "tokenizer_revision": TOKENIZER[1],
    }
    row.update(method)
    return row


def build_rows() -> list[dict[str, str]]:
    all_methods = methods()
    rows = []
    for suite, model, tokens, seeds, names, overrides in SUITES:
        chosen = [m for m in all_methods if names is None or m["method"] in names]
        for dataset, seed, method in itertools.product(DATASET_ORDER, seeds, chosen):
            row = _row(suite, dataset, model, tokens, seed, method)
            row.update(overrides)
            rows.append(row)
    for i, row in enumerate(rows):
        row["row_index"] = str(i)
    return [{c: row[c] for c in COLUMNS} for row in rows]


def check_matched_arms(rows) -> None:
    """Raise ValueError unless every cell holds its suite's methods with paired arms."""
    if not rows:
        raise ValueError("the manifest has no rows")
    sparse = [r["row_id"] for r in rows if int(r["eval_interval"]) > 50]
    if sparse:
        raise ValueError(f"evaluation interval above 50 steps: {sparse[:3]}")
    expected = {suite: ({m["method"] for m in methods()} if names is None else set(names))
                for suite, _, _, _, names, _ in SUITES}
    cells = defaultdict(list)
    for r in rows:
        if r["phase"] in expected:
            cells[(r["phase"], r["dataset"], r["model"], r["train_tokens"], r["seed"])].append(r)
    free = {"row_index", "row_id", "method", "activation"}
    for key, members in cells.items():
        missing = expected[key[0]] - {r["method"] for r in members}
        if missing:
            raise ValueError(f"cell {key} lacks {sorted(missing)}")
        by_opt = defaultdict(list)
        for r in members:
            by_opt[r["optimizer"]].append(r)
        for opt, arms in by_opt.items():
            if len(arms) != 2:
                raise ValueError(f"cell {key} has {len(arms)} {opt} rows, expected a SiLU/GRAIN pair")
            diff = {c: (arms[0][c], arms[1][c]) for c in COLUMNS if c not in free and arms[0][c] != arms[1][c]}
            if diff:
                raise ValueError(f"the {opt} arms of cell {key} differ beyond the activation: {diff}")
    absent = {S100, S300, L100} - {r["phase"] for r in rows}
    if absent:
        raise ValueError(f"endpoint suites missing: {sorted(absent)}")


def write(rows, path) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=list(COLUMNS), lineterminator="\n")
        w.writeheader()
        w.writerows(rows)


def summary(rows) -> list[str]:
    lines = [f"rows {len(rows)}"]
    lines += [f"{p}: {n}" for p, n in sorted(Counter(r["phase"] for r in rows).items())]
    lines += [f"{p}/{d}: {n}" for (p, d), n in sorted(Counter((r["phase"], r["dataset"]) for r in rows).items())]
    return lines


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--output", type=Path, default=Path("experiments/protocol/activation_optimizer_manifest.csv"))
    ap.add_argument("--print-summary", action="store_true")
    a = ap.parse_args(argv)
    rows = build_rows()
    check_matched_arms(rows)
    write(rows, a.output)
    if a.print_summary:
        print("\n".join(summary(rows)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
