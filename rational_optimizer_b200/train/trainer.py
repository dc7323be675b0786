"""Language-model trainer: the reference trainer's command line, records and
protocol on the B200 execution path (reference training/train.py:1904-3312).

Run one process per GPU::

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rational_optimizer_b200.train \\
        --activation grain --optimizer tiller_v1 --layers 18 --d-model 1024 --heads 16 \\
        --ffn-dim 3072 --seq-len 1024 --batch-size 4 --steps 2000 ...

Every reference flag is accepted with the same meaning; the JSONL events
(``config``/``resumed``/``train``/``eval``/``stopped_early``/
``timing_guard_failed``/``optimizer_timing_guard_failed``/
``resume_checkpoint``/``summary``/``checkpoint``) carry the same keys, and
exit code 88 still means "timing guard tripped".  Differences are in how a
step executes: bf16 GEMMs on the tensor cores with fp32 master weights, the
fused GRAIN/RMSNorm/RoPE/cross-entropy kernels, gradients averaged over one
flat buffer by the NVLink all-reduce kernels (NCCL as fallback) instead of
DDP buckets, and one host synchronisation per step (the loss read) instead
of one per micro-batch.  Flags added here: ``--vocab-size`` and
``--zipf-alpha`` for the offline ``synthetic/zipf`` source, ``--tokenizer
bytes``, ``--compute-dtype``, ``--grad-transport``, ``--strict-exact-resume``
(the protocol's run-local resume mode), ``--dist-timeout-s`` and
``--allow-cpu``.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import sys
import time
from pathlib import Path

import torch

from ..parallel import param_ready
from ..models.transformer import (ACCEPTED_ACTIVATIONS, GRAIN_ACTIVATION_IDS, CausalTransformer,
                                  apply_rlb_positive_gauge, grain_settings)
from ..optim.composite import (ACTIVE_OPTIMIZERS, RATIONAL_SPECIFIC_OPTIMIZERS,
                               TILLER_THEN_MUON_OPTIMIZER, configure_optimizer)
from ..optim.baselines import resolve_ademamix_warmup
from ..parallel.dist import cleanup_distributed, reduce_max, reduce_mean, setup_distributed
from ..parallel.grad_sync import GradientSynchronizer
from ..utils import faults
from . import audit, resume, telemetry
from .data import sample_batch
from .engine import clip_grad_norm, learning_rate as _lr
from .integrity import model_state_sha256, sampled_start_fingerprint, tensor_sample_sha256
from .tokens import load_or_tokenize, sanitize_name, vocab_size_for

RLB_MATRIX_SYNC_OPTIMIZERS = {TILLER_THEN_MUON_OPTIMIZER}
RLB_COEFFICIENT_SYNC_OPTIMIZERS = {TILLER_THEN_MUON_OPTIMIZER}
TIMING_GUARD_EXIT = 88
PROVENANCE_ENV = (
    "TILLER_ROW_ID", "TILLER_ARM_ID", "TILLER_DESIGN_VERSION", "TILLER_MANIFEST_SHA256",
    "TILLER_FREEZE_SHA256", "TILLER_RUNTIME_FREEZE_SHA256", "TILLER_ENVIRONMENT_SHA256",
    "TILLER_ARRAY_JOB_ID", "TILLER_ARRAY_TASK_ID", "TILLER_ARRAY_TASK_COUNT", "TILLER_ARRAY_TASK_MIN",
    "TILLER_ARRAY_TASK_MAX", "TILLER_ARRAY_TASK_STEP", "TILLER_ARRAY_TASK_THROTTLE",
    "TILLER_SPOOLED_LAUNCHER_SHA256", "TILLER_RUNTIME_ENVIRONMENT_VALIDATED",
    "TILLER_DISTRIBUTION_CLOSURE_SHA256", "TILLER_SUBMISSION_NONCE", "TILLER_SUBMISSION_INTENT_SHA256",
    "TILLER_SUBMISSION_RESULT_SHA256", "TILLER_SUBMISSION_DEPENDENCY_JOB_ID",
    "TILLER_PREFLIGHT_ATTEMPT_ID", "TILLER_PREFLIGHT_SPOOLED_LAUNCHER_SHA256",
)


def learning_rate(step, args):
    """Linear warm-up then cosine decay to ``min_lr`` (training/train.py:1889-1895)."""
    return _lr(step, lr=args.lr, min_lr=args.min_lr, warmup_steps=args.warmup_steps,
               total_steps=args.steps)


def write_jsonl(path: Path, record: dict) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("a", encoding="utf-8") as fh:
        fh.write(json.dumps(record, sort_keys=True) + "\n")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="rational_optimizer_b200.train")
    B = argparse.BooleanOptionalAction
    p.add_argument("--activation", choices=ACCEPTED_ACTIVATIONS, default="silu", metavar="{silu,grain}")
    p.add_argument("--run-name", default="lm_optimizer_sweep")
    p.add_argument("--dataset-name", default="HuggingFaceFW/fineweb")
    p.add_argument("--dataset-config", default="sample-10BT")
    p.add_argument("--dataset-revision", default=None)
    p.add_argument("--dataset-streaming", action=B, default=False)
    p.add_argument("--dataset-text-column", default="text")
    p.add_argument("--train-split", default="train")
    p.add_argument("--validation-split", default="validation")
    for name in ("train-skip-documents", "validation-skip-documents", "train-skip-tokens",
                 "validation-skip-tokens"):
        p.add_argument(f"--{name}", type=int, default=0)
    p.add_argument("--trust-remote-code", action=B, default=False)
    p.add_argument("--tokenizer", default="gpt2")
    p.add_argument("--tokenizer-revision", default=None)
    p.add_argument("--hf-cache", default="experiments/cache/huggingface")
    p.add_argument("--cache-dir", default="experiments/cache/tokens")
    p.add_argument("--output-dir", default="experiments/runs/lm_optimizer_sweep")
    p.add_argument("--prepare-only", action="store_true")
    p.add_argument("--refresh-cache", action="store_true")
    p.add_argument("--max-train-tokens", type=int, default=100_000_000)
    p.add_argument("--max-val-tokens", type=int, default=2_000_000)
    p.add_argument("--tokenize-batch-size", type=int, default=1024)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch-size", type=int, default=32)
    p.add_argument("--grad-accum", type=int, default=1)
    p.add_argument("--steps", type=int, default=0)
    p.add_argument("--layers", type=int, default=12)
    p.add_argument("--d-model", type=int, default=768)
    p.add_argument("--heads", type=int, default=12)
    p.add_argument("--ffn-dim", type=int, default=2048)
    p.add_argument("--init-std", type=float, default=0.02)
    p.add_argument("--rational-init", choices=["silu"], default="silu")
    p.add_argument("--post-rational-init", default="identity")
    p.add_argument("--rational-group-size", type=int, default=256)
    p.add_argument("--rational-max-groups", type=int, default=32)
    p.add_argument("--rational-basis-eps", type=float, default=1e-6)
    p.add_argument("--optimizer", choices=ACTIVE_OPTIMIZERS, default="adamw")
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--min-lr", type=float, default=3e-5)
    p.add_argument("--warmup-steps", type=int, default=200)
    p.add_argument("--weight-decay", type=float, default=0.1)
    p.add_argument("--fairness-contract", choices=["none", audit.EXACT_LR_WD_CONTRACT], default="none")
    p.add_argument("--experiment-identity", choices=["none", *audit.TILLER_EXPERIMENT_IDENTITIES],
                   default="none")
    p.add_argument("--beta1", type=float, default=0.9)
    p.add_argument("--beta2", type=float, default=0.95)
    p.add_argument("--eps", type=float, default=1e-8)
    p.add_argument("--factored-min-dim", type=int, default=128)
    p.add_argument("--factored-clip-threshold", type=float, default=1.0)
    p.add_argument("--ademamix-beta3", type=float, default=0.9999)
    p.add_argument("--ademamix-alpha", type=float, default=5.0)
    p.add_argument("--ademamix-beta3-warmup-steps", type=int, default=-1)
    p.add_argument("--ademamix-alpha-warmup-steps", type=int, default=-1)
    p.add_argument("--schedule-free-beta1", type=float, default=0.9)
    p.add_argument("--schedule-free-warmup-steps", type=int, default=0)
    p.add_argument("--came-beta3", type=float, default=0.999)
    p.add_argument("--came-confidence-scale", type=float, default=1.0)
    p.add_argument("--came-confidence-min", type=float, default=0.25)
    p.add_argument("--came-confidence-max", type=float, default=4.0)
    p.add_argument("--soap-precondition-frequency", type=int, default=50)
    p.add_argument("--soap-large-side-identity-threshold", type=int, default=2048)
    p.add_argument("--soap-one-sided", action=B, default=False)
    p.add_argument("--muon-momentum", type=float, default=0.95)
    p.add_argument("--muon-ns-steps", type=int, default=5)
    p.add_argument("--muon-adjust-lr-fn", choices=["original", "match_rms_adamw"], default="match_rms_adamw")
    p.add_argument("--sam-rho", type=float, default=0.0)
    p.add_argument("--sam-adaptive", action=B, default=False)
    p.add_argument("--grad-clip", type=float, default=1.0)
    p.add_argument("--log-interval", type=int, default=10)
    p.add_argument("--eval-interval", type=int, default=250)
    p.add_argument("--eval-batches", type=int, default=20)
    p.add_argument("--early-stop-min-step", type=int, default=0)
    p.add_argument("--early-stop-max-val-loss", type=float, default=0.0)
    p.add_argument("--early-stop-loss-increase", type=float, default=0.0)
    p.add_argument("--timing-guard-max-seconds-per-step", type=float, default=0.0)
    p.add_argument("--timing-guard-max-optimizer-step-seconds", type=float, default=0.0)
    p.add_argument("--timing-guard-min-step", type=int, default=0)
    p.add_argument("--probe-batch-size", type=int, default=2)
    S = argparse.SUPPRESS
    p.add_argument("--telemetry-grain-stat-every", dest="telemetry_rlb_stat_every", type=int, default=4)
    p.add_argument("--telemetry-rlb-stat-every", dest="telemetry_rlb_stat_every", type=int, default=S, help=S)
    p.add_argument("--telemetry-grain-stat-samples", dest="telemetry_rlb_stat_samples", type=int, default=512)
    p.add_argument("--telemetry-rlb-stat-samples", dest="telemetry_rlb_stat_samples", type=int, default=S, help=S)
    p.add_argument("--telemetry-denominator-probe-points", type=int, default=129)
    p.add_argument("--grain-training-telemetry", action=B, default=True)
    p.add_argument("--matrix-spectrum-interval", type=int, default=500)
    p.add_argument("--matrix-spectrum-max-dim", type=int, default=512)
    p.add_argument("--grain-init-gauge-log-scale", dest="rlb_init_gauge_log_scale", type=float, default=0.0)
    p.add_argument("--rlb-init-gauge-log-scale", dest="rlb_init_gauge_log_scale", type=float, default=S, help=S)
    p.add_argument("--grain-init-gauge-seed", dest="rlb_init_gauge_seed", type=int, default=424242)
    p.add_argument("--rlb-init-gauge-seed", dest="rlb_init_gauge_seed", type=int, default=S, help=S)
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--save-checkpoint", action="store_true")
    p.add_argument("--checkpoint-dir", default=None)
    p.add_argument("--resume-checkpoint", default=None)
    p.add_argument("--resume-checkpoint-interval", type=int, default=0)
    # additions of this framework
    p.add_argument("--vocab-size", type=int, default=50304,
                   help="vocabulary of the synthetic/zipf and synthetic/uniform sources")
    p.add_argument("--zipf-alpha", type=float, default=1.1)
    p.add_argument("--compute-dtype", choices=["bf16", "fp32"], default="bf16")
    p.add_argument("--grad-transport", choices=["p2p", "nccl", "owner", "owner-bf16", "owner-int8"], default=None)
    p.add_argument("--strict-exact-resume", action="store_true",
                   help="run-local checkpoint, interrupted-commit recovery, argument-digest contract")
    p.add_argument("--dist-timeout-s", type=float, default=600.0)
    p.add_argument("--allow-cpu", action="store_true", help="run on CPU (gloo) when no GPU is present")
    return p


def parse_args(argv=None):
    return build_parser().parse_args(argv)


_FRAMEWORK_ONLY_ARGS = ("vocab_size", "zipf_alpha", "compute_dtype", "grad_transport",
                        "strict_exact_resume", "dist_timeout_s", "allow_cpu")


def reference_namespace(args) -> argparse.Namespace:
    """``args`` without this framework's additions: the namespace the reference would hold."""
    return argparse.Namespace(**{k: v for k, v in vars(args).items() if k not in _FRAMEWORK_ONLY_ARGS})


def validate_optimizer_protocol(args):
    if args.optimizer not in ACTIVE_OPTIMIZERS:
        raise ValueError(f"Accepted optimizer choices: {', '.join(ACTIVE_OPTIMIZERS)}")
    if args.optimizer in RATIONAL_SPECIFIC_OPTIMIZERS and args.activation not in GRAIN_ACTIVATION_IDS:
        raise ValueError(f"optimizer {args.optimizer} requires the GRAIN activation")
    if float(args.sam_rho) != 0.0 or bool(args.sam_adaptive):
        raise ValueError("the published experiment protocol requires SAM to remain disabled")
    strict_local = bool(getattr(args, "strict_exact_resume", False)) and args.resume_checkpoint is not None
    if strict_local:
        resume.validate_strict(args)
    if args.fairness_contract == audit.EXACT_LR_WD_CONTRACT:
        if not 0.0 <= float(args.min_lr) <= float(args.lr):
            raise ValueError("the exact LR/WD contract requires 0 <= min_lr <= lr")
        if float(args.weight_decay) < 0.0:
            raise ValueError("the exact LR/WD contract requires nonnegative weight decay")
        if args.resume_checkpoint is not None and not strict_local:
            raise ValueError("fairness-contracted runs may not resume from an external checkpoint")
    if (args.experiment_identity in audit.TILLER_EXPERIMENT_IDENTITIES
            and args.fairness_contract != audit.EXACT_LR_WD_CONTRACT):
        raise ValueError("the TILLER matrix identity requires the exact LR/WD contract")


@torch.no_grad()
def evaluate(model, tokens, args, offsets, rank, device, is_distributed):
    param_ready.wait_all()
    model.eval()
    gen = torch.Generator(device="cpu")
    gen.manual_seed(args.seed + 1_000_003 + rank)
    total = None
    for _ in range(args.eval_batches):
        x, y = sample_batch(tokens, args.batch_size, args.seq_len, offsets, gen, device)
        loss = model.forward_loss(x, y).detach().float()
        total = loss if total is None else total + loss
    local = float(total.item()) / max(1, args.eval_batches) if total is not None else 0.0
    return reduce_mean(local, device, is_distributed)


class Run:
    """State of one training run (the loop lives in :meth:`train`)."""

    def __init__(self, args):
        self.args = args
        self.strict = bool(args.strict_exact_resume)

    def emit(self, record, *, to_file=True):
        if self.strict:
            record = resume.audited_summary(record, self.args)
        if self.rank == 0:
            print(json.dumps(record, sort_keys=True), flush=True)
            if to_file:
                write_jsonl(self.out_path, record)

    def barrier(self):
        if self.is_distributed:
            torch.distributed.barrier()

    def setup(self):
        args = self.args
        info = setup_distributed(timeout_s=float(args.dist_timeout_s))
        self.info = info
        self.is_distributed, self.rank, self.world = info.is_distributed, info.rank, info.world_size
        self.device = device = info.device
        if device.type != "cuda" and not args.allow_cpu:
            raise RuntimeError("this trainer runs on CUDA (pass --allow-cpu for a CPU run)")
        torch.manual_seed(args.seed)
        if device.type == "cuda":
            torch.cuda.manual_seed_all(args.seed)
        self.train_tokens = load_or_tokenize(args, "train", args.max_train_tokens)
        self.val_tokens = load_or_tokenize(args, "validation", args.max_val_tokens)
        if device.type == "cuda":
            self.train_tokens = self.train_tokens.pin_memory()
            self.val_tokens = self.val_tokens.pin_memory()
        vocab = vocab_size_for(args)
        self.global_tokens = args.batch_size * args.grad_accum * self.world * args.seq_len
        if args.steps <= 0:
            args.steps = max(1, self.train_tokens.numel() // self.global_tokens)
        model = CausalTransformer(args, vocab)
        if args.compute_dtype == "fp32":
            model.set_compute_dtype(torch.float32)
        self.initial_state_sha256 = model_state_sha256(model) if self.rank == 0 else None
        model = model.to(device)
        apply_rlb_positive_gauge(model, args.rlb_init_gauge_log_scale, args.rlb_init_gauge_seed)
        telemetry.enable_rlb_training_telemetry(model, args)
        self.param_count = sum(p.numel() for p in model.parameters())
        self.identity = audit.audit_tiller_experiment_identity(
            args, world_size=self.world, global_tokens=self.global_tokens,
            train_token_count=self.train_tokens.numel(), val_token_count=self.val_tokens.numel(),
            parameter_count=self.param_count)
        if self.is_distributed:
            with torch.no_grad():
                for t in list(model.parameters()) + list(model.buffers()):
                    torch.distributed.broadcast(t, src=0)
        self.model = model
        self.rational_param_count = sum(
            p.numel() for n, p in model.named_parameters()
            if p.requires_grad and (".rlb_activation." in n or n.endswith(".numerator")
                                    or n.endswith(".denominator")))
        self.optimizer = configure_optimizer(model, args)
        from ..optim.composite import owner_layers
        layers, owner_of = owner_layers(self.optimizer)
        self.sync = GradientSynchronizer(model, transport=args.grad_transport, owner_layers=layers,
                                         layer_owner=owner_of)
        self.clip_observer = self.optimizer if hasattr(self.optimizer, "record_realized_clipping") else None
        self.fairness = audit.audit_optimizer_lr_wd_fairness(model, self.optimizer, args)
        self.offsets = torch.arange(args.seq_len + 1)
        self.train_gen = torch.Generator(device="cpu")
        self.train_gen.manual_seed(args.seed + 997 * self.rank)
        self.out_path = Path(args.output_dir) / args.run_name / f"{args.activation}.jsonl"
        self.probe_state = telemetry.prepare_probe_batch(self.val_tokens, args, self.offsets, self.rank,
                                                         device, self.out_path, barrier=self.barrier)
        self.resume_path = None if args.resume_checkpoint is None else Path(args.resume_checkpoint)
        self.resume_payload = None
        if self.resume_path is not None:
            self.resume_payload = resume.load(
                self.resume_path, args=self._contract_view(), rank=self.rank, world_size=self.world,
                is_distributed=self.is_distributed, device=device, model=model,
                optimizer=self.optimizer, train_generator=self.train_gen,
                probe_state=self.probe_state, strict=self.strict)
        self.resume_step = 0 if self.resume_payload is None else int(self.resume_payload["completed_step"])
        if self.resume_step < 0 or self.resume_step >= args.steps:
            raise RuntimeError(f"invalid exact-resume completed step: {self.resume_step}")

    def _contract_view(self):
        """Arguments bound into the resume contract (the reference namespace)."""
        return reference_namespace(self.args)

    def config_record(self):
        args = self.args
        g = (grain_settings(args.ffn_dim, args.rational_group_size, args.rational_max_groups)
             if args.activation in GRAIN_ACTIVATION_IDS else None)
        gv = lambda key: None if g is None else g[key]
        only = lambda names, value: value if args.optimizer in names else None
        slurm_job = os.environ.get("SLURM_JOB_ID")
        self.slurm = {"slurm_job_id": slurm_job,
                      "slurm_restart_count": int(os.environ.get("SLURM_RESTART_COUNT", "0") or 0),
                      "slurm_node": os.environ.get("SLURMD_NODENAME") or os.environ.get("SLURM_NODELIST")}
        self.timing_attempt_id = (f"{slurm_job or 'manual'}:{self.slurm['slurm_restart_count']}:"
                                  f"{int(time.time())}")
        r0 = self.rank == 0
        rec = {
            "event": "config", "activation": args.activation,
            "activation_display_name": "GRAIN" if args.activation in GRAIN_ACTIVATION_IDS else "SwiGLU",
            **self.slurm, "timing_attempt_id": self.timing_attempt_id,
            "optimizer_telemetry_steps": None if self.telemetry_steps is None else list(self.telemetry_steps),
            "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"),
            "slurm_job_gpus": os.environ.get("SLURM_JOB_GPUS"),
            "gpu_metadata": telemetry.nvidia_smi_metadata(
                strict=os.environ.get("TILLER_STRICT_GPU_METADATA", "0") == "1") if r0 else None,
            "initial_state_sha256": self.initial_state_sha256,
            "train_token_sample_sha256": tensor_sample_sha256(self.train_tokens) if r0 else None,
            "val_token_sample_sha256": tensor_sample_sha256(self.val_tokens) if r0 else None,
            "first_batch_index_sha256": sampled_start_fingerprint(
                self.train_tokens.numel(), args.seq_len, args.batch_size, args.grad_accum, args.seed) if r0 else None,
            "validation_index_sha256": sampled_start_fingerprint(
                self.val_tokens.numel(), args.seq_len, args.batch_size, args.eval_batches,
                args.seed + 1_000_003) if r0 else None,
            "timing_guard_max_seconds_per_step": args.timing_guard_max_seconds_per_step,
            "timing_guard_max_optimizer_step_seconds": args.timing_guard_max_optimizer_step_seconds,
            "timing_guard_min_step": args.timing_guard_min_step,
            "resume_checkpoint": None if self.resume_path is None else str(self.resume_path.resolve()),
            "resume_checkpoint_interval": args.resume_checkpoint_interval,
            "dataset": args.dataset_name, "dataset_config": args.dataset_config,
            "dataset_revision": args.dataset_revision, "dataset_streaming": args.dataset_streaming,
            "dataset_text_column": args.dataset_text_column, "train_split": args.train_split,
            "validation_split": args.validation_split,
            "train_skip_documents": args.train_skip_documents,
            "validation_skip_documents": args.validation_skip_documents,
            "train_skip_tokens": args.train_skip_tokens, "validation_skip_tokens": args.validation_skip_tokens,
            "seed": args.seed, "tokenizer": args.tokenizer, "tokenizer_revision": args.tokenizer_revision,
            "train_tokens": self.train_tokens.numel(), "val_tokens": self.val_tokens.numel(),
            "world_size": self.world, "batch_size_per_gpu": args.batch_size,
            "global_tokens_per_step": self.global_tokens, "grad_accum": args.grad_accum,
            "seq_len": args.seq_len, "steps": args.steps, "layers": args.layers, "d_model": args.d_model,
            "heads": args.heads, "ffn_dim": args.ffn_dim, "params": self.param_count,
            "init_std": args.init_std, "rational_init": args.rational_init,
            "post_rational_init": args.post_rational_init, "rational_group_size": args.rational_group_size,
            "rational_max_groups": args.rational_max_groups, "rational_basis_eps": args.rational_basis_eps,
            "grain_init": gv("base_init"), "grain_centers": gv("centers"),
            "grain_coefficient_limit": gv("coeff_limit"), "grain_groups": gv("groups"),
            "grain_hidden_dim": gv("hidden_dim"), "grain_input_affine": gv("input_affine"),
            "grain_fused": gv("fused"), "grain_center_odd": gv("center_odd"),
            "grain_train_centers": gv("train_centers"), "grain_atom_scale_init": gv("atom_scale_init"),
            "grain_atom_scale_limit": gv("atom_scale_limit"),
            "grain_live_stats_scope": telemetry.rlb_live_stats_scope(self.model),
            "grain_ddp_sync_check_interval": self.sync_check_interval,
            "grain_telemetry_stat_every": args.telemetry_rlb_stat_every,
            "grain_telemetry_stat_samples": args.telemetry_rlb_stat_samples,
            "telemetry_denominator_probe_points": args.telemetry_denominator_probe_points,
            "matrix_spectrum_interval": args.matrix_spectrum_interval,
            "matrix_spectrum_max_dim": args.matrix_spectrum_max_dim, "optimizer": args.optimizer,
            "optimizer_formal_candidate": "tiller_then_muon" if args.optimizer == TILLER_THEN_MUON_OPTIMIZER else None,
            "tiller_then_muon_switch_after_step": 1000 if args.optimizer == TILLER_THEN_MUON_OPTIMIZER else None,
            "tiller_then_muon_state_transition": (
                "preserve_compatible_state" if args.optimizer == TILLER_THEN_MUON_OPTIMIZER else None),
            "fairness_contract": args.fairness_contract, "experiment_identity": args.experiment_identity,
            "optimizer_lr_wd_fairness": self.fairness, "tiller_experiment_identity": self.identity,
            "source_manifest_sha256": os.environ.get("RATIONALOPT_SOURCE_MANIFEST_SHA256"),
            "source_manifest_row_sha256": os.environ.get("RATIONALOPT_SOURCE_MANIFEST_ROW_SHA256"),
            "source_manifest_row_id": os.environ.get("RATIONALOPT_SOURCE_MANIFEST_ROW_ID"),
            "source_manifest_row_index": os.environ.get("RATIONALOPT_SOURCE_MANIFEST_ROW_INDEX"),
            "source_freeze_sha256": os.environ.get("RATIONALOPT_SOURCE_FREEZE_SHA256"),
            "optimizer_lr": args.lr, "optimizer_min_lr": args.min_lr,
            "optimizer_weight_decay": args.weight_decay, "optimizer_beta1": args.beta1,
            "optimizer_beta2": args.beta2, "optimizer_eps": args.eps, "warmup_steps": args.warmup_steps,
            "grad_clip": args.grad_clip, "log_interval": args.log_interval,
            "eval_interval": args.eval_interval, "eval_batches": args.eval_batches,
            "early_stop_min_step": args.early_stop_min_step,
            "early_stop_max_val_loss": args.early_stop_max_val_loss,
            "early_stop_loss_increase": args.early_stop_loss_increase,
            "factored_min_dim": only({"adafactor_came"}, args.factored_min_dim),
            "factored_clip_threshold": only({"adafactor_came"}, args.factored_clip_threshold),
            "ademamix_beta3": only({"ademamix"}, args.ademamix_beta3),
            "ademamix_alpha": only({"ademamix"}, args.ademamix_alpha),
            "ademamix_beta3_warmup_steps": only(
                {"ademamix"}, resolve_ademamix_warmup(args.ademamix_beta3_warmup_steps, args.steps)),
            "ademamix_alpha_warmup_steps": only(
                {"ademamix"}, resolve_ademamix_warmup(args.ademamix_alpha_warmup_steps, args.steps)),
            "schedule_free_beta1": only({"schedule_free_adamw"}, args.schedule_free_beta1),
            "schedule_free_warmup_steps": only({"schedule_free_adamw"}, args.schedule_free_warmup_steps),
            "came_beta3": only({"adafactor_came"}, args.came_beta3),
            "came_confidence_scale": only({"adafactor_came"}, args.came_confidence_scale),
            "came_confidence_min": only({"adafactor_came"}, args.came_confidence_min),
            "came_confidence_max": only({"adafactor_came"}, args.came_confidence_max),
            "soap_precondition_frequency": only({"soap_adamw"}, args.soap_precondition_frequency),
            "soap_large_side_identity_threshold": only({"soap_adamw"}, args.soap_large_side_identity_threshold),
            "soap_one_sided": only({"soap_adamw"}, args.soap_one_sided),
            "muon_adjust_lr_fn": only({"muon", TILLER_THEN_MUON_OPTIMIZER}, args.muon_adjust_lr_fn),
            "muon_momentum": only({"muon", TILLER_THEN_MUON_OPTIMIZER}, args.muon_momentum),
            "muon_ns_steps": only({"muon", TILLER_THEN_MUON_OPTIMIZER}, args.muon_ns_steps),
            "sam_rho": args.sam_rho, "sam_adaptive": args.sam_adaptive,
            "grain_coefficient_parameters": (
                self.rational_param_count if args.optimizer in RATIONAL_SPECIFIC_OPTIMIZERS else None),
            "compute_dtype": args.compute_dtype, "grad_transport": self.sync.transport,
        }
        for name in PROVENANCE_ENV:
            rec[name.lower()] = os.environ.get(name)
        return rec

    def save_resume(self, completed_step, active_seconds):
        resume.save(self.resume_path, args=self._contract_view(), rank=self.rank, world_size=self.world,
                    is_distributed=self.is_distributed, device=self.device, model=self.model,
                    optimizer=self.optimizer, train_generator=self.train_gen,
                    probe_state=self.probe_state, completed_step=completed_step,
                    best_val_loss=self.best_val_loss, step_times=self.step_times,
                    optimizer_step_times=self.optimizer_step_times,
                    grad_clip_observed_steps=self.clip_observed, grad_clip_triggered_steps=self.clip_triggered,
                    run_cuda_max_memory_allocated=self.mem_alloc, run_cuda_max_memory_reserved=self.mem_res,
                    active_seconds=active_seconds, strict=self.strict,
                    cpu_probe_state=telemetry.cpu_probe_state)

    def _memory_peaks(self, reset=False):
        if self.device.type != "cuda":
            return
        self.mem_alloc = max(self.mem_alloc, int(torch.cuda.max_memory_allocated(self.device)))
        self.mem_res = max(self.mem_res, int(torch.cuda.max_memory_reserved(self.device)))
        if reset:
            torch.cuda.reset_peak_memory_stats(self.device)

    def _timing_guard(self, step, seconds, limit, *, event, key, limit_key, strict_ge):
        guard_min = max(1, int(self.args.timing_guard_min_step))
        if limit <= 0.0 or step + 1 < guard_min:
            return
        worst = reduce_max(seconds, self.device, self.is_distributed)
        tripped = worst >= limit if strict_ge else worst > limit
        if not tripped:
            return
        self.emit({"event": event, "activation": self.args.activation, "step": step + 1, key: worst,
                   limit_key: limit, "timing_guard_min_step": guard_min, **self.slurm,
                   "timing_attempt_id": self.timing_attempt_id,
                   "active_seconds_after_event": time.perf_counter() - self.start_time})
        self.barrier()
        cleanup_distributed(self.info)
        raise SystemExit(TIMING_GUARD_EXIT)

    def train(self):
        args, device = self.args, self.device
        self.telemetry_steps = telemetry.parse_optimizer_telemetry_steps(
            os.environ.get("TILLER_OPTIMIZER_TELEMETRY_STEPS"), args.steps)
        self.sync_check_interval = max(0, int(os.environ.get("RLB_DDP_SYNC_CHECK_INTERVAL", "0") or 0))
        config = self.config = self.config_record()
        if self.resume_payload is None:
            self.emit(config)
        else:
            if self.rank == 0:
                print(json.dumps(config, sort_keys=True), flush=True)
            self.emit({"event": "resumed", "activation": args.activation, "step": self.resume_step,
                       "checkpoint": str(self.resume_path.resolve()), **self.slurm,
                       "timing_attempt_id": self.timing_attempt_id})
        rp = self.resume_payload or {}
        self.step_times = [float(v) for v in rp.get("step_times", [])]
        self.optimizer_step_times = [float(v) for v in rp.get("optimizer_step_times", [])]
        self.best_val_loss = float(rp.get("best_val_loss", math.inf))
        self.clip_observed = int(rp.get("grad_clip_observed_steps", 0))
        self.clip_triggered = int(rp.get("grad_clip_triggered_steps", 0))
        self.mem_alloc = int(rp.get("run_cuda_max_memory_allocated", 0))
        self.mem_res = int(rp.get("run_cuda_max_memory_reserved", 0))
        cuda = device.type == "cuda"
        ev0 = torch.cuda.Event(enable_timing=True) if cuda else None
        ev1 = torch.cuda.Event(enable_timing=True) if cuda else None
        if cuda:
            torch.cuda.reset_peak_memory_stats(device)
            torch.cuda.synchronize(device)
        self.start_time = time.perf_counter() - float(rp.get("active_seconds", 0.0))
        lr_trace = hashlib.sha256()
        lr_audit_steps = 0
        loss_since_log, steps_since_log = 0.0, 0
        stop_reason = stop_step = None
        model, opt = self.model, self.optimizer
        for step in range(self.resume_step, args.steps):
            faults.maybe_inject("train_step", self.rank, step + 1)
            model.train()
            t_step = time.perf_counter()
            will_log = (step + 1) % args.log_interval == 0 or step == 0 or step + 1 == args.steps
            will_eval = args.eval_interval > 0 and (
                step == 0 or (step + 1) % args.eval_interval == 0 or step + 1 == args.steps)
            capture = will_log and self.rank == 0
            if capture and cuda:
                self._memory_peaks(reset=True)
                torch.cuda.synchronize(device)
            telemetry.set_optimizer_telemetry_capture(
                opt, capture and (self.telemetry_steps is None or step + 1 in self.telemetry_steps))
            t_fb = time.perf_counter()
            lr = learning_rate(step, args)
            for group in opt.param_groups:
                group["lr"] = lr * float(group.get("lr_scale", 1.0))
            audit.assert_optimizer_realized_lr(opt, lr, args)
            self.sync.zero_grad()
            loss_sum = None
            for micro in range(args.grad_accum):
                x, y = sample_batch(self.train_tokens, args.batch_size, args.seq_len, self.offsets,
                                    self.train_gen, device)
                loss = model.forward_loss(x, y)
                if micro == args.grad_accum - 1:
                    self.sync.begin_backward()
                (loss / args.grad_accum).backward()
                loss_sum = loss.detach().float() if loss_sum is None else loss_sum + loss.detach().float()
            self.sync.synchronize()
            if capture and cuda:
                torch.cuda.synchronize(device)
            fb_seconds = time.perf_counter() - t_fb
            # with clipping off the norm is only measured, on log steps
            norm = (clip_grad_norm(self.sync.params, args.grad_clip, self.sync.flat_covering())
                    if (args.grad_clip > 0 or capture) else None)
            if self.clip_observer is not None:
                self.clip_observer.record_realized_clipping(norm if args.grad_clip > 0 or capture else None,
                                                            args.grad_clip)
            t_opt = time.perf_counter()
            if ev0 is not None:
                ev0.record()
            opt.step()
            if ev1 is not None:
                ev1.record()
            audit.assert_optimizer_realized_lr(opt, lr, args)
            if args.fairness_contract == audit.EXACT_LR_WD_CONTRACT:
                lr_trace.update(f"{step + 1}:{float(lr).hex()}\n".encode("ascii"))
                lr_audit_steps += 1
            matrix_sync = coef_sync = None
            if (args.optimizer in RLB_MATRIX_SYNC_OPTIMIZERS and telemetry.optimizer_method_specific_sync_active(opt)
                    and self.sync_check_interval > 0
                    and (step == 0 or (step + 1) % self.sync_check_interval == 0 or will_eval
                         or step + 1 == args.steps)):
                matrix_sync = audit.assert_rlb_matrix_parameters_synced(model, args, device, self.is_distributed)
            if (args.optimizer in RLB_COEFFICIENT_SYNC_OPTIMIZERS
                    and telemetry.optimizer_method_specific_sync_active(opt)
                    and (step == 0 or will_eval or step + 1 == args.steps)):
                coef_sync = audit.assert_rlb_coefficient_parameters_synced(model, args, device, self.is_distributed)
            # one host synchronisation per step: loss, clip flag and optimizer time together
            packed = torch.stack([loss_sum / args.grad_accum,
                                  norm.float() if norm is not None else loss_sum.new_zeros(())])
            local = packed.cpu()
            if cuda:
                opt_seconds = ev0.elapsed_time(ev1) / 1000.0
                self._memory_peaks()
            else:
                opt_seconds = time.perf_counter() - t_opt
            norm_value = float(local[1]) if norm is not None else None
            triggered = bool(args.grad_clip > 0 and norm_value is not None and norm_value > float(args.grad_clip))
            step_time = time.perf_counter() - t_step
            self.step_times.append(step_time)
            self.optimizer_step_times.append(opt_seconds)
            mean_loss = reduce_mean(float(local[0]), device, self.is_distributed)
            loss_since_log += mean_loss
            steps_since_log += 1
            self.clip_observed += 1
            self.clip_triggered += int(triggered)
            if not math.isfinite(mean_loss):
                stop_reason, stop_step = "nonfinite_train_loss", step + 1
                self.emit({"event": "stopped_early", "activation": args.activation, "step": stop_step,
                           "reason": stop_reason, "loss": mean_loss, "timing_attempt_id": self.timing_attempt_id,
                           "active_seconds_after_event": time.perf_counter() - self.start_time})
                break
            if will_log:
                recent = self.step_times[-args.log_interval:]
                recent_opt = self.optimizer_step_times[-args.log_interval:]
                mean_step = sum(recent) / len(recent)
                mean_opt = sum(recent_opt) / len(recent_opt)
                rec = {"event": "train", "activation": args.activation, "step": step + 1,
                       "loss": loss_since_log / max(1, steps_since_log), "lr": lr, "sam_rho": 0.0,
                       "tokens_per_second": self.global_tokens / mean_step, "seconds_per_step": mean_step,
                       "grad_global_norm_before_clip": telemetry.finite_float(norm_value),
                       "grad_clip_triggered": triggered, "grad_clip_threshold": args.grad_clip,
                       "forward_backward_seconds": telemetry.finite_float(fb_seconds),
                       "optimizer_step_seconds": telemetry.finite_float(mean_opt),
                       "ddp_parameter_sync_max_abs": telemetry.finite_float(matrix_sync),
                       "grain_coefficient_sync_max_abs": telemetry.finite_float(coef_sync),
                       "timing_attempt_id": self.timing_attempt_id}
                if cuda:
                    rec["cuda_max_memory_allocated"] = int(torch.cuda.max_memory_allocated(device))
                    rec["cuda_max_memory_reserved"] = int(torch.cuda.max_memory_reserved(device))
                if self.rank == 0:
                    rec.update(telemetry.collect_optimizer_telemetry(opt))
                    rec.update(telemetry.collect_rlb_telemetry(model, args))
                rec["active_seconds_after_event"] = time.perf_counter() - self.start_time
                loss_since_log, steps_since_log = 0.0, 0
                self.emit(rec)
                self._timing_guard(step, mean_step, float(args.timing_guard_max_seconds_per_step),
                                   event="timing_guard_failed", key="seconds_per_step",
                                   limit_key="max_seconds_per_step", strict_ge=False)
                self._timing_guard(step, mean_opt, float(args.timing_guard_max_optimizer_step_seconds),
                                   event="optimizer_timing_guard_failed", key="optimizer_step_seconds",
                                   limit_key="max_optimizer_step_seconds", strict_ge=True)
            if will_eval:
                t_eval = time.perf_counter()
                val = evaluate(model, self.val_tokens, args, self.offsets, self.rank, device, self.is_distributed)
                if cuda:
                    torch.cuda.synchronize(device)
                rec = {"event": "eval", "activation": args.activation, "step": step + 1, "val_loss": val,
                       "val_ppl": math.exp(min(20.0, val)),
                       "grain_coefficient_sync_max_abs": telemetry.finite_float(coef_sync),
                       "timing_attempt_id": self.timing_attempt_id,
                       "active_seconds_at_val_loss": time.perf_counter() - self.start_time}
                rec.update(telemetry.evaluate_probe(model, self.probe_state, device, self.is_distributed))
                if self.rank == 0 and args.matrix_spectrum_interval > 0 and (
                        step == 0 or (step + 1) % args.matrix_spectrum_interval == 0 or step + 1 == args.steps):
                    rec.update(telemetry.collect_matrix_spectrum_telemetry(model, args))
                if cuda:
                    torch.cuda.synchronize(device)
                    self._memory_peaks()
                rec["active_seconds_after_event"] = time.perf_counter() - self.start_time
                rec["eval_seconds"] = time.perf_counter() - t_eval
                self.emit(rec)
                current = step + 1
                previous_best = self.best_val_loss
                nonfinite = not math.isfinite(val)
                if not nonfinite:
                    self.best_val_loss = min(self.best_val_loss, val)
                min_met = current >= max(1, int(args.early_stop_min_step))
                max_loss, increase = float(args.early_stop_max_val_loss), float(args.early_stop_loss_increase)
                too_large = max_loss > 0.0 and val > max_loss
                worse = (increase > 0.0 and math.isfinite(previous_best) and not nonfinite
                         and val > previous_best + increase)
                if nonfinite or (min_met and (too_large or worse)):
                    stop_reason = ("nonfinite_val_loss" if nonfinite else
                                   "val_loss_above_threshold" if too_large else "val_loss_regressed_from_best")
                    stop_step = current
                    self.emit({"event": "stopped_early", "activation": args.activation, "step": stop_step,
                               "reason": stop_reason, "val_loss": val,
                               "best_val_loss": self.best_val_loss if math.isfinite(self.best_val_loss) else None,
                               "early_stop_max_val_loss": max_loss, "early_stop_loss_increase": increase,
                               "timing_attempt_id": self.timing_attempt_id,
                               "active_seconds_after_event": time.perf_counter() - self.start_time})
                    break
                interval = max(0, int(args.resume_checkpoint_interval))
                if (self.resume_path is not None and interval > 0 and current < args.steps
                        and current % interval == 0):
                    self.save_resume(current, time.perf_counter() - self.start_time)
                    if self.rank == 0:
                        write_jsonl(self.out_path, {
                            "event": "resume_checkpoint", "activation": args.activation, "step": current,
                            "path": str(self.resume_path.resolve()), "timing_attempt_id": self.timing_attempt_id,
                            "active_seconds_after_event": time.perf_counter() - self.start_time})
        return self.finish(stop_reason, stop_step, lr_audit_steps, lr_trace)

    def finish(self, stop_reason, stop_step, lr_audit_steps, lr_trace):
        args, device = self.args, self.device
        total = time.perf_counter() - self.start_time
        drop = min(5, max(0, len(self.step_times) - 1))
        timed = self.step_times[drop:]
        mean_step = sum(timed) / max(1, len(timed))
        completed = stop_step if stop_step is not None else args.steps
        completed_tokens = int(completed) * int(self.global_tokens)
        cuda = device.type == "cuda"
        if cuda:
            self._memory_peaks()
            if self.is_distributed:
                peaks = torch.tensor([self.mem_alloc, self.mem_res], device=device, dtype=torch.int64)
                torch.distributed.all_reduce(peaks, op=torch.distributed.ReduceOp.MAX)
                self.mem_alloc, self.mem_res = int(peaks[0].item()), int(peaks[1].item())
        summary = {
            "event": "summary", "activation": args.activation, **self.slurm,
            "timing_attempt_id": self.timing_attempt_id,
            "timing_guard_max_seconds_per_step": args.timing_guard_max_seconds_per_step,
            "timing_guard_max_optimizer_step_seconds": args.timing_guard_max_optimizer_step_seconds,
            "timing_guard_min_step": args.timing_guard_min_step, "mean_seconds_per_step": mean_step,
            "tokens_per_second": self.global_tokens / mean_step if mean_step > 0 else None,
            "training_loop_tokens_per_second": completed_tokens / max(total, 1e-12),
            "total_seconds": total, "steps": args.steps, "completed_steps": completed,
            "completed_tokens": completed_tokens, "realized_lr_audit_steps": lr_audit_steps,
            "realized_lr_trace_sha256": (lr_trace.hexdigest()
                                         if args.fairness_contract == audit.EXACT_LR_WD_CONTRACT else None),
            "grad_clip_observed_steps": self.clip_observed, "grad_clip_triggered_steps": self.clip_triggered,
            "grad_clip_trigger_fraction": (0.0 if self.clip_observed == 0
                                           else self.clip_triggered / self.clip_observed),
            "cuda_run_max_memory_allocated": self.mem_alloc if cuda else None,
            "cuda_run_max_memory_reserved": self.mem_res if cuda else None,
            "cuda_run_memory_peak_scope": "global_max_all_ranks" if cuda else None,
            "stopped_early": stop_reason is not None, "stop_reason": stop_reason,
        }
        self.emit(summary)
        if args.save_checkpoint and self.rank == 0:
            ckpt_dir = (Path(args.checkpoint_dir) if args.checkpoint_dir is not None
                        else Path(args.output_dir) / args.run_name / "checkpoints")
            ckpt_dir.mkdir(parents=True, exist_ok=True)
            path = ckpt_dir / f"{sanitize_name(args.activation)}_seed{args.seed}.pt"
            torch.save({"model": self.model.state_dict(), "args": vars(reference_namespace(args)),
                        "config": self.config, "summary": summary, "param_count": self.param_count}, path)
            self.emit({"event": "checkpoint", "activation": args.activation, "path": str(path),
                       "seed": args.seed})
        return summary


def main(argv=None):
    args = parse_args(argv)
    validate_optimizer_protocol(args)
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    if args.prepare_only:
        train_tokens = load_or_tokenize(args, "train", args.max_train_tokens)
        val_tokens = load_or_tokenize(args, "validation", args.max_val_tokens)
        print(json.dumps({"event": "prepared", "train_tokens": train_tokens.numel(),
                          "val_tokens": val_tokens.numel()}), flush=True)
        return 0
    run = Run(args)
    run.setup()
    try:
        run.train()
    finally:
        if getattr(run.sync, "communicator", None) is not None:
            run.sync.communicator.close()
    cleanup_distributed(run.info)
    return 0


if __name__ == "__main__":
    sys.exit(main())
