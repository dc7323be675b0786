"""Optimizers: TILLER, tiller_then_muon, Muon, fused AdamW and the published baselines."""
from .adamw import FusedAdamW
from .muon import Muon
from .tiller import (FAMILY_ID, PREFIX, TILLERAttentionOptimizer, TILLERRouter,
                     configure_microbatch_count, tiller_scaling_formula)

__all__ = ["FAMILY_ID", "PREFIX", "TILLERAttentionOptimizer", "TILLERRouter",
           "configure_microbatch_count", "tiller_scaling_formula", "FusedAdamW", "Muon"]
