"""Portable modern-MHA decoder study (reference experiments/mha_1b_tokens).

A Qwen3-style decoder (separate Q/K/V projections with per-head Q/K RMSNorm,
split-half RoPE with theta 1e6, SwiGLU or parameter-matched GRAIN MLP, tied
embeddings) trained on packed uint32 token caches under four conditions:
``swiglu_adamw``, ``swiglu_muon``, ``grain_tiller`` and
``grain_tiller100_muon``; checkpoints are atomic, checksum-verified and
resume bitwise at update boundaries.
"""
