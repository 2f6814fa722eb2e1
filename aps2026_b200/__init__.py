"""aps2026_b200: B200-native (sm_100a) non-GEMM prefill layer ops of
Phi-tiny-MoE behind a C ABI (include/aps2026_b200.h).

``aps2026_b200.ops`` mirrors the reference's ``tensor_ops`` GPU ops on torch
tensors; ``aps2026_b200.prefill`` runs the layer pipeline (prefix-trie
dedup, per-layer non-GEMM ops, multi-GPU sharding). The CUDA library must be
built (``python -m aps2026_b200.build``); nothing falls back to the CPU.
"""
from ._lib import LIB_PATH, declared_functions, lib  # noqa: F401

__version__ = "0.1.0"
