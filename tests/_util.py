"""Shared helpers of the test suite: seeded inputs and host/device moves."""
from __future__ import annotations

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(g: np.random.Generator, shape, mean=0.0, std=1.0) -> np.ndarray:
    return (g.standard_normal(shape) * std + mean).astype(np.float32)


def to_dev(a: np.ndarray, device):
    import torch

    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def to_host(t, dtype=None) -> np.ndarray:
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a
