"""Prompt sharding across GPUs for the prefill batch.

Prompts are independent (causal attention, no KV cache: src/model.cu:40-44),
so the batch splits by prompt with no cross-GPU traffic until the final
hidden states are gathered. Prompts that share a first token may share a
trie prefix, so they stay together: groups keyed by the first token are
assigned largest-first to the rank with the fewest tokens (LPT bin packing),
which keeps every rank's deduplicated row count -- its share of the work --
close to equal. The assignment is deterministic.
"""
from __future__ import annotations

from typing import Sequence


def shard_prompts(prompts: Sequence[Sequence[int]], world: int) -> list[list[int]]:
    """Prompt indices per rank (each list ascending)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    groups: dict[int, list[int]] = {}
    for i, p in enumerate(prompts):
        key = int(p[0]) if len(p) else -1
        groups.setdefault(key, []).append(i)
    ordered = sorted(groups.values(), key=lambda g: (-sum(len(prompts[i]) for i in g), g[0]))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for g in ordered:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].extend(g)
        load[r] += sum(len(prompts[i]) for i in g)
    return [sorted(x) for x in out]
