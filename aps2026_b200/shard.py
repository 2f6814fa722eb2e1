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


def chunk_plan(prompts: Sequence[Sequence[int]], world: int, chunks: int) -> list[list[list[int]]]:
    """plan[rank][chunk] = global prompt indices: the rank shards of
    shard_prompts, each split again into `chunks` sub-batches the same way
    (empty sub-batches dropped)."""
    plan = []
    for mine in shard_prompts(prompts, world):
        sub = shard_prompts([prompts[i] for i in mine], chunks) if mine else []
        plan.append([[mine[j] for j in part] for part in sub if part])
    return plan


def gather_order(plan: list[list[list[int]]]) -> list[int]:
    """Global prompt indices in the order rank 0 holds them after the
    per-chunk gathers: chunk-major, then rank, then prompt."""
    order: list[int] = []
    for c in range(max((len(p) for p in plan), default=0)):
        for r in range(len(plan)):
            if c < len(plan[r]):
                order.extend(plan[r][c])
    return order
