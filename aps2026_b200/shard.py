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


def split_by_fraction(prompts: Sequence[Sequence[int]], idx: Sequence[int],
                      fractions: Sequence[float]) -> list[list[int]]:
    """Splits the prompts `idx` (kept in order, prompts that share a first
    token kept together) into consecutive parts holding about `fractions`
    of their tokens."""
    groups: dict[int, list[int]] = {}
    for i in idx:
        groups.setdefault(int(prompts[i][0]) if len(prompts[i]) else -1, []).append(i)
    total = sum(len(prompts[i]) for i in idx)
    targets = [f * total for f in fractions]
    parts: list[list[int]] = [[] for _ in fractions]
    c, filled = 0, 0.0
    for g in groups.values():
        size = sum(len(prompts[i]) for i in g)
        # next part once this group would overshoot the target by more than
        # half of its own size
        while c < len(parts) - 1 and filled + size / 2 > targets[c]:
            c, filled = c + 1, 0.0
        parts[c].extend(g)
        filled += size
    return [sorted(p) for p in parts]


def chunk_plan(prompts: Sequence[Sequence[int]], world: int, chunks: int,
               fractions: Sequence[float] | None = None) -> list[list[list[int]]]:
    """plan[rank][chunk] = global prompt indices: the rank shards of
    shard_prompts, each split again into `chunks` sub-batches -- balanced,
    or holding `fractions` of the rank's tokens in order (a large first
    chunk hides the gather of the earlier chunks behind the later ones);
    empty sub-batches dropped."""
    plan = []
    for mine in shard_prompts(prompts, world):
        if not mine:
            plan.append([])
            continue
        if fractions is not None:
            if len(fractions) != chunks:
                raise ValueError("one fraction per chunk")
            sub = split_by_fraction(prompts, mine, fractions)
            plan.append([p for p in sub if p])
        else:
            sub = shard_prompts([prompts[i] for i in mine], chunks)
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
