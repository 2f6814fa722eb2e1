"""Multi-rank prefill on CPU ranks (gloo, world size 2): prompt sharding, one
trie per chunk, per-rank layer pipelines and the gather of final hidden
states to rank 0 reproduce the single-process result row for row.

Each rank runs the CPU oracle's layer pipeline on its chunks (the GPU ranks
run b2_prefill_layers with the same plan) and rank 0 collects the chunks
through prefill.FinalGather -- the point-to-point transfer the GPU ranks use,
here over gloo -- in shard.gather_order; the GEMM stand-ins are a fixed
function of (prompt, position), so sharding cannot change any row. Prompt
sets with ragged lengths give ranks and chunks of different token counts
and ranks with different numbers of chunks.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

HID, QH, KVH, HD, INTER, LAYERS = 32, 2, 1, 8, 16, 2


def _prompts(case="equal"):
    g = np.random.default_rng(40)
    if case == "ragged":  # unequal shards and chunks
        return [g.integers(0, 500, int(n)).astype(np.int32) for n in g.integers(3, 20, 9)]
    if case == "uneven_chunks":  # rank 0 holds one chunk, rank 1 two
        return [g.integers(0, 500, n).astype(np.int32) for n in (12, 10, 7)]
    ps = [g.integers(0, 500, int(g.integers(8, 14))).astype(np.int32) for _ in range(8)]
    for i in range(1, 8, 2):  # pairs of prompts of equal length keep the rank shards equal in tokens
        ps[i] = g.integers(0, 500, len(ps[i - 1])).astype(np.int32)
    return ps


def _standin_rows(prompt_idx: int, length: int) -> dict:
    """Per-token GEMM stand-ins of one prompt. expert_out holds each token's
    two expert rows in slot order; the batch places them at the token's
    route positions, as the grouped W2 GEMM would."""
    g = np.random.default_rng(1000 + prompt_idx)
    n = lambda *s: g.standard_normal(s).astype(np.float32)  # noqa: E731
    return dict(q=n(length, QH * HD), k=n(length, KVH * HD), attn=n(length, HID), logits=n(length, 16),
                gate_up=n(2 * length, 2 * INTER), expert_out=n(2 * length, HID))


def _weights():
    g = np.random.default_rng(41)
    n = lambda *s: g.standard_normal(s).astype(np.float32)  # noqa: E731
    emb = (0.02 * n(500, HID)).astype(np.float32)
    ln = lambda: (1 + 0.1 * n(HID), 0.1 * n(HID))  # noqa: E731
    return emb, [ln() for _ in range(LAYERS)], [ln() for _ in range(LAYERS)], ln()


def _run_chunk(prompts, idx):
    """Final hidden states (token rows) of the prompts `idx`, by the oracle."""
    import oracle

    sub = [prompts[i] for i in idx]
    trie = oracle.prefix_trie(sub, vocab=500)
    assert trie["nodes"] == sum(len(p) for p in sub)  # no shared prefixes: node rows are token rows
    rows = {k: [] for k in ("q", "k", "attn", "logits", "gate_up", "expert_out")}
    for i in idx:
        s = _standin_rows(i, len(prompts[i]))
        for k in rows:
            rows[k].append(s[k])
    standin = {k: np.ascontiguousarray(np.concatenate(v)) for k, v in rows.items()}
    # token t's slot-s expert row goes to its route position in this batch
    rp = oracle.moe_route(standin["logits"])["route_positions"]
    placed = np.empty_like(standin["expert_out"])
    placed[rp] = standin["expert_out"]
    standin["expert_out"] = placed
    emb, ln1, ln2, fin = _weights()
    _, y = oracle.prefill_layers(emb, trie["node_token"], trie["node_depth"], [standin], ln1, ln2, fin, LAYERS,
                                 q_heads=QH, kv_heads=KVH, head_dim=HD, inter=INTER)
    return y[trie["token_node"]]


def _rank_main(rank, world, port, out_path, case):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aps2026_b200.prefill import FinalGather, chunk_tokens
        from aps2026_b200.shard import chunk_plan

        prompts = _prompts(case)
        plan = chunk_plan(prompts, world, 2)
        gather = FinalGather(chunk_tokens(prompts, plan), rank, HID, "cpu")
        own, works = [], []
        for c in range(gather.chunks()):
            rows = torch.from_numpy(_run_chunk(prompts, plan[rank][c])) if c < len(plan[rank]) else None
            own.append(rows)
            works += gather.post(c, rows)
        for w in works:
            w.wait()
        if rank == 0:
            parts = [gather.rows(c, r, own[c]) for c in range(gather.chunks()) for r in range(world)
                     if c < len(plan[r])]
            np.save(out_path, torch.cat(parts).numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_chunk_plan_covers_every_prompt_once():
    from aps2026_b200.shard import chunk_plan, gather_order, shard_prompts

    prompts = _prompts()
    for world in (1, 2, 3, 8):
        plan = chunk_plan(prompts, world, 2)
        flat = sorted(i for parts in plan for part in parts for i in part)
        assert flat == list(range(len(prompts)))
        assert sorted(gather_order(plan)) == flat
    # shared first tokens stay on one rank
    same = [np.array([7, 1, 2]), np.array([7, 1, 3]), np.array([9, 9]), np.array([5])]
    shards = shard_prompts(same, 2)
    assert any({0, 1} <= set(s) for s in shards)


@pytest.mark.parametrize("case", ["equal", "ragged", "uneven_chunks"])
def test_two_cpu_ranks_gather_matches_single_process(tmp_path, case):
    from aps2026_b200.prefill import chunk_tokens
    from aps2026_b200.shard import chunk_plan, gather_order

    world = 2
    prompts = _prompts(case)
    plan = chunk_plan(prompts, world, 2)
    tokens = chunk_tokens(prompts, plan)
    if case == "ragged":
        assert tokens[0] != tokens[1]
    if case == "uneven_chunks":
        assert len(plan[0]) != len(plan[1])
    out = str(tmp_path / "gathered.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), out, case), nprocs=world, join=True,
                       start_method="spawn")
    got = np.load(out)
    want = np.concatenate([_run_chunk(prompts, [i]) for i in gather_order(plan)])
    np.testing.assert_array_equal(got, want)


def test_chunk_plan_fractions():
    from aps2026_b200.shard import chunk_plan

    prompts = [np.full(2048, i, dtype=np.int32) for i in range(64)]
    for fr, want in (((0.75, 0.25), [6, 2]), ((0.5, 0.5), [4, 4]), ((0.4, 0.35, 0.25), [3, 3, 2]),
                     ((0.5, 0.3, 0.2), [4, 2, 2]), ((0.5, 0.375, 0.125), [4, 3, 1])):
        plan = chunk_plan(prompts, 8, len(fr), fr)
        for parts in plan:
            assert [len(p) for p in parts] == want
            flat = [i for p in parts for i in p]
            assert flat == sorted(flat)  # consecutive, in order
        assert sorted(i for parts in plan for p in parts for i in p) == list(range(64))
    # bench.py's default shares at N > 1 give every rank the same chunk sizes
    # at 2, 4 and 8 ranks
    for world, want in ((2, [16, 12, 4]), (4, [8, 6, 2]), (8, [4, 3, 1])):
        plan = chunk_plan(prompts, world, 3, (0.5, 0.375, 0.125))
        assert all([len(p) for p in parts] == want for parts in plan)
    # prompts sharing a first token stay in one chunk
    same = [np.array([7, 1, 2]), np.array([7, 1, 3]), np.array([9, 9]), np.array([5, 5])]
    plan = chunk_plan(same, 1, 2, (0.5, 0.5))
    assert any({0, 1} <= set(p) for p in plan[0])
    with pytest.raises(ValueError):
        chunk_plan(prompts, 2, 3, (0.5, 0.5))


def _rank_with_failed_peer(rank, world, port, out_path):
    """Rank 1 'fails' (exits without cleanup) before it sends its rows; rank
    0's receive (FinalGather, as the GPU ranks use it) must end with an
    error, not wait forever."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)
    from aps2026_b200.prefill import FinalGather

    t0 = time.monotonic()
    gather = FinalGather([[4], [4]], 0, 8, "cpu")
    try:
        for w in gather.post(0, None):
            w.wait()
        status = "no error"
    except Exception as e:  # noqa: BLE001 -- any error type counts as detection
        status = "error " + type(e).__name__
    with open(out_path, "w") as f:
        f.write(f"{status}\n{time.monotonic() - t0:.1f}\n")
    os._exit(0)  # a group with a dead peer cannot be torn down cleanly


def test_failed_rank_is_detected_by_the_gather(tmp_path):
    out = str(tmp_path / "status.txt")
    mp.start_processes(_rank_with_failed_peer, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    status, seconds = open(out).read().split("\n")[:2]
    assert status.startswith("error"), status
    assert float(seconds) < 60.0
