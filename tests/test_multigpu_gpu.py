"""Prompt-sharded prefill on 2 GPUs (NCCL): every rank runs its chunks with
b2_prefill_layers and the final hidden states are sent to rank 0
(prefill.FinalGather: NCCL send / recv per chunk); the collected rows equal
a single-GPU run of the whole batch, bit for bit (B2_FLAG_EXACT_ORDER).
Cases: equal shards; prompts of ragged lengths (ranks and chunks of
different token counts); and ranks holding different numbers of chunks.
Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HID_LAYERS = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _standins_for(prompts, chunks, device, layers_pool):
    """Stand-ins whose rows are a fixed function of (prompt, position), each
    chunk's expert rows placed at that chunk's route positions (as the
    grouped W2 GEMM of that sub-batch would write them); chunks are stacked
    in order, as ShardedPrefill slices them."""
    import torch

    from aps2026_b200 import ops, prefill

    keys = ("q", "k", "attn", "logits", "gate_up", "expert_out")
    sets = []
    for pool_i in range(layers_pool):
        blocks = {k: [] for k in keys}
        for part in chunks:
            rows = {k: [] for k in keys}
            for i in part:
                g = torch.Generator(device="cpu").manual_seed(10_000 * pool_i + i)
                n = len(prompts[i])
                rows["q"].append(torch.randn(n, prefill.Q_HEADS * prefill.HEAD_DIM, generator=g))
                rows["k"].append(torch.randn(n, prefill.KV_HEADS * prefill.HEAD_DIM, generator=g))
                rows["attn"].append(torch.randn(n, prefill.HIDDEN, generator=g))
                rows["logits"].append(torch.randn(n, prefill.EXPERTS, generator=g))
                rows["gate_up"].append(torch.randn(2 * n, 2 * prefill.INTER, generator=g))
                rows["expert_out"].append(torch.randn(2 * n, prefill.HIDDEN, generator=g))
            t = {k: torch.cat(v).to(device) for k, v in rows.items()}
            rp = ops.moe_route_gpu(t["logits"]).route_positions.long()
            placed = torch.empty_like(t["expert_out"])
            placed[rp] = t["expert_out"]
            t["expert_out"] = placed
            for k in keys:
                blocks[k].append(t[k])
        t = {k: torch.cat(v) for k, v in blocks.items()}
        sets.append(prefill.StandIns(t["q"], t["k"], t["attn"], t["logits"], t["gate_up"], t["expert_out"]))
    return sets


def _prompts(case):
    from aps2026_b200 import prefill

    if case == "equal":
        return prefill.prompts_config5(seed=31, batch=8, length=96)
    g = np.random.default_rng(32)
    if case == "ragged":
        return [g.integers(0, prefill.VOCAB, int(n)).astype(np.int32) for n in g.integers(40, 160, 9)]
    # "uneven_chunks": rank 0 holds one chunk, rank 1 two (rank 0 receives a
    # chunk index it has no rows of its own for)
    return [g.integers(0, prefill.VOCAB, n).astype(np.int32) for n in (120, 100, 70)]


def _run(rank, world, port, out_path, case):
    import torch
    import torch.distributed as dist

    from aps2026_b200 import prefill
    from aps2026_b200.shard import chunk_plan

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
    try:
        prompts = _prompts(case)
        plan = chunk_plan(prompts, world, 2)
        w = prefill.Weights.make(dev, 7, layers=HID_LAYERS)
        sets = _standins_for(prompts, plan[rank], dev, 2)
        runner = prefill.ShardedPrefill(prompts, plan, w, dev, sets, HID_LAYERS, rank=rank, exact=True)
        runner.step()
        last = torch.empty((len(prompts), prefill.HIDDEN), device=dev)
        if rank == 0:
            runner.last_token_rows(last)
            torch.cuda.synchronize()
            np.save(out_path, last.cpu().numpy())
        if world > 1:
            runner.release()
            dist.barrier()
    finally:
        if world > 1:
            dist.destroy_process_group()


@pytest.mark.parametrize("case", ["equal", "ragged", "uneven_chunks"])
def test_two_gpu_gather_matches_one_gpu(tmp_path, case):
    import torch
    import torch.multiprocessing as mp

    from aps2026_b200.shard import chunk_plan, gather_order

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    prompts = _prompts(case)
    plan = chunk_plan(prompts, 2, 2)
    tokens = [[sum(len(prompts[i]) for i in part) for part in parts] for parts in plan]
    if case != "equal":  # the case really is uneven
        assert tokens[0] != tokens[1]
    two, one = str(tmp_path / "two.npy"), str(tmp_path / "one.npy")
    mp.start_processes(_run, args=(2, _free_port(), two, case), nprocs=2, join=True, start_method="spawn")
    mp.start_processes(_run, args=(1, _free_port(), one, case), nprocs=1, join=True, start_method="spawn")
    o2 = gather_order(plan)
    o1 = gather_order(chunk_plan(prompts, 1, 2))
    got, want = np.load(two), np.load(one)
    pos1 = {p: k for k, p in enumerate(o1)}
    np.testing.assert_array_equal(got, want[[pos1[p] for p in o2]])
