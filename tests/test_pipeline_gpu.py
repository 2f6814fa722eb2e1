"""The layer pipeline (b2_prefill_layers: trie rows, all layers, final
add + LayerNorm) against the oracle's restatement of the reference layer
loop, on identical seeded inputs.

With B2_FLAG_EXACT_ORDER the whole multi-layer pipeline, including the
fused un-permute + add + LayerNorm, must be bit-identical to the reference's
unfused op sequence; with tree-order reductions the final outputs must meet
the north_star tolerance.
"""
import numpy as np
import pytest

import oracle
from tests._util import to_host

pytestmark = pytest.mark.gpu


def _run(cuda, prompts, layers, pool, exact, seed=5, hidden=4096):
    import torch

    from aps2026_b200 import prefill

    w = prefill.Weights.make(cuda, seed, layers=layers, hidden=hidden)
    batch = prefill.Batch.build(prompts, cuda)
    gen = torch.Generator(device=cuda).manual_seed(seed + 1)
    standins = [prefill.StandIns.make(batch.rows, cuda, gen, hidden=hidden) for _ in range(pool)]
    host = [dict(q=to_host(s.q).copy(), k=to_host(s.k).copy(), attn=to_host(s.attn).copy(),
                 logits=to_host(s.logits).copy(), gate_up=to_host(s.gate_up).copy(),
                 expert_out=to_host(s.expert_out).copy()) for s in standins]
    pipe = prefill.Pipeline(batch, w, cuda, exact=exact, hidden=hidden)
    pipe.bind_layers(standins, layers)
    timer = prefill.StageTimer(layers)
    pipe.run(timer=timer)
    torch.cuda.synchronize()
    d = timer.durations()
    assert all(v > 0 for vals in d.values() for v in vals)
    want_x, want_y = oracle.prefill_layers(
        to_host(w.emb), batch.trie.node_token, batch.trie.node_depth, host,
        [(to_host(a), to_host(b)) for a, b in w.ln1], [(to_host(a), to_host(b)) for a, b in w.ln2],
        (to_host(w.final[0]), to_host(w.final[1])), layers)
    return pipe, standins, host, want_x, want_y


@pytest.mark.parametrize("exact", [True, False])
def test_pipeline_small_shared_prefix(cuda, exact):
    from aps2026_b200 import prefill

    prompts = prefill.prompts_config4(seed=11, batch=4, length=40, shared=8)
    pipe, standins, host, want_x, want_y = _run(cuda, prompts, layers=3, pool=2, exact=exact)
    assert pipe.batch.rows == 8 + 4 * 32
    if exact:
        oracle.assert_bitexact(to_host(pipe.final_x), want_x, "final residual")
        oracle.assert_bitexact(to_host(pipe.final_out), want_y, "final LayerNorm")
    else:
        oracle.assert_close(to_host(pipe.final_out), want_y, what="final LayerNorm")
    # the last layer's gated SiLU (its output feeds only the stand-in expert
    # GEMM): bit-exact in exact order, within tolerance with expf
    inter = pipe.act.shape[1]
    gu = host[(3 - 1) % 2]["gate_up"]
    want_act = oracle.silu_mul(gu[:, :inter], gu[:, inter:])
    if exact:
        oracle.assert_bitexact(to_host(pipe.act), want_act, "SiLU")
    else:
        oracle.assert_close(to_host(pipe.act), want_act, what="SiLU")
    # the in-place updates of the stand-ins (RoPE on q/k; attn += x) agree too
    for s, h in zip(standins, host):
        oracle.assert_bitexact(to_host(s.q), h["q"], "rope q")
        oracle.assert_bitexact(to_host(s.k), h["k"], "rope k")
        if exact:
            oracle.assert_bitexact(to_host(s.attn), h["attn"], "attn + x")


def test_pipeline_config4_one_layer_exact(cuda):
    """BASELINE config 4 at full size: 16 prompts x 1024 tokens, 256 shared,
    one decoder layer (plus the final add + LayerNorm)."""
    from aps2026_b200 import prefill

    prompts = prefill.prompts_config4()
    pipe, _, _, want_x, want_y = _run(cuda, prompts, layers=1, pool=1, exact=True)
    assert pipe.batch.rows == 256 + 16 * 768
    oracle.assert_bitexact(to_host(pipe.final_x), want_x, "final residual")
    oracle.assert_bitexact(to_host(pipe.final_out), want_y, "final LayerNorm")


def test_expand_and_last_rows(cuda):
    import torch

    from aps2026_b200 import prefill

    prompts = prefill.prompts_config4(seed=12, batch=3, length=20, shared=5)
    pipe, _, _, _, want_y = _run(cuda, prompts, layers=1, pool=1, exact=True, hidden=256)
    tokens = torch.empty((pipe.batch.tokens, 256), device=cuda)
    pipe.expand_to_tokens(tokens)
    last = torch.empty((3, 256), device=cuda)
    pipe.last_token_rows(last)
    torch.cuda.synchronize()
    tn = pipe.batch.trie.token_node
    oracle.assert_bitexact(to_host(tokens), want_y[tn], "expanded rows")
    ends = np.cumsum([len(p) for p in prompts]) - 1
    oracle.assert_bitexact(to_host(last), want_y[tn[ends]], "last-token rows")


def _grouped_prompts(seed=13):
    """Six prompts in three first-token groups (3 + 2 + 1) with shared
    prefixes inside each group, so chunks hold whole groups and node rows
    differ from token rows."""
    from aps2026_b200 import prefill

    g = np.random.default_rng(seed)
    out = []
    for n, shared in ((3, 10), (2, 20), (1, 0)):
        prefix = g.integers(0, prefill.VOCAB, max(shared, 1))
        for _ in range(n):
            out.append(np.concatenate([prefix, g.integers(0, prefill.VOCAB, 48 - prefix.size)]).astype(np.int32))
    return out


def _sharded(cuda, prompts, plan, concurrent, layers=2, pool=2, device_trie=True):
    import torch

    from aps2026_b200 import prefill

    w = prefill.Weights.make(cuda, 9, layers=layers)
    rows = prefill.ShardedPrefill.rows_needed(prompts, plan[0])
    gen = torch.Generator(device=cuda).manual_seed(21)  # same stand-ins for every runner
    sets = [prefill.StandIns.make(rows, cuda, gen) for _ in range(pool)]
    return prefill.ShardedPrefill(prompts, plan, w, cuda, sets, layers, exact=True, concurrent=concurrent,
                                  device_trie=device_trie)


@pytest.mark.parametrize("device_trie", [True, False])
def test_sharded_concurrent_chunks_match_serial_and_rebuild(cuda, device_trie):
    """One rank, three chunks: chunks on concurrent prioritised streams give
    the same token rows as one stream, bit for bit; so does an end-to-end
    step whose tries are rebuilt from host token ids -- on the device, or on
    the host and uploaded -- through the reused pinned buffers (rebuilt
    twice, to cycle both buffer sets)."""
    import torch

    from aps2026_b200.shard import chunk_plan

    prompts = _grouped_prompts()
    plan = chunk_plan(prompts, 1, 3)
    assert len(plan[0]) == 3
    serial = _sharded(cuda, prompts, plan, concurrent=False)
    serial.step()
    conc = _sharded(cuda, prompts, plan, concurrent=True)
    assert conc.streams is not None
    conc.step()
    e2e = _sharded(cuda, prompts, plan, concurrent=True, device_trie=device_trie)
    for _ in range(2):
        e2e.rebuild()
        for b, b0 in zip(e2e.batches, serial.batches):
            for name in ("node_token", "node_depth", "token_node", "last_rows"):
                assert torch.equal(getattr(b, name), getattr(b0, name)), name
    e2e.step()
    torch.cuda.synchronize()
    for c in range(3):
        assert torch.equal(conc.send[c], serial.send[c]), f"chunk {c}: concurrent != serial"
        assert torch.equal(e2e.send[c], serial.send[c]), f"chunk {c}: rebuilt != built"
    last = torch.empty((len(prompts), 4096), device=cuda)
    want = torch.empty_like(last)
    e2e.last_token_rows(last)
    serial.last_token_rows(want)
    torch.cuda.synchronize()
    assert torch.equal(last, want)
