"""Host logic on the CPU: the prefix trie against the oracle's restatement of
the reference walk, oracle properties (routing permutation, softmax rows),
and input validation."""
import numpy as np
import pytest

import oracle
from aps2026_b200 import ops
from tests._util import normal, rng


def _prompts(g, batch, length, shared, vocab=32064):
    base = g.integers(0, vocab, shared)
    out = []
    for _ in range(batch):
        n = length if isinstance(length, int) else int(g.integers(length[0], length[1]))
        tail = g.integers(0, vocab, max(n - shared, 0))
        out.append(np.concatenate([base[: min(shared, n)], tail]).astype(np.int32))
    return out


@pytest.mark.parametrize("batch,length,shared", [(16, 1024, 256), (5, (1, 40), 3), (1, 7, 0), (8, 50, 50)])
def test_trie_matches_reference_walk(batch, length, shared):
    g = rng(30)
    prompts = _prompts(g, batch, length, shared, vocab=50 if batch == 5 else 32064)
    got = ops.prefix_trie(prompts, with_ancestors=True)
    want = oracle.prefix_trie(prompts)
    assert got.nodes == want["nodes"]
    oracle.assert_bitexact(got.token_node, want["token_node"], "token_node")
    oracle.assert_bitexact(got.node_token, want["node_token"], "node_token")
    oracle.assert_bitexact(got.node_depth, want["node_depth"], "node_depth")
    oracle.assert_bitexact(got.node_anc, want["node_anc"], "node_anc")


def test_trie_config4_shape():
    g = rng(3)
    prompts = _prompts(g, 16, 1024, 256)
    t = ops.prefix_trie(prompts)
    assert t.nodes == 256 + 16 * 768  # shared prefix collapses to one chain
    # every token's node carries its token and depth
    ids = np.concatenate(prompts)
    depth = np.concatenate([np.arange(len(p)) for p in prompts])
    assert (t.node_token[t.token_node] == ids).all()
    assert (t.node_depth[t.token_node] == depth).all()


def test_trie_errors():
    with pytest.raises(ValueError, match="empty input batch"):
        ops.prefix_trie([])
    with pytest.raises(ValueError, match="out of vocabulary"):
        ops.prefix_trie([[1, 2, 40000]])
    with pytest.raises(ValueError, match="out of vocabulary"):
        ops.prefix_trie([[1, -1]])
    with pytest.raises(ValueError, match="too long"):
        ops.prefix_trie([[1] * 10], max_len=9)
    with pytest.raises(ValueError, match="empty input"):
        ops.prefix_trie([[1], []])


@pytest.mark.parametrize("T,E", [(1, 16), (1000, 16), (777, 5)])
def test_oracle_routing_is_a_stable_permutation(T, E):
    g = rng(31)
    logits = normal(g, (T, E))
    r = oracle.moe_route(logits)
    routes, rp, ar, off = r["routes"], r["route_positions"], r["assignment_rows"], r["offsets"]
    assert (routes[:, 0] != routes[:, 1]).all()
    assert np.array_equal(np.sort(rp), np.arange(2 * T))          # a permutation
    assert np.array_equal(ar[rp], np.repeat(np.arange(T), 2))       # inverse relation
    assert np.array_equal(np.diff(off), r["counts"])
    for e in range(E):
        seg = ar[off[e]:off[e + 1]]
        assert (np.diff(seg.astype(np.int64)) > 0).all()             # stable: ascending tokens
        assert (routes[seg] == e).any(axis=1).all()


def test_oracle_routing_rule():
    # quantised scores, scan order, replace only on > best + 0.02
    logits = np.zeros((4, 4), np.float32)
    logits[0] = [0.10, 0.115, 0.13, 0.0]     # 0.13 > 0.10 + 0.02 -> expert 2; second: 0.115 vs 0.10 -> 0
    logits[1] = [0.0, 0.0, 0.0, 0.0]         # all tied -> 0, 1
    logits[2] = [-1.0, -0.5, -0.2, -0.7]     # first 2; second 1
    logits[3] = [0.0004, 0.0006, 0.0, 0.0]   # quantised to 0.0 and 0.001 -> ties -> 0, 1
    r = oracle.moe_route(logits)
    assert r["routes"].tolist() == [[2, 0], [0, 1], [2, 1], [0, 1]]


def test_oracle_softmax_rows():
    g = rng(32)
    s = normal(g, (2, 50, 50), std=2.0)
    p = oracle.causal_softmax(s, np.float32(0.5), 20)
    i, j = np.arange(50)[:, None], np.arange(50)[None, :]
    inside = (j <= i) & (j > i - 20)
    assert (p[:, ~inside] == 0).all()
    np.testing.assert_allclose(p.sum(-1), 1.0, rtol=1e-5)


def test_close_mask_or_criterion():
    want = np.array([1.0, 1e-3, 0.0, 1.0], np.float32)
    got = np.array([1.0 + 9e-6, 1e-3 + 9e-7, 9e-7, np.nan], np.float32)
    assert oracle.close_mask(got, want).tolist() == [True, True, True, False]


def test_bytes_per_row_accounting():
    """The algorithmic bytes behind every GB/s figure: each logical tensor
    read or written once. The reference's unfused config-5 sequence moves
    6,835,072 B per row (per layer: add + LN 65,536, RoPE 20,480, add + LN
    65,536, routing 82, SiLU 10,752, un-permute 49,162; minus layer 0's carry
    32,768; plus gather 32,768 and the final add + LN 65,536); the fused
    un-permute + add + LN saves the 16 KB write and re-read of each MoE
    output row per layer."""
    from aps2026_b200 import prefill

    h = 4096 * 4
    d = prefill.bytes_per_row(32)
    assert d["gather"] == 2 * h and d["ln0"] == 2 * h
    assert d["rope"] == 2 * (16 + 4) * 128 * 4
    assert d["add_ln"] == 4 * h
    assert d["route"] == 16 * 4 + 2 + 2 * 4 * 2
    assert d["silu"] == 2 * 448 * 12
    assert d["fused"] == 49_162 + 4 * h - 2 * h  # un-permute + add + LN, one pass
    reference = 32 * (65_536 + 20_480 + 65_536 + 82 + 10_752 + 49_162) - 32_768 + 32_768 + 65_536
    assert reference == 6_835_072
    assert d["total"] == reference - 32 * 2 * h == 5_786_496
