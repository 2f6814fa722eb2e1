"""The device prefix trie (b2_prefix_trie_device) against the host walk
(b2_prefix_trie_build, itself checked against a restatement of the
reference's map-based walk in tests/test_host_cpu.py): identical node
numbering, tokens and depths, and node_prompt witnesses whose token rows
spell each node's ancestor chain."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _upload(prompts, cuda):
    import torch

    ids = torch.from_numpy(np.concatenate(prompts).astype(np.int32)).to(cuda)
    offs = np.zeros(len(prompts) + 1, np.int32)
    offs[1:] = np.cumsum([len(p) for p in prompts])
    return ids, torch.from_numpy(offs).to(cuda), offs


def _check_same(prompts, cuda, vocab=32064):
    from aps2026_b200 import ops

    ids, offs_d, offs = _upload(prompts, cuda)
    got = ops.prefix_trie_device(ids, offs_d, vocab=vocab)
    want = ops.prefix_trie(prompts, vocab=vocab, with_ancestors=True)
    assert got.nodes == want.nodes
    np.testing.assert_array_equal(got.token_node.cpu().numpy().view(np.uint32), want.token_node)
    np.testing.assert_array_equal(got.node_token.cpu().numpy().view(np.uint32), want.node_token)
    np.testing.assert_array_equal(got.node_depth.cpu().numpy().view(np.uint32), want.node_depth)
    # witness: prompt p holds node n at depth d, and its token rows 0..d are n's ancestor chain
    tn = want.token_node
    wp = got.node_prompt.cpu().numpy()
    for n in np.random.default_rng(0).choice(want.nodes, size=min(200, want.nodes), replace=False):
        p, d = int(wp[n]), int(want.node_depth[n])
        np.testing.assert_array_equal(tn[offs[p]:offs[p] + d + 1], want.node_anc[n, :d + 1])
    assert ops.device_status() == 0
    return got


def test_device_trie_random_shared_prefixes(cuda):
    g = np.random.default_rng(1)
    stems = [g.integers(0, 50, int(g.integers(1, 40))) for _ in range(6)]
    prompts = []
    for _ in range(40):
        s = stems[int(g.integers(0, len(stems)))][: int(g.integers(1, 41))]
        prompts.append(np.concatenate([s, g.integers(0, 50, int(g.integers(0, 30)))]).astype(np.int32))
    _check_same(prompts, cuda, vocab=50)


def test_device_trie_duplicates_and_prefixes(cuda):
    a = np.arange(100, dtype=np.int32)
    prompts = [a, a.copy(), a[:30], a[:31], np.concatenate([a[:50], [7, 7]]).astype(np.int32), a[:1],
               np.array([5], np.int32), np.concatenate([a, a]).astype(np.int32)]
    _check_same(prompts, cuda)


def test_device_trie_many_small_prompts(cuda):
    # more prompts than warps per CTA, small vocabulary: long chains of b*
    g = np.random.default_rng(2)
    prompts = [g.integers(0, 3, int(g.integers(1, 12))).astype(np.int32) for _ in range(300)]
    _check_same(prompts, cuda, vocab=3)


@pytest.mark.parametrize("which", ["config4", "config5"])
def test_device_trie_benchmark_batches(cuda, which):
    from aps2026_b200 import prefill

    prompts = prefill.prompts_config4() if which == "config4" else prefill.prompts_config5()
    got = _check_same(prompts, cuda)
    assert got.nodes == (256 + 16 * 768 if which == "config4" else 64 * 2048)


def test_device_trie_reports_bad_input(cuda):
    import torch

    from aps2026_b200 import ops

    ops.device_status()
    ids, offs_d, _ = _upload([np.array([1, 2, 3], np.int32), np.array([4, 99], np.int32)], cuda)
    ops.prefix_trie_device(ids, offs_d, vocab=50)  # 99 is outside the vocabulary
    assert ops.device_status() & 16
    offs_bad = torch.tensor([0, 0, 5], dtype=torch.int32, device=cuda)  # an empty prompt
    ops.prefix_trie_device(ids, offs_bad, vocab=100)
    assert ops.device_status() & 16
    with pytest.raises(ops.InvalidArgument):
        ops.prefix_trie_device(ids, torch.zeros(1, dtype=torch.int32, device=cuda))
