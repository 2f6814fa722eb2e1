"""The prefix-tree attention core (b2_attention_tree) against the oracle's
restatement of k_attention_tree_gqa4 and against that reference kernel
itself (oracle/_ref), on trie rows of prompts with shared prefixes.
B2_FLAG_EXACT_ORDER: bit-exact; tree-order softmax sums: north_star
tolerance."""
import numpy as np
import pytest

import oracle
from tests._util import normal, rng, to_dev, to_host

pytestmark = pytest.mark.gpu


def _case(seed, prompts, length, shared, q_heads=16, kv_heads=4, hd=128):
    g = rng(seed)
    base = g.integers(0, 500, shared)
    ps = [np.concatenate([base, g.integers(0, 500, length - shared)]).astype(np.int32) for _ in range(prompts)]
    t = oracle.prefix_trie(ps, vocab=500)
    R = t["nodes"]
    q = normal(g, (R, q_heads * hd))
    k = normal(g, (R, kv_heads * hd))
    v = normal(g, (R, kv_heads * hd))
    return t, q, k, v


# head_dim 128 runs the query-blocked kernel (4 path rows per CTA) and, in tree
# order, the tensor-core kernel on 32-row path blocks; 64 the per-row kernel;
# lengths not divisible by 4 or 32 leave partial blocks and blocks that
# straddle prompt starts (30 prompts of 9 tokens: nearly every 32-row block is
# left to the CUDA-core kernel); window 100 < depth.
@pytest.mark.parametrize("prompts,length,shared,window,hd", [(3, 300, 40, 2047, 128), (2, 700, 10, 100, 128),
                                                              (1, 5, 0, 2047, 128), (5, 37, 3, 2047, 128),
                                                              (30, 9, 2, 2047, 128), (3, 130, 20, 50, 64)])
@pytest.mark.parametrize("exact", [True, False])
def test_attention_tree_vs_oracle(cuda, prompts, length, shared, window, hd, exact):
    import torch

    from aps2026_b200 import ops

    t, q, k, v = _case(50, prompts, length, shared, hd=hd)
    R, stride = t["nodes"], t["node_anc"].shape[1]
    want = oracle.attention_tree(q, k, v, t["node_depth"], t["node_anc"], 16, 4, hd, window)
    out = torch.full((R, 16 * hd), float("nan"), device=cuda)
    pos, anc = to_dev(t["node_depth"], cuda), to_dev(np.ascontiguousarray(t["node_anc"]), cuda)
    ops.attention_tree_gpu(to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda), out, pos, anc, stride, R, 16, 4, hd,
                           window, exact=exact)
    torch.cuda.synchronize()
    if exact:
        oracle.assert_bitexact(to_host(out), want, "attention exact")
    else:
        oracle.assert_close(to_host(out), want, what="attention")
    assert ops.device_status() == 0


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref/libref.so not built")
def test_attention_tree_vs_reference_kernel(cuda):
    import torch

    from aps2026_b200 import ops

    t, q, k, v = _case(51, 4, 400, 64)
    R, stride = t["nodes"], t["node_anc"].shape[1]
    qd, kd, vd = to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda)
    pos, anc = to_dev(t["node_depth"], cuda), to_dev(np.ascontiguousarray(t["node_anc"]), cuda)
    ref = torch.empty((R, 16 * 128), device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    rc = oracle.ref().ref_k_attention_tree(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), ref.data_ptr(),
                                           pos.data_ptr(), anc.data_ptr(), stride, R, stride, 16, 4, 128, st)
    assert rc == 0
    torch.cuda.synchronize()
    want = oracle.attention_tree(q, k, v, t["node_depth"], t["node_anc"], 16, 4, 128, oracle.ref().ref_sliding_window())
    oracle.assert_bitexact(want, to_host(ref), "oracle vs reference attention")
    out = torch.empty_like(ref)
    ops.attention_tree_gpu(qd, kd, vd, out, pos, anc, stride, R, 16, 4, 128, 2047, exact=True)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), to_host(ref), "b2 exact vs reference attention")


def test_attention_tree_bad_index_is_reported(cuda):
    import torch

    from aps2026_b200 import ops

    t, q, k, v = _case(52, 1, 20, 0)
    R, stride = t["nodes"], t["node_anc"].shape[1]
    anc = np.ascontiguousarray(t["node_anc"]).copy()
    anc[5, 2] = R + 100                       # a chain entry outside the rows
    depth = t["node_depth"].copy()
    depth[7] = stride                          # a position outside the ancestor table
    out = torch.empty((R, 16 * 128), device=cuda)
    ops.attention_tree_gpu(to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda), out, to_dev(depth, cuda),
                           to_dev(anc, cuda), stride, R, 16, 4, 128, 2047)
    status = ops.device_status()
    assert status & 8
    assert torch.equal(out[7], torch.zeros_like(out[7]))


def test_attention_tree_inconsistent_ancestors_fall_back_per_row(cuda):
    """Rows linked as parent and child whose ancestor rows disagree further
    up (not a trie's table) are computed one row at a time, each from its
    own ancestor row, as the reference kernel reads them."""
    import torch

    from aps2026_b200 import ops

    t, q, k, v = _case(53, 2, 60, 0)
    R, stride = t["nodes"], t["node_anc"].shape[1]
    anc = np.ascontiguousarray(t["node_anc"]).copy()
    anc[10, 3] = 70  # a node of the other prompt, still a valid row
    want = oracle.attention_tree(q, k, v, t["node_depth"], anc, 16, 4, 128, 2047)
    out = torch.empty((R, 16 * 128), device=cuda)
    ops.attention_tree_gpu(to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda), out, to_dev(t["node_depth"], cuda),
                           to_dev(anc, cuda), stride, R, 16, 4, 128, 2047, exact=True)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), want, "attention, inconsistent ancestors")
    assert ops.device_status() == 0


@pytest.mark.parametrize("hd", [128, 64])
def test_attention_tree_compact_chains_match_dense(cuda, hd):
    """The compact ancestor form (device trie witnesses + token_node) gives
    the same outputs as the dense table, bit for bit, on a batch with shared
    prefixes; a witness that does not reach a row's depth is reported."""
    import torch

    from aps2026_b200 import ops

    g = rng(54)
    base = g.integers(0, 500, 40)
    prompts = [np.concatenate([base[:int(g.integers(0, 41))], g.integers(0, 500, int(g.integers(1, 200)))])
               .astype(np.int32) for _ in range(7)]
    ids = torch.from_numpy(np.concatenate(prompts)).to(cuda)
    offs = np.zeros(len(prompts) + 1, np.int32)
    offs[1:] = np.cumsum([len(p) for p in prompts])
    offs_d = torch.from_numpy(offs).to(cuda)
    dt = ops.prefix_trie_device(ids, offs_d, vocab=500)
    t = oracle.prefix_trie(prompts, vocab=500)
    R, stride = t["nodes"], t["node_anc"].shape[1]
    assert dt.nodes == R
    q, k, v = normal(g, (R, 16 * hd)), normal(g, (R, 4 * hd)), normal(g, (R, 4 * hd))
    qd, kd, vd = to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda)
    pos = to_dev(t["node_depth"], cuda)
    dense = torch.empty((R, 16 * hd), device=cuda)
    ops.attention_tree_gpu(qd, kd, vd, dense, pos, to_dev(np.ascontiguousarray(t["node_anc"]), cuda), stride, R, 16,
                           4, hd, 2047, exact=True)
    compact = torch.full_like(dense, float("nan"))
    ops.attention_tree_compact_gpu(qd, kd, vd, compact, pos, dt.node_prompt, offs_d, dt.token_node, stride, R, 16, 4,
                                   hd, 2047, exact=True)
    torch.cuda.synchronize()
    assert torch.equal(compact, dense)
    assert ops.device_status() == 0
    bad = dt.node_prompt.clone()
    deep = int(np.argmax(t["node_depth"]))
    short = int(np.argmin([len(p) for p in prompts]))
    bad[deep] = short  # that prompt is shorter than the node's depth
    ops.attention_tree_compact_gpu(qd, kd, vd, compact, pos, bad, offs_d, dt.token_node, stride, R, 16, 4, hd, 2047)
    assert ops.device_status() & 8
    assert torch.equal(compact[deep], torch.zeros_like(compact[deep]))


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref/libref.so not built")
def test_packed_segments_match_reference_grouped_kernel(cuda):
    """attention_gpu's packed-segment attention (k_attention_grouped_gqa4) is
    the compact-chain kernel with token_node = identity and one chain per
    segment -- the mapping the C++ shim uses; bit-exact to the reference."""
    import torch

    from aps2026_b200 import ops

    lens = [300, 5, 129, 1, 64]
    rows = sum(lens)
    offs = np.zeros(len(lens) + 1, np.int32)
    offs[1:] = np.cumsum(lens)
    seg = np.repeat(np.arange(len(lens), dtype=np.int32), lens)
    pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
    base = offs[:-1][seg]
    g = rng(55)
    q, k, v = normal(g, (rows, 16 * 128)), normal(g, (rows, 4 * 128)), normal(g, (rows, 4 * 128))
    qd, kd, vd = to_dev(q, cuda), to_dev(k, cuda), to_dev(v, cuda)
    ref = torch.full((rows, 16 * 128), float("nan"), device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    base_d, pos_d = to_dev(base, cuda), to_dev(pos, cuda)  # alive until the kernels have run
    rc = oracle.ref().ref_k_attention_grouped(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), ref.data_ptr(),
                                              base_d.data_ptr(), pos_d.data_ptr(), rows, max(lens), 16, 4, 128, st)
    assert rc == 0
    out = torch.full_like(ref, float("nan"))
    ident = torch.arange(rows, dtype=torch.int32, device=cuda)
    seg_d, offs_d = to_dev(seg, cuda), to_dev(offs, cuda)
    ops.attention_tree_compact_gpu(qd, kd, vd, out, pos_d, seg_d, offs_d, ident, max(lens), rows, 16, 4, 128,
                                   exact=True)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), to_host(ref), "compact chains vs k_attention_grouped_gqa4")


def _compact_case(cuda, seed, prompts_n, max_len, shared):
    import torch

    from aps2026_b200 import ops

    g = rng(seed)
    base = g.integers(0, 500, shared)
    prompts = [np.concatenate([base[:int(g.integers(0, shared + 1))], g.integers(0, 500, int(g.integers(1, max_len)))])
               .astype(np.int32) for _ in range(prompts_n)]
    offs = np.zeros(len(prompts) + 1, np.int32)
    offs[1:] = np.cumsum([len(p) for p in prompts])
    offs_d = torch.from_numpy(offs).to(cuda)
    dt = ops.prefix_trie_device(torch.from_numpy(np.concatenate(prompts)).to(cuda), offs_d, vocab=500)
    R = dt.nodes
    q, k, v = (to_dev(normal(g, (R, n * 128)), cuda) for n in (16, 4, 4))
    stride = max(len(p) for p in prompts)
    return dict(q=q, k=k, v=v, pos=dt.node_depth, prompt=dt.node_prompt, offs=offs_d, token_node=dt.token_node,
                stride=stride, rows=R)


def _run_compact(c, exact, out=None):
    import torch

    from aps2026_b200 import ops

    out = torch.full_like(c["q"], float("nan")) if out is None else out
    ops.attention_tree_compact_gpu(c["q"], c["k"], c["v"], out, c["pos"], c["prompt"], c["offs"], c["token_node"],
                                   c["stride"], c["rows"], 16, 4, 128, 2047, exact=exact)
    return out


def test_attention_tree_order_compact_scratch_reuse(cuda):
    """Tree order with compact chains, three calls in a row -- a large batch,
    a small one, the large one again -- so the tensor-core path's scratch
    comes from the library's pool at two sizes: every output within the
    tolerance of the exact-order output, and the repeated call bit-identical
    to the first."""
    import torch

    from aps2026_b200 import ops

    big = _compact_case(cuda, 56, 12, 900, 300)
    small = _compact_case(cuda, 57, 5, 120, 40)
    first = _run_compact(big, False)
    mid = _run_compact(small, False)
    again = _run_compact(big, False)
    want_big, want_small = _run_compact(big, True), _run_compact(small, True)
    torch.cuda.synchronize()
    oracle.assert_close(to_host(first), to_host(want_big), what="tree order vs exact order (large batch)")
    oracle.assert_close(to_host(mid), to_host(want_small), what="tree order vs exact order (small batch)")
    assert torch.equal(first, again)
    assert ops.device_status() == 0


def test_attention_tree_order_under_graph_capture(cuda):
    """The tree-order call captured in a CUDA graph (its scratch becomes a
    graph allocation) and replayed twice gives the eager call's outputs, bit
    for bit."""
    import torch

    from aps2026_b200 import ops

    c = _compact_case(cuda, 58, 8, 500, 200)
    eager = _run_compact(c, False)
    torch.cuda.synchronize()
    out = torch.full_like(c["q"], float("nan"))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        _run_compact(c, False, out)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _run_compact(c, False, out)
    for _ in range(2):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    del graph
    assert ops.device_status() == 0
