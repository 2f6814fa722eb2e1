"""Parity of every C-ABI op against the CPU oracle on the same seeded inputs.

Integer / index / copy outputs must be bit-exact. Floating-point outputs must
meet the north_star tolerance, |d| <= 1e-6 OR |d|/|ref| <= 1e-5 (the OR form
of the reference's own validation); with B2_FLAG_EXACT_ORDER they must be
bit-exact, since that mode keeps the reference's serial reduction order.
"""
import math

import numpy as np
import pytest

import oracle
from tests._util import normal, rng, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda):
    import aps2026_b200.ops as ops

    return ops


def _sync():
    import torch

    torch.cuda.synchronize()


# ---- gather -------------------------------------------------------------------


# register-staged rows (h < 1024 or unaligned) and bulk-copy rows (one 16 KB
# chunk at h = 4096; two at h = 5000; many units per CTA at 20,000 rows)
@pytest.mark.parametrize("vocab,h,count", [(32064, 4096, 512), (1000, 4096, 1), (97, 37, 50), (64, 4100, 33),
                                           (300, 5000, 777), (4000, 1024, 3001), (32064, 4096, 20000),
                                           (50, 1020, 9)])
def test_gather_rows_bitexact(ops, cuda, vocab, h, count):
    import torch

    g = rng(10)
    emb = normal(g, (vocab, h), std=0.02)
    rows = g.integers(0, vocab, count).astype(np.uint32)
    out = torch.empty((count, h), dtype=torch.float32, device=cuda)
    ops.gather_rows_gpu(to_dev(emb, cuda), to_dev(rows, cuda), out)
    _sync()
    oracle.assert_bitexact(to_host(out), oracle.gather_rows(emb, rows), "gather")


@pytest.mark.parametrize("h", [64, 4096, 5000])
def test_gather_rows_empty_and_bad_index(ops, cuda, h):
    import torch

    emb = torch.randn(10, h, device=cuda)
    out = torch.full((3, h), 7.0, device=cuda)
    ops.gather_rows_gpu(emb, torch.zeros(0, dtype=torch.int32, device=cuda), out[:0])
    assert ops.device_status() == 0
    rows = torch.tensor([1, 10, 2], dtype=torch.int32, device=cuda)  # 10 is out of range
    ops.gather_rows_gpu(emb, rows, out)
    status = ops.device_status()
    assert status & 1, "out-of-range index not reported"
    assert torch.equal(out[1], torch.zeros(h, device=cuda))
    assert torch.equal(out[0], emb[1]) and torch.equal(out[2], emb[2])
    assert ops.device_status() == 0, "status word not cleared"


# ---- LayerNorm ----------------------------------------------------------------------

# register rows (h <= 8192 tree order, <= 4096 exact order), bulk-copy staged
# rows (aligned, h % 4 == 0, longer), scalar staged rows (h % 4 != 0); in
# exact order, >= one 16-row batch per SM (2,368 rows on 148 SMs) with h a
# multiple of 128 (and, with a residual, at least as many chunks as ring
# stages) take the chain pipeline: just above the threshold with a 1-row last
# batch (2369), one row below it (2367, per-row kernels), a 1-row last batch
# over several batches per CTA (9473), h at the add modes' minimum (640), an
# odd chunk count (1152), and many batches per CTA (20000)
PIPE_SHAPES = [(2369, 4096), (2367, 4096), (9473, 4096), (9500, 640), (9488, 1152), (20000, 1024)]
LN_SHAPES = [(512, 4096), (7, 4096), (3, 100), (5, 4100), (2, 12288), (1, 8192), (4, 2048), (3, 16384),
             (2, 37), (4800, 4096), (5003, 4100)] + PIPE_SHAPES


@pytest.mark.parametrize("rows,h", LN_SHAPES)
@pytest.mark.parametrize("exact", [False, True])
def test_layer_norm(ops, cuda, rows, h, exact):
    import torch

    g = rng(0)
    x, w, b = normal(g, (rows, h)), normal(g, h, 1.0, 0.1), normal(g, h, 0.0, 0.1)
    y = torch.empty((rows, h), device=cuda)
    ops.layer_norm_gpu(to_dev(x, cuda), to_dev(w, cuda), to_dev(b, cuda), 1e-5, y, exact=exact)
    _sync()
    want = oracle.layer_norm(x, w, b, 1e-5)
    if exact:
        oracle.assert_bitexact(to_host(y), want, "layer_norm exact")
    else:
        oracle.assert_close(to_host(y), want, what="layer_norm")


@pytest.mark.parametrize("rows,h", LN_SHAPES)
@pytest.mark.parametrize("exact", [False, True])
def test_add_layer_norm(ops, cuda, rows, h, exact):
    import torch

    g = rng(1)
    x, r = normal(g, (rows, h)), normal(g, (rows, h))
    w, b = normal(g, h, 1.0, 0.1), normal(g, h, 0.0, 0.1)
    xd, y = to_dev(x, cuda), torch.empty((rows, h), device=cuda)
    ops.add_layer_norm_gpu(xd, to_dev(r, cuda), to_dev(w, cuda), to_dev(b, cuda), 1e-5, y, exact=exact)
    _sync()
    want_x, want_y = oracle.add_layer_norm(x, r, w, b, 1e-5)
    oracle.assert_bitexact(to_host(xd), want_x, "add_layer_norm x")
    if exact:
        oracle.assert_bitexact(to_host(y), want_y, "add_layer_norm exact")
    else:
        oracle.assert_close(to_host(y), want_y, what="add_layer_norm")


def test_layer_norm_shape_errors(ops, cuda):
    import torch

    x = torch.zeros(4, 16, device=cuda)
    with pytest.raises(ValueError):
        ops.layer_norm_gpu(x, torch.ones(15, device=cuda), torch.zeros(16, device=cuda), 1e-5, torch.empty_like(x))
    with pytest.raises(ValueError):
        ops.add_layer_norm_gpu(x, torch.zeros(3, 16, device=cuda), torch.ones(16, device=cuda),
                               torch.zeros(16, device=cuda), 1e-5, torch.empty_like(x))


# ---- RoPE ------------------------------------------------------------------------------


@pytest.mark.parametrize("rows,qh,kh,hd", [(512, 32, 8, 128), (300, 16, 4, 128), (17, 4, 1, 64), (9, 3, 2, 6)])
def test_rope_bitexact(ops, cuda, rows, qh, kh, hd):
    g = rng(2)
    q, k = normal(g, (rows, qh * hd)), normal(g, (rows, kh * hd))
    max_seq = 700
    pos = g.integers(0, max_seq, rows).astype(np.uint32)
    pos[: min(rows, 4)] = [0, 1, max_seq - 1, 5][: min(rows, 4)]
    qd, kd = to_dev(q, cuda), to_dev(k, cuda)
    ops.apply_rope_tree_gpu(qd, kd, to_dev(pos, cuda), rows, max_seq, qh, kh, hd, 10000.0)
    _sync()
    cos, sin = oracle.rope_table(max_seq, hd, 10000.0)
    wq, wk = oracle.rope(q, k, pos, qh, kh, hd, cos, sin)
    oracle.assert_bitexact(to_host(qd), wq, "rope q")
    oracle.assert_bitexact(to_host(kd), wk, "rope k")


def test_rope_packed_segments(ops, cuda):
    g = rng(3)
    lens = [5, 1, 12]
    rows, qh, kh, hd = sum(lens), 2, 1, 128
    q, k = normal(g, (rows, qh * hd)), normal(g, (rows, kh * hd))
    qd, kd = to_dev(q, cuda), to_dev(k, cuda)
    ops.apply_rope_gpu(qd, kd, lens, qh, kh, hd, 10000.0)
    _sync()
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.uint32)
    cos, sin = oracle.rope_table(max(lens), hd, 10000.0)
    wq, wk = oracle.rope(q, k, pos, qh, kh, hd, cos, sin)
    oracle.assert_bitexact(to_host(qd), wq, "rope q")
    oracle.assert_bitexact(to_host(kd), wk, "rope k")


def test_rope_table_matches_oracle(ops):
    c, s = ops.rope_table_host(4096, 128, 10000.0)
    oc, os_ = oracle.rope_table(4096, 128, 10000.0)
    oracle.assert_bitexact(c.numpy(), oc, "cos")
    oracle.assert_bitexact(s.numpy(), os_, "sin")


# ---- causal softmax ---------------------------------------------------------------------


@pytest.mark.parametrize("heads,T,window", [(2, 2048, 2047), (1, 2048, 4096), (3, 64, 2047), (2, 256, 100),
                                              (2, 37, 2047), (1, 4096, 2047), (1, 8192, 2047)])
@pytest.mark.parametrize("exact", [False, True])
def test_causal_softmax(ops, cuda, heads, T, window, exact):
    import torch

    g = rng(4)
    s = normal(g, (heads, T, T), std=2.0)
    probs = torch.full((heads, T, T), float("nan"), device=cuda)
    scale = 1.0 / math.sqrt(128.0)
    ops.causal_softmax_gpu(to_dev(s, cuda), probs, scale, window, exact=exact)
    _sync()
    want = oracle.causal_softmax(s, np.float32(scale), window)
    got = to_host(probs)
    if exact:
        oracle.assert_bitexact(got, want, "softmax exact")
    else:
        oracle.assert_close(got, want, what="softmax")
        # masked cells are exactly zero
        i = np.arange(T)[:, None]
        j = np.arange(T)[None, :]
        masked = (j > i) | (j < i + 1 - window)
        assert (got[:, masked] == 0).all()


@pytest.mark.parametrize("T", [256, 2048])
def test_causal_softmax_extreme_scores(ops, cuda, T):
    """Wide scores: exponentials that underflow to exactly 0 (below -104) or
    are tiny enough for the direct division, next to ordinary ones; and
    +-inf scores, whose rows must match the reference's arithmetic."""
    import torch

    g = rng(41)
    s = normal(g, (2, T, T), std=600.0)
    s[1, 5, :3] = np.float32(-np.inf)
    s[1, 7, 2] = np.float32(np.inf)
    scale = np.float32(1.0 / math.sqrt(128.0))
    want = oracle.causal_softmax(s, scale, 2047)
    for exact in (True, False):
        probs = torch.full((2, T, T), float("nan"), device=cuda)
        ops.causal_softmax_gpu(to_dev(s, cuda), probs, float(scale), 2047, exact=exact)
        _sync()
        got = to_host(probs)
        finite = np.isfinite(want)
        assert (np.isnan(got) == np.isnan(want)).all()
        if exact:
            oracle.assert_bitexact(got[finite], want[finite], "softmax exact, wide scores")
        else:
            oracle.assert_close(got[finite], want[finite], what="softmax, wide scores")


# ---- MoE routing ---------------------------------------------------------------------------


def _route_and_compare(ops, cuda, logits):
    import torch

    got = ops.moe_route_gpu(to_dev(logits, cuda))
    torch.cuda.synchronize()
    want = oracle.moe_route(logits)
    for name in ("routes", "counts", "offsets", "assignment_rows", "route_positions",
                 "work_expert64", "work_start64", "work_expert128", "work_start128"):
        g = to_host(getattr(got, name))
        w = want[name]
        oracle.assert_bitexact(g.view(w.dtype).reshape(w.shape), w, name)
    return got


# Sizes around the 256-token tile boundaries and both sides of 16384.
@pytest.mark.parametrize("T", [1, 31, 255, 256, 257, 1025, 4096, 8192, 12289, 16384, 16385, 100003])
def test_moe_route_bitexact(ops, cuda, T):
    g = rng(5)
    _route_and_compare(ops, cuda, normal(g, (T, 16)))


@pytest.mark.parametrize("T", [3000, 20000])
@pytest.mark.parametrize("E", [2, 8, 13, 32])
def test_moe_route_expert_counts(ops, cuda, E, T):
    g = rng(6)
    _route_and_compare(ops, cuda, normal(g, (T, E)))


def test_moe_route_ties_and_quantum(ops, cuda):
    g = rng(7)
    # Coarse logits make many scores equal after quantisation, and values
    # that differ by less than the 2e-2 tie margin exercise the scan rule.
    logits = (np.round(g.standard_normal((5000, 16)) * 20) / 1000).astype(np.float32)
    logits[:10] = 0.0
    logits[10:20] = np.float32(0.0005)  # the rounding boundary of the quantum
    logits[20:30, ::2] = -0.0
    _route_and_compare(ops, cuda, logits)


def test_moe_route_repeat_reuses_workspace(ops, cuda):
    import torch

    g = rng(8)
    logits = to_dev(normal(g, (4096, 16)), cuda)
    ws = ops.RouteWorkspace(4096, 16, cuda)
    a = ops.moe_route_gpu(logits, ws=ws)
    b = ops.moe_route_gpu(logits, ws=ws)
    torch.cuda.synchronize()
    assert torch.equal(a.assignment_rows, b.assignment_rows)


# ---- SiLU / combine / add --------------------------------------------------------------------


@pytest.mark.parametrize("rows,cols", [(16384, 448), (5, 7), (3, 1000)])
def test_silu_mul_bitexact(ops, cuda, rows, cols):
    import torch

    g = rng(9)
    gate, up = normal(g, (rows, cols)), normal(g, (rows, cols))
    out = torch.empty((rows, cols), device=cuda)
    ops.silu_mul_gpu(to_dev(gate, cuda), to_dev(up, cuda), out)
    _sync()
    oracle.assert_bitexact(to_host(out), oracle.silu_mul(gate, up), "silu_mul")


@pytest.mark.parametrize("rows,cols", [(16384, 448), (5, 7), (3, 1000)])
def test_silu_mul_tree_mode(ops, cuda, rows, cols):
    """b2_silu_mul_flags without B2_FLAG_EXACT_ORDER: expf and __fdividef,
    within the tree-order tolerance, including the saturated tails."""
    import torch

    g = rng(61)
    gate = normal(g, (rows, cols), std=30.0)
    gate.ravel()[:4] = np.float32([-200.0, 200.0, -88.5, 0.0])[: min(4, gate.size)]
    up = normal(g, (rows, cols))
    out = torch.empty((rows, cols), dtype=torch.float32, device=cuda)
    gd, ud = to_dev(gate, cuda), to_dev(up, cuda)
    ops.silu_mul_gpu(gd, ud, out, exact=False)
    _sync()
    oracle.assert_close(to_host(out), oracle.silu_mul(gate, up), what="silu_mul tree mode")


def test_silu_mul_concatenated_layout(ops, cuda):
    import torch

    g = rng(11)
    gu = normal(g, (1024, 896))  # [2T, gate | up]
    d = to_dev(gu, cuda)
    out = torch.empty((1024, 448), device=cuda)
    ops.silu_mul_gpu(d[:, :448], d[:, 448:], out)
    _sync()
    oracle.assert_bitexact(to_host(out), oracle.silu_mul(gu[:, :448], gu[:, 448:]), "silu_mul concat")


@pytest.mark.parametrize("T,h", [(8192, 4096), (3, 4096), (50, 37)])
def test_moe_combine_bitexact(ops, cuda, T, h):
    import torch

    g = rng(12)
    r = oracle.moe_route(normal(g, (T, 16)))
    eo = normal(g, (2 * T, h))
    out = torch.empty((T, h), device=cuda)
    ops.moe_combine_gpu(to_dev(eo, cuda), to_dev(r["routes"], cuda), to_dev(r["route_positions"], cuda), out)
    _sync()
    oracle.assert_bitexact(to_host(out), oracle.moe_combine(eo, r["routes"], r["route_positions"], T), "combine")


@pytest.mark.parametrize("T,h", [(4096, 4096), (5, 100), (3, 12288), (6, 8192), (4801, 4096)] + PIPE_SHAPES)
@pytest.mark.parametrize("exact", [False, True])
def test_moe_combine_add_layer_norm(ops, cuda, T, h, exact):
    import torch

    g = rng(13)
    r = oracle.moe_route(normal(g, (T, 16)))
    eo, carry = normal(g, (2 * T, h)), normal(g, (T, h))
    w, b = normal(g, h, 1.0, 0.1), normal(g, h, 0.0, 0.1)
    x_out, y = torch.empty((T, h), device=cuda), torch.empty((T, h), device=cuda)
    ops.moe_combine_add_layer_norm_gpu(to_dev(eo, cuda), to_dev(r["routes"], cuda), to_dev(r["route_positions"], cuda),
                                       to_dev(carry, cuda), to_dev(w, cuda), to_dev(b, cuda), 1e-5, x_out, y,
                                       exact=exact)
    _sync()
    wx, wy = oracle.moe_combine_add_layer_norm(eo, r["routes"], r["route_positions"], carry, w, b, 1e-5)
    oracle.assert_bitexact(to_host(x_out), wx, "combine+add")
    if exact:
        oracle.assert_bitexact(to_host(y), wy, "combine+add+LN exact")
    else:
        oracle.assert_close(to_host(y), wy, what="combine+add+LN")


@pytest.mark.parametrize("n", [1 << 22, 1001, 4])
def test_add_bitexact(ops, cuda, n):
    g = rng(14)
    a, b = normal(g, n), normal(g, n)
    ad = to_dev(a, cuda)
    ops.add_inplace_gpu(ad, to_dev(b, cuda))
    _sync()
    oracle.assert_bitexact(to_host(ad), oracle.add(a, b), "add")


# ---- the kernels' exponential ---------------------------------------------------------------


def test_fast_exp_matches_exp_double_on_every_float(ops, cuda):
    """(float)exp((double)x) as the kernels compute it (table-driven, with a
    deferral to exp(double) near float rounding midpoints) equals CUDA's own
    exp(double) rounded to float for EVERY float x in [-80, 80], plus a
    sweep beyond, where the kernels call exp(double) directly."""
    import ctypes as C

    from aps2026_b200 import _lib

    def run(lo, hi):
        c, m, s = C.c_uint64(), C.c_uint64(), C.c_uint64()
        rc = _lib.lib().b2_selfcheck_exp(lo, hi, C.addressof(c), C.addressof(m), C.addressof(s))
        assert rc == 0, _lib.last_error()
        return c.value, m.value, s.value

    bits = lambda f: int(np.float32(f).view(np.uint32))  # noqa: E731
    total = mism = slow = 0
    for lo, hi in [(0, bits(80.0) + 1), (0x80000000, bits(-80.0) + 1),     # every float with |x| <= 80
                   (bits(80.0) + 1, bits(200.0)), (bits(-80.0) + 1, bits(-200.0)),
                   (bits(-200.0), 0xFF800001),                             # every float below -200, and -inf
                   (0x7F800000, 0x7F800001 + 16), (0xFF800001, 0xFF800001 + 16)]:  # +inf and NaNs
        c, m, s = run(lo, hi)
        total, mism, slow = total + c, mism + m, slow + s
    assert total > 2_200_000_000
    assert mism == 0, f"{mism} of {total} floats differ from (float)exp((double)x)"
    # the deferral is rare inside |x| <= 80 (expected ~8e-6 of those arguments)
    inside = 2 * (bits(80.0) + 1)
    outside = total - inside
    assert slow - outside < 1e-4 * inside


def test_bounded_wait_gives_up_and_reports(ops, cuda):
    """The bounded shared-memory barrier wait of the bulk-copy kernels, on a
    barrier nothing completes: it gives up after its limit, the kernel
    returns, B2_CHECK_WAIT is reported, and the context keeps working."""
    import time

    import torch

    from aps2026_b200 import _lib

    ops.device_status()
    t0 = time.perf_counter()
    assert _lib.lib().b2_selfcheck_wait(20_000_000) == 0  # 20 ms
    assert ops.device_status() & 32
    assert time.perf_counter() - t0 < 5.0
    a, b = torch.ones(1000, device=cuda), torch.ones(1000, device=cuda)
    ops.add_inplace_gpu(a, b)
    torch.cuda.synchronize()
    assert float(a[0]) == 2.0
