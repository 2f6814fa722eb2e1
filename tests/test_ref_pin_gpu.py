"""Pins the oracle -- and the product kernels -- to the REFERENCE's own CUDA
kernels (ezzy0654/aps2026 src/tensor.cu, built from its own source into
oracle/_ref/libref.so) on identical seeded inputs.

Two relations are checked per op:
  reference kernel == oracle            (bit for bit: the oracle is pinned)
  reference kernel == product kernel    (bit for bit for integer ops and
                                         B2_FLAG_EXACT_ORDER float ops;
                                         north_star tolerance for the
                                         default tree-order reductions)
The causal softmax has no standalone reference kernel; its probabilities are
read out of the reference attention kernel by one-hot keys and values (the
dot products and the value sums then add exact zeros only).
"""
import math

import numpy as np
import pytest

import oracle
from tests._util import normal, rng, to_dev, to_host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref/libref.so not built")]


@pytest.fixture(scope="module")
def ops(cuda):
    import aps2026_b200.ops as ops

    return ops


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def _run(rc):
    import torch

    assert rc == 0, f"reference launch failed: cuda error {rc}"
    torch.cuda.synchronize()


def test_ref_gather(ops, cuda):
    import torch

    g = rng(20)
    emb = normal(g, (5000, 4096), std=0.02)
    rows = g.integers(0, 5000, 300).astype(np.uint32)
    e, r = to_dev(emb, cuda), to_dev(rows, cuda)
    ref_out = torch.empty((300, 4096), device=cuda)
    _run(oracle.ref().ref_k_gather_rows(e.data_ptr(), r.data_ptr(), ref_out.data_ptr(), 300, 4096, _stream()))
    oracle.assert_bitexact(oracle.gather_rows(emb, rows), to_host(ref_out), "oracle vs ref gather")
    out = torch.empty_like(ref_out)
    ops.gather_rows_gpu(e, r, out)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), to_host(ref_out), "b2 vs ref gather")


# 2369 and 9473 x 4096: the exact-order chain pipeline (>= 2,368 rows), 1-row last batch
@pytest.mark.parametrize("rows,h", [(512, 4096), (9, 100), (3, 4100), (2369, 4096), (9473, 4096)])
def test_ref_layer_norm(ops, cuda, rows, h):
    import torch

    g = rng(21)
    x, w, b = normal(g, (rows, h)), normal(g, h, 1.0, 0.1), normal(g, h, 0.0, 0.1)
    xd, wd, bd = to_dev(x, cuda), to_dev(w, cuda), to_dev(b, cuda)
    ref_y = torch.empty_like(xd)
    _run(oracle.ref().ref_k_layer_norm(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), ref_y.data_ptr(), rows, h,
                                       1e-5, _stream()))
    ry = to_host(ref_y)
    oracle.assert_bitexact(oracle.layer_norm(x, w, b, 1e-5), ry, "oracle vs ref LN")
    for exact in (True, False):
        y = torch.empty_like(xd)
        ops.layer_norm_gpu(xd, wd, bd, 1e-5, y, exact=exact)
        torch.cuda.synchronize()
        if exact:
            oracle.assert_bitexact(to_host(y), ry, "b2 exact vs ref LN")
        else:
            oracle.assert_close(to_host(y), ry, what="b2 vs ref LN")


@pytest.mark.parametrize("rows,h", [(512, 4096), (5, 36), (9473, 4096)])
def test_ref_add_layer_norm(ops, cuda, rows, h):
    import torch

    g = rng(22)
    x, r = normal(g, (rows, h)), normal(g, (rows, h))
    w, b = normal(g, h, 1.0, 0.1), normal(g, h, 0.0, 0.1)
    rd, wd, bd = to_dev(r, cuda), to_dev(w, cuda), to_dev(b, cuda)
    ref_x, ref_y = to_dev(x, cuda), torch.empty((rows, h), device=cuda)
    _run(oracle.ref().ref_k_add_layer_norm(ref_x.data_ptr(), rd.data_ptr(), wd.data_ptr(), bd.data_ptr(),
                                           ref_y.data_ptr(), rows, h, 1e-5, _stream()))
    ox, oy = oracle.add_layer_norm(x, r, w, b, 1e-5)
    oracle.assert_bitexact(ox, to_host(ref_x), "oracle vs ref add-LN x")
    oracle.assert_bitexact(oy, to_host(ref_y), "oracle vs ref add-LN y")
    xd, y = to_dev(x, cuda), torch.empty((rows, h), device=cuda)
    ops.add_layer_norm_gpu(xd, rd, wd, bd, 1e-5, y, exact=True)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(xd), to_host(ref_x), "b2 vs ref add-LN x")
    oracle.assert_bitexact(to_host(y), to_host(ref_y), "b2 exact vs ref add-LN y")


@pytest.mark.parametrize("qh,kh", [(32, 8), (16, 4)])
def test_ref_rope(ops, cuda, qh, kh):
    import torch

    g = rng(23)
    rows, hd, max_seq = 512, 128, 512
    q, k = normal(g, (rows, qh * hd)), normal(g, (rows, kh * hd))
    pos = np.arange(rows, dtype=np.uint32)
    g.shuffle(pos)
    cos, sin = ops.rope_table_gpu(max_seq, hd, 10000.0, cuda)
    pd = to_dev(pos, cuda)
    rq, rk = to_dev(q, cuda), to_dev(k, cuda)
    _run(oracle.ref().ref_k_rope(rq.data_ptr(), rk.data_ptr(), pd.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                 rows, qh, kh, hd, _stream()))
    oc, os_ = oracle.rope_table(max_seq, hd, 10000.0)
    wq, wk = oracle.rope(q, k, pos, qh, kh, hd, oc, os_)
    oracle.assert_bitexact(wq, to_host(rq), "oracle vs ref rope q")
    oracle.assert_bitexact(wk, to_host(rk), "oracle vs ref rope k")
    bq, bk = to_dev(q, cuda), to_dev(k, cuda)
    ops.apply_rope_tree_gpu(bq, bk, pd, rows, max_seq, qh, kh, hd, 10000.0)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(bq), to_host(rq), "b2 vs ref rope q")
    oracle.assert_bitexact(to_host(bk), to_host(rk), "b2 vs ref rope k")


def test_ref_rope_cpu_twin_agrees():
    """The reference's host apply_rope (per-element cos/sin, no fused
    multiply-add) agrees with the oracle within tolerance."""
    g = rng(24)
    lens = np.array([7, 3], dtype=np.uint64)
    rows, qh, kh, hd = 10, 4, 1, 128
    q, k = normal(g, (rows, qh * hd)), normal(g, (rows, kh * hd))
    rq, rk = q.copy(), k.copy()
    oracle.ref().ref_cpu_apply_rope(rq.ctypes.data, rk.ctypes.data, lens.ctypes.data, 2, qh, kh, hd, 10000.0,
                                    None)
    pos = np.concatenate([np.arange(7), np.arange(3)]).astype(np.uint32)
    c, s = oracle.rope_table(7, hd, 10000.0)
    wq, wk = oracle.rope(q, k, pos, qh, kh, hd, c, s)
    oracle.assert_close(wq, rq, what="rope q vs reference host op")
    oracle.assert_close(wk, rk, what="rope k vs reference host op")


@pytest.mark.parametrize("T", [1, 300, 8192, 40000])
def test_ref_moe_route(ops, cuda, T):
    import torch

    g = rng(25)
    logits = normal(g, (T, 16))
    if T >= 300:
        logits[:100] = (np.round(logits[:100] * 20) / 1000).astype(np.float32)  # ties
    ld = to_dev(logits, cuda)
    n64, n128 = ops.queue_lengths(T, 16)
    z = lambda n, dt=torch.int32: torch.full((n,), -1, dtype=dt, device=cuda)  # noqa: E731
    routes, counts, offsets = z(2 * T, torch.uint8), z(16), z(17)
    arows, rpos, we64, ws64, we128, ws128 = z(2 * T), z(2 * T), z(n64), z(n64), z(n128), z(n128)
    _run(oracle.ref().ref_k_moe_route(ld.data_ptr(), T, routes.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                                      arows.data_ptr(), rpos.data_ptr(), we64.data_ptr(), ws64.data_ptr(),
                                      we128.data_ptr(), ws128.data_ptr(), _stream()))
    want = oracle.moe_route(logits)
    ref = dict(routes=to_host(routes).reshape(T, 2), counts=to_host(counts, np.uint32),
               offsets=to_host(offsets, np.uint32), assignment_rows=to_host(arows, np.uint32),
               route_positions=to_host(rpos, np.uint32), work_expert64=to_host(we64, np.uint32),
               work_start64=to_host(ws64, np.uint32), work_expert128=to_host(we128, np.uint32),
               work_start128=to_host(ws128, np.uint32))
    got = ops.moe_route_gpu(ld)
    torch.cuda.synchronize()
    for name, rv in ref.items():
        ov = want[name]
        gv = to_host(getattr(got, name)).view(ov.dtype).reshape(ov.shape)
        if name.startswith("work_start"):
            # the reference writes start entries only where the expert queue is used
            used = ref["work_expert" + name[len("work_start"):]] != 0xFFFFFFFF
            rv, ov, gv = rv[used], ov[used], gv[used]
        oracle.assert_bitexact(ov, rv, f"oracle vs ref {name}")
        oracle.assert_bitexact(gv, rv, f"b2 vs ref {name}")


def test_ref_silu_combine_add(ops, cuda):
    import torch

    g = rng(26)
    T, h, inter = 2048, 4096, 448
    gate, up = normal(g, (2 * T, inter)), normal(g, (2 * T, inter))
    gd, ud = to_dev(gate, cuda), to_dev(up, cuda)
    ref_act = torch.empty_like(gd)
    _run(oracle.ref().ref_k_silu_mul(gd.data_ptr(), ud.data_ptr(), ref_act.data_ptr(), gate.size, _stream()))
    oracle.assert_bitexact(oracle.silu_mul(gate, up), to_host(ref_act), "oracle vs ref silu")
    act = torch.empty_like(gd)
    ops.silu_mul_gpu(gd, ud, act)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(act), to_host(ref_act), "b2 vs ref silu")
    # ... and the reference's host silu + mul agrees bit for bit too
    host = np.empty_like(gate)
    oracle.ref().ref_cpu_silu_mul(gate.ctypes.data, up.ctypes.data, host.ctypes.data, gate.size, None)
    oracle.assert_bitexact(host, to_host(ref_act), "ref host vs ref kernel silu")

    r = oracle.moe_route(normal(g, (T, 16)))
    eo = normal(g, (2 * T, h))
    ed, rt, rp = to_dev(eo, cuda), to_dev(r["routes"], cuda), to_dev(r["route_positions"], cuda)
    ref_out = torch.empty((T, h), device=cuda)
    _run(oracle.ref().ref_k_moe_combine(ed.data_ptr(), rt.data_ptr(), rp.data_ptr(), ref_out.data_ptr(), T, h,
                                        _stream()))
    oracle.assert_bitexact(oracle.moe_combine(eo, r["routes"], r["route_positions"], T), to_host(ref_out),
                           "oracle vs ref combine")
    out = torch.empty_like(ref_out)
    ops.moe_combine_gpu(ed, rt, rp, out)
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), to_host(ref_out), "b2 vs ref combine")

    a, b = normal(g, T * h), normal(g, T * h)
    ra, bd = to_dev(a, cuda), to_dev(b, cuda)
    _run(oracle.ref().ref_k_add(ra.data_ptr(), bd.data_ptr(), a.size, _stream()))
    oracle.assert_bitexact(oracle.add(a, b), to_host(ra), "oracle vs ref add")


@pytest.mark.parametrize("T", [1, 2, 77, 128])
def test_ref_softmax_via_attention(ops, cuda, T):
    """Probabilities of the reference attention kernel (one-hot K and V, so
    the scores are the query entries and the outputs are the probabilities)
    vs the oracle softmax and the product softmax (exact and default)."""
    import torch

    g = rng(27)
    hd, qh, kh = 128, 4, 1
    q = normal(g, (T, qh, hd), std=2.0 * math.sqrt(128.0) / 4)
    eye = np.zeros((T, kh * hd), np.float32)
    eye[np.arange(T), np.arange(T)] = 1.0
    pos = np.arange(T, dtype=np.uint32)
    anc = np.tile(np.arange(T, dtype=np.uint32), (T, 1))
    qd, kd = to_dev(q.reshape(T, qh * hd), cuda), to_dev(eye, cuda)
    pd, ad = to_dev(pos, cuda), to_dev(anc, cuda)
    out = torch.empty((T, qh * hd), device=cuda)
    _run(oracle.ref().ref_k_attention_tree(qd.data_ptr(), kd.data_ptr(), kd.data_ptr(), out.data_ptr(),
                                           pd.data_ptr(), ad.data_ptr(), T, T, T, qh, kh, hd, _stream()))
    ref_p = to_host(out).reshape(T, qh, hd)[:, :, :T].transpose(1, 0, 2)  # [heads, query, key]
    scores = np.ascontiguousarray(q[:, :, :T].transpose(1, 0, 2))
    scale = np.float32(1.0) / np.sqrt(np.float32(128.0))  # 1.0f / sqrtf(128.0f), as the kernel forms it
    window = oracle.ref().ref_sliding_window()
    want = oracle.causal_softmax(scores, scale, window)
    oracle.assert_bitexact(want, np.ascontiguousarray(ref_p), "oracle vs ref softmax")
    for exact in (True, False):
        probs = torch.empty((qh, T, T), device=cuda)
        ops.causal_softmax_gpu(to_dev(scores, cuda), probs, float(scale), window, exact=exact)
        torch.cuda.synchronize()
        if exact:
            oracle.assert_bitexact(to_host(probs), np.ascontiguousarray(ref_p), "b2 exact vs ref softmax")
        else:
            oracle.assert_close(to_host(probs), ref_p, what="b2 vs ref softmax")


def test_ref_moe_gather_compact(ops, cuda):
    """The permutation gather with the assignment rows of a real routing, vs
    the reference's k_moe_gather_compact and the oracle, bit for bit."""
    import torch

    g = rng(27)
    T, h = 3000, 4096
    x = normal(g, (T, h))
    logits = normal(g, (T, 16))
    r = oracle.moe_route(logits)
    arows = r["assignment_rows"]
    xd, ad = to_dev(x, cuda), to_dev(arows, cuda)
    ref = torch.full((2 * T, h), float("nan"), device=cuda)
    _run(oracle.ref().ref_k_moe_gather_compact(xd.data_ptr(), ad.data_ptr(), ref.data_ptr(), 2 * T, h, _stream()))
    got = torch.full_like(ref, float("nan"))
    ops.moe_gather_compact_gpu(xd, ad, got)
    torch.cuda.synchronize()
    want = oracle.gather_rows(x, arows)
    oracle.assert_bitexact(to_host(ref), want, "oracle vs reference gather_compact")
    oracle.assert_bitexact(to_host(got), want, "b2 vs reference gather_compact")
