"""Generates the committed golden vectors of the reference (test fixtures).

Two fixture files, both from the reference's OWN code built from its source
tree (oracle/_ref/libref.so, see oracle/Makefile) on small seeded inputs:

  ref_host_ops.npz  the reference's host ops (tensor_ops::layer_norm,
                    apply_rope, silu + mul, add_inplace; src/tensor.cu:302-367)
                    -- runs anywhere:  python tests/golden/make_golden.py host
  ref_kernels.npz   the reference's CUDA kernels (k_layer_norm,
                    k_add_layer_norm, k_rope, the routing trio, k_silu_mul,
                    k_moe_combine, k_gather_rows, and the softmax of
                    k_attention_tree_gqa4 read out through one-hot keys and
                    values) -- needs a GPU:  python tests/golden/make_golden.py gpu

Inputs are drawn from numpy's PCG64 with fixed seeds and stored next to the
outputs, so the fixtures are self-contained. tests/test_golden_cpu.py checks
the CPU oracle against both files without a GPU.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

HERE = Path(__file__).resolve().parent


def _n(g, shape, mean=0.0, std=1.0):
    return (g.standard_normal(shape) * std + mean).astype(np.float32)


def host_ops() -> dict:
    r = oracle.ref()
    g = np.random.default_rng(100)
    out = {}
    rows, h = 16, 4096
    x, w, b = _n(g, (rows, h)), _n(g, h, 1.0, 0.1), _n(g, h, 0.0, 0.1)
    y = np.empty_like(x)
    r.ref_cpu_layer_norm(x.ctypes.data, w.ctypes.data, b.ctypes.data, y.ctypes.data, rows, h, 1e-5, None)
    out.update(ln_x=x, ln_w=w, ln_b=b, ln_y=y)

    lens = np.array([9, 4], dtype=np.uint64)
    qh, kh, hd = 4, 1, 128
    q, k = _n(g, (13, qh * hd)), _n(g, (13, kh * hd))
    rq, rk = q.copy(), k.copy()
    r.ref_cpu_apply_rope(rq.ctypes.data, rk.ctypes.data, lens.ctypes.data, 2, qh, kh, hd, 10000.0, None)
    out.update(rope_q=q, rope_k=k, rope_lens=lens.astype(np.uint32), rope_q_out=rq, rope_k_out=rk)

    gate, up = _n(g, 3000, std=4.0), _n(g, 3000)
    act = np.empty_like(gate)
    r.ref_cpu_silu_mul(gate.ctypes.data, up.ctypes.data, act.ctypes.data, gate.size, None)
    out.update(silu_gate=gate, silu_up=up, silu_out=act)

    a, bb = _n(g, 3000), _n(g, 3000)
    s = a.copy()
    r.ref_cpu_add_inplace(s.ctypes.data, bb.ctypes.data, a.size, None)
    out.update(add_a=a, add_b=bb, add_out=s)
    return out


def gpu_kernels() -> dict:
    import torch

    r = oracle.ref()
    dev = torch.device("cuda", 0)
    st = torch.cuda.current_stream().cuda_stream
    keep = []  # device copies stay alive until the end: a temporary's block could be reused before its kernel runs

    def d(a):
        t = torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a)).to(dev)
        keep.append(t)
        return t

    host = lambda t: t.cpu().numpy()  # noqa: E731

    def run(rc):
        assert rc == 0, rc
        torch.cuda.synchronize()

    g = np.random.default_rng(200)
    out = {}
    # LayerNorm and add + LayerNorm
    rows, h = 8, 4096
    x, res = _n(g, (rows, h)), _n(g, (rows, h))
    w, b = _n(g, h, 1.0, 0.1), _n(g, h, 0.0, 0.1)
    y = torch.empty((rows, h), device=dev)
    run(r.ref_k_layer_norm(d(x).data_ptr(), d(w).data_ptr(), d(b).data_ptr(), y.data_ptr(), rows, h, 1e-5, st))
    out.update(ln_x=x, ln_w=w, ln_b=b, ln_y=host(y))
    xs = d(x)
    run(r.ref_k_add_layer_norm(xs.data_ptr(), d(res).data_ptr(), d(w).data_ptr(), d(b).data_ptr(), y.data_ptr(),
                               rows, h, 1e-5, st))
    out.update(aln_res=res, aln_x_out=host(xs), aln_y=host(y))

    # RoPE (tree form: trie depths as positions)
    n, qh, kh, hd, max_seq = 64, 16, 4, 128, 300
    q, k = _n(g, (n, qh * hd)), _n(g, (n, kh * hd))
    pos = g.integers(0, max_seq, n).astype(np.uint32)
    cos, sin = oracle.rope_table(max_seq, hd, 10000.0)
    qd, kd = d(q), d(k)
    run(r.ref_k_rope(qd.data_ptr(), kd.data_ptr(), d(pos).data_ptr(), d(cos).data_ptr(), d(sin).data_ptr(), n, qh,
                     kh, hd, st))
    out.update(rope_q=q, rope_k=k, rope_pos=pos, rope_max_seq=np.array(max_seq), rope_q_out=host(qd),
               rope_k_out=host(kd))

    # routing (with quantisation ties)
    T = 1000
    logits = _n(g, (T, 16))
    logits[:200] = (np.round(logits[:200] * 20) / 1000).astype(np.float32)
    n64, n128 = (2 * T + 63) // 64 + 16, (2 * T + 127) // 128 + 16
    z = lambda m, dt=torch.int32: torch.full((m,), -1, dtype=dt, device=dev)  # noqa: E731
    rt, cnt, off, ar, rp, we64, ws64, we128, ws128 = (z(2 * T, torch.uint8), z(16), z(17), z(2 * T), z(2 * T),
                                                       z(n64), z(n64), z(n128), z(n128))
    run(r.ref_k_moe_route(d(logits).data_ptr(), T, rt.data_ptr(), cnt.data_ptr(), off.data_ptr(), ar.data_ptr(),
                          rp.data_ptr(), we64.data_ptr(), ws64.data_ptr(), we128.data_ptr(), ws128.data_ptr(), st))
    u = lambda t: host(t).view(np.uint32)  # noqa: E731
    out.update(route_logits=logits, route_routes=host(rt).reshape(T, 2), route_counts=u(cnt), route_offsets=u(off),
               route_assignment_rows=u(ar), route_positions=u(rp), route_we64=u(we64), route_ws64=u(ws64),
               route_we128=u(we128), route_ws128=u(ws128))

    # SiLU * up
    gate, up = _n(g, (64, 448), std=3.0), _n(g, (64, 448))
    act = torch.empty((64, 448), device=dev)
    run(r.ref_k_silu_mul(d(gate).data_ptr(), d(up).data_ptr(), act.data_ptr(), gate.size, st))
    out.update(silu_gate=gate, silu_up=up, silu_out=host(act))

    # combine (uses the routing above)
    hc = 256
    eo = _n(g, (2 * T, hc))
    comb = torch.empty((T, hc), device=dev)
    run(r.ref_k_moe_combine(d(eo).data_ptr(), rt.data_ptr(), rp.data_ptr(), comb.data_ptr(), T, hc, st))
    out.update(comb_expert_out=eo, comb_out=host(comb))

    # gather
    emb = _n(g, (500, 64), std=0.02)
    idx = g.integers(0, 500, 100).astype(np.uint32)
    gat = torch.empty((100, 64), device=dev)
    run(r.ref_k_gather_rows(d(emb).data_ptr(), d(idx).data_ptr(), gat.data_ptr(), 100, 64, st))
    out.update(gather_emb=emb, gather_rows=idx, gather_out=host(gat))

    # softmax through the attention kernel: one-hot K and V
    Ts, heads, hd = 96, 4, 128
    qs = _n(g, (Ts, heads, hd), std=2.0 * math.sqrt(128.0) / 4)
    eye = np.zeros((Ts, hd), np.float32)
    eye[np.arange(Ts), np.arange(Ts)] = 1.0
    anc = np.tile(np.arange(Ts, dtype=np.uint32), (Ts, 1))
    o = torch.empty((Ts, heads * hd), device=dev)
    run(r.ref_k_attention_tree(d(qs.reshape(Ts, -1)).data_ptr(), d(eye).data_ptr(), d(eye).data_ptr(),
                               o.data_ptr(), d(np.arange(Ts, dtype=np.uint32)).data_ptr(), d(anc).data_ptr(),
                               Ts, Ts, Ts, heads, 1, hd, st))
    probs = host(o).reshape(Ts, heads, hd)[:, :, :Ts].transpose(1, 0, 2)
    out.update(softmax_scores=np.ascontiguousarray(qs[:, :, :Ts].transpose(1, 0, 2)),
               softmax_probs=np.ascontiguousarray(probs), softmax_window=np.array(r.ref_sliding_window()))
    return out


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "host"
    dest = Path(sys.argv[2]) if len(sys.argv) > 2 else HERE
    if which == "host":
        np.savez_compressed(dest / "ref_host_ops.npz", **host_ops())
    elif which == "gpu":
        np.savez_compressed(dest / "ref_kernels.npz", **gpu_kernels())
    else:
        raise SystemExit("usage: make_golden.py host|gpu [dest_dir]")
    print("wrote", which, "fixtures to", dest)
