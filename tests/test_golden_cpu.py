"""Pins the CPU oracle to the reference's own outputs without a GPU.

Fixtures (tests/golden/make_golden.py):
  ref_host_ops.npz -- the reference's host ops (tensor_ops::layer_norm,
                      apply_rope, silu + mul, add_inplace);
  ref_kernels.npz  -- the reference's CUDA kernels, run on a B200 from the
                      reference's own source (oracle/_ref).
The kernel fixtures must match the oracle bit for bit (the oracle follows
the kernels' arithmetic, fused multiply-adds included). The host ops agree
bit for bit too except apply_rope, whose host build fuses the other product
of `x1 * c + x0 * s` than nvcc does in k_rope; it agrees within tolerance.
"""
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def host_ops():
    return np.load(GOLDEN / "ref_host_ops.npz")


@pytest.fixture(scope="module")
def kernels():
    path = GOLDEN / "ref_kernels.npz"
    if not path.exists():
        pytest.fail("tests/golden/ref_kernels.npz missing: run make_golden.py gpu on a GPU box")
    return np.load(path)


def test_host_layer_norm(host_ops):
    f = host_ops
    oracle.assert_bitexact(oracle.layer_norm(f["ln_x"], f["ln_w"], f["ln_b"], 1e-5), f["ln_y"], "LN")


def test_host_rope(host_ops):
    f = host_ops
    lens = f["rope_lens"]
    pos = np.concatenate([np.arange(n) for n in lens]).astype(np.uint32)
    c, s = oracle.rope_table(int(lens.max()), 128, 10000.0)
    q, k = oracle.rope(f["rope_q"], f["rope_k"], pos, 4, 1, 128, c, s)
    oracle.assert_close(q, f["rope_q_out"], what="rope q")
    oracle.assert_close(k, f["rope_k_out"], what="rope k")


def test_host_silu_add(host_ops):
    f = host_ops
    oracle.assert_bitexact(oracle.silu_mul(f["silu_gate"][None], f["silu_up"][None])[0], f["silu_out"], "silu")
    oracle.assert_bitexact(oracle.add(f["add_a"], f["add_b"]), f["add_out"], "add")


def test_kernel_layer_norms(kernels):
    f = kernels
    oracle.assert_bitexact(oracle.layer_norm(f["ln_x"], f["ln_w"], f["ln_b"], 1e-5), f["ln_y"], "k_layer_norm")
    x, y = oracle.add_layer_norm(f["ln_x"], f["aln_res"], f["ln_w"], f["ln_b"], 1e-5)
    oracle.assert_bitexact(x, f["aln_x_out"], "k_add_layer_norm x")
    oracle.assert_bitexact(y, f["aln_y"], "k_add_layer_norm y")


def test_kernel_rope(kernels):
    f = kernels
    c, s = oracle.rope_table(int(f["rope_max_seq"]), 128, 10000.0)
    q, k = oracle.rope(f["rope_q"], f["rope_k"], f["rope_pos"], 16, 4, 128, c, s)
    oracle.assert_bitexact(q, f["rope_q_out"], "k_rope q")
    oracle.assert_bitexact(k, f["rope_k_out"], "k_rope k")


def test_kernel_routing(kernels):
    f = kernels
    r = oracle.moe_route(f["route_logits"])
    oracle.assert_bitexact(r["routes"], f["route_routes"], "routes")
    for name, key in [("counts", "route_counts"), ("offsets", "route_offsets"),
                      ("assignment_rows", "route_assignment_rows"), ("route_positions", "route_positions"),
                      ("work_expert64", "route_we64"), ("work_expert128", "route_we128")]:
        oracle.assert_bitexact(r[name], f[key], name)
    for ex, st in (("route_we64", "route_ws64"), ("route_we128", "route_ws128")):
        used = f[ex] != 0xFFFFFFFF
        name = "work_start" + ex[-2:] if ex.endswith("64") else "work_start128"
        oracle.assert_bitexact(r["work_start64" if ex.endswith("e64") else "work_start128"][used], f[st][used], name)


def test_kernel_silu_combine_gather(kernels):
    f = kernels
    oracle.assert_bitexact(oracle.silu_mul(f["silu_gate"], f["silu_up"]), f["silu_out"], "k_silu_mul")
    T = f["route_logits"].shape[0]
    oracle.assert_bitexact(oracle.moe_combine(f["comb_expert_out"], f["route_routes"], f["route_positions"], T),
                           f["comb_out"], "k_moe_combine")
    oracle.assert_bitexact(oracle.gather_rows(f["gather_emb"], f["gather_rows"]), f["gather_out"], "k_gather_rows")


def test_kernel_softmax(kernels):
    f = kernels
    scale = np.float32(1.0) / np.sqrt(np.float32(128.0))
    want = oracle.causal_softmax(f["softmax_scores"], scale, int(f["softmax_window"]))
    oracle.assert_bitexact(want, f["softmax_probs"], "softmax of k_attention_tree_gqa4")
