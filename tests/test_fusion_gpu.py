"""The GEMM fusion hooks (include/aps2026_b200_fusion.cuh): RoPE applied in a
projection GEMM's epilogue and LayerNorm applied in the next GEMM's prologue
give bit for bit what the separate b2_rope / b2_layer_norm launches give.

tests/fusion_harness.cu, compiled here, is a plain GEMM standing in for a
caller's kernel, with and without the hooks (ezzy0654/aps2026
docs/2026-08-26-optimization.md:217-219 names the RoPE epilogue; the
reference's 8x8 tile keeps each rotation pair in one thread). Compared:
  - GEMM + epilogue vs GEMM then b2_rope (q and k, 4 + 1 heads of 128);
  - GEMM with the prologue on x and b2_layer_norm_stats vs GEMM on
    b2_layer_norm's output, in reference order (bit for bit) and in tree
    order (the statistics of the two calls may differ in the last ulp:
    tolerance);
  - the prologue alone at 9,473 x 4,096 (a size at which b2_layer_norm takes
    its chain pipeline) vs b2_layer_norm, bit for bit, and the statistics vs
    the CPU oracle's LayerNorm.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from tests._util import normal, rng, to_dev, to_host

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def ops(cuda):
    import aps2026_b200.ops as ops

    return ops


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    so = tmp_path_factory.mktemp("fusion") / "libfusion_harness.so"
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-Xcompiler", "-fPIC", "-shared", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "fusion_harness.cu"),
                    "-o", str(so)], check=True, capture_output=True)
    lib = C.CDLL(str(so))
    vp, sz = C.c_void_p, C.c_size_t
    lib.harness_gemm.argtypes = [vp, vp, vp, sz, sz, sz, sz] + [vp] * 7 + [C.c_int, C.c_int, vp]
    lib.harness_prologue.argtypes = [vp] * 6 + [sz, sz, vp]
    return lib


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _gemm(h, a, b, n, head_dim=128, stats=None, ln=None, rope=None):
    import torch

    m, k = a.shape
    c = torch.empty((m, n), device=a.device)
    mean, inv = stats if stats else (None, None)
    gamma, beta = ln if ln else (None, None)
    cos, sin, pos = rope if rope else (None, None, None)
    rc = h.harness_gemm(_p(a), _p(b), _p(c), m, n, k, head_dim, _p(mean), _p(inv), _p(gamma), _p(beta), _p(cos),
                        _p(sin), _p(pos), int(stats is not None), int(rope is not None), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    return c


def test_rope_epilogue_matches_b2_rope(harness, ops, cuda):
    g = rng(61)
    M, K, max_seq = 300, 96, 700
    a = to_dev(normal(g, (M, K)), cuda)
    bq, bk = to_dev(normal(g, (4 * 128, K)), cuda), to_dev(normal(g, (128, K)), cuda)
    pos = to_dev(g.integers(0, max_seq, M).astype(np.int32), cuda)
    cos, sin = ops.rope_table_gpu(max_seq, 128, ops.ROPE_THETA, cuda)
    q, k = _gemm(harness, a, bq, 4 * 128), _gemm(harness, a, bk, 128)
    ops.apply_rope_tree_gpu(q, k, pos, M, max_seq, 4, 1, 128, ops.ROPE_THETA)
    qf = _gemm(harness, a, bq, 4 * 128, rope=(cos, sin, pos))
    kf = _gemm(harness, a, bk, 128, rope=(cos, sin, pos))
    oracle.assert_bitexact(to_host(qf), to_host(q), "q: GEMM + RoPE epilogue vs GEMM then b2_rope")
    oracle.assert_bitexact(to_host(kf), to_host(k), "k: GEMM + RoPE epilogue vs GEMM then b2_rope")


@pytest.mark.parametrize("exact", [True, False])
def test_layer_norm_prologue_matches_b2_layer_norm(harness, ops, cuda, exact):
    import torch

    g = rng(62)
    M, K = 200, 1024
    x = to_dev(normal(g, (M, K)), cuda)
    gamma, beta = to_dev(normal(g, K, 1.0, 0.1), cuda), to_dev(normal(g, K, 0.0, 0.1), cuda)
    b = to_dev(normal(g, (256, K)), cuda)
    y = torch.empty_like(x)
    ops.layer_norm_gpu(x, gamma, beta, ops.NORM_EPS, y, exact=exact)
    want = _gemm(harness, y, b, 256)
    stats = ops.layer_norm_stats_gpu(x, ops.NORM_EPS, exact=exact)
    got = _gemm(harness, x, b, 256, stats=stats, ln=(gamma, beta))
    if exact:
        oracle.assert_bitexact(to_host(got), to_host(want), "GEMM with LN prologue vs GEMM on b2_layer_norm")
    else:
        # a dot product of 1024 terms amplifies a last-ulp difference of the
        # statistics; compare the operands themselves, then the products loosely
        out = torch.empty_like(x)
        assert harness.harness_prologue(_p(x), _p(stats[0]), _p(stats[1]), _p(gamma), _p(beta), _p(out), M, K,
                                        _stream()) == 0
        torch.cuda.synchronize()
        oracle.assert_close(to_host(out), to_host(y), what="LN prologue operand vs b2_layer_norm (tree order)")
        np.testing.assert_allclose(to_host(got), to_host(want), rtol=1e-4, atol=1e-4)


def test_layer_norm_prologue_at_pipeline_size(harness, ops, cuda):
    import torch

    g = rng(63)
    M, K = 9473, 4096  # b2_layer_norm (reference order) runs its chain pipeline at this size
    xh = normal(g, (M, K))
    wh, bh = normal(g, K, 1.0, 0.1), normal(g, K, 0.0, 0.1)
    x, gamma, beta = to_dev(xh, cuda), to_dev(wh, cuda), to_dev(bh, cuda)
    y = torch.empty_like(x)
    ops.layer_norm_gpu(x, gamma, beta, ops.NORM_EPS, y, exact=True)
    mean, inv = ops.layer_norm_stats_gpu(x, ops.NORM_EPS, exact=True)
    out = torch.empty_like(x)
    assert harness.harness_prologue(_p(x), _p(mean), _p(inv), _p(gamma), _p(beta), _p(out), M, K, _stream()) == 0
    torch.cuda.synchronize()
    oracle.assert_bitexact(to_host(out), to_host(y), "LN prologue vs b2_layer_norm at 9473 x 4096")
    oracle.assert_bitexact(to_host(y), oracle.layer_norm(xh, wh, bh, 1e-5), "b2_layer_norm vs oracle")


def test_layer_norm_stats_arguments(ops, cuda):
    import torch

    from aps2026_b200 import _lib

    lib = _lib.lib()
    x = torch.zeros((2, 8), device=cuda)
    m = torch.empty(2, device=cuda)
    assert lib.b2_layer_norm_stats(x.data_ptr(), 2, 8, 1e-5, 1, None, m.data_ptr(), None) == \
        _lib.B2_ERR_INVALID_ARGUMENT
    assert lib.b2_layer_norm_stats(x.data_ptr(), 2, 0, 1e-5, 1, m.data_ptr(), m.data_ptr(), None) == \
        _lib.B2_ERR_INVALID_ARGUMENT
    assert lib.b2_layer_norm_stats(x.data_ptr(), 0, 8, 1e-5, 1, None, None, None) == _lib.B2_OK
