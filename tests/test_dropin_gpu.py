"""The drop-in claim end to end: the reference's own model code
(src/model.cu, src/layer.cu, compiled unchanged) gives the same logits with
its own tensor_ops and with the C++ shim over libaps2026_b200.so in their
place (oracle/dropin_harness.cu, oracle/Makefile).

Weights are a seeded synthetic model.bin in the reference's loader format
(tests/_dropin.py; the course's model.bin and inputs are not available), so
this checks parity with the reference, not the course's answers.bin.
PhiTinyMoEModel::generate exercises the trie path (gather_rows_gpu,
layer_norm_gpu / add_layer_norm_gpu, apply_rope_tree_gpu,
attention_tree_gpu); forward(use_gpu = true) the packed path
(apply_rope_gpu, attention_gpu, add_inplace_gpu). Both run every layer's
MoE through moe_forward_grouped_gpu, whose routing (b2_moe_route) and
un-permute (b2_moe_combine) the b2 library takes over through the hooks of
aps2026_b200/shim/apply_moe_hook.py; the GEMMs are the reference's in both
libraries. Routing after every LayerNorm makes this a sharp test: a
last-ulp difference in one LayerNorm output, or one differently ordered
assignment row, flips an expert choice or a GEMM row and changes the
logits.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
LIBS = {k: ROOT / "oracle" / "_ref" / f"libdropin_{k}.so" for k in ("ref", "b2")}


def _mem_available_gb() -> float:
    for line in Path("/proc/meminfo").read_text().splitlines():
        if line.startswith("MemAvailable:"):
            return int(line.split()[1]) / 2**20
    return 0.0


@pytest.fixture(scope="module")
def runs(tmp_path_factory):
    if not all(p.exists() for p in LIBS.values()):
        pytest.skip("drop-in libraries not built (oracle/Makefile needs the reference tree)")
    # each process holds the 32 layers' weights on the host and the device (~15 GB each)
    if _mem_available_gb() < 48:
        pytest.skip("needs 48 GB of free host memory")
    sys.path.insert(0, str(ROOT / "tests"))
    import _dropin

    d = tmp_path_factory.mktemp("dropin")
    model = d / "model.bin"
    _dropin.write_model(model, seed=0)
    out = {}
    # One OpenMP thread: forward(use_gpu = true) ends in the reference's host
    # layer_norm (src/model.cu:33, src/tensor.cu:327-341), whose OpenMP
    # threads all call Tensor::ensure_host (src/tensor.cu:91-101) on the
    # device-only hidden state and output at once; with several threads
    # that races on the host buffer's allocation (heap corruption and
    # nondeterministic logits, seen here with the reference's own ops).
    env = dict(os.environ, OMP_NUM_THREADS="1")
    for k, lib in LIBS.items():
        npz = d / f"{k}.npz"
        subprocess.run([sys.executable, str(ROOT / "tests" / "_dropin.py"), str(lib), str(model), str(npz)],
                       check=True, timeout=900, env=env)
        out[k] = dict(np.load(npz))
    model.unlink()
    print("\ndrop-in generate ms (3 calls): ref", out["ref"]["generate_ms"], "b2", out["b2"]["generate_ms"],
          "| forward ms: ref", out["ref"]["forward_ms"], "b2", out["b2"]["forward_ms"])
    return out


def test_generate_logits_identical(runs):
    ref, b2 = runs["ref"]["generate"], runs["b2"]["generate"]
    assert np.isfinite(ref).all()
    assert ref.std() > 0.1  # the synthetic model is not degenerate
    assert np.array_equal(ref.view(np.uint32), b2.view(np.uint32)), \
        f"{int((ref != b2).sum())} of {ref.size} logits differ"


def test_forward_logits_identical(runs):
    ref, b2 = runs["ref"]["forward"], runs["b2"]["forward"]
    assert np.isfinite(ref).all()
    assert np.array_equal(ref.view(np.uint32), b2.view(np.uint32)), \
        f"{int((ref != b2).sum())} of {ref.size} logits differ"


@pytest.mark.parametrize("name", ["rope_q", "rope_k", "attention", "add"])
def test_packed_ops_identical(runs, name):
    """apply_rope_gpu, attention_gpu (three packed segments) and
    add_inplace_gpu called through the reference's Tensor class."""
    ref, b2 = runs["ref"][name], runs["b2"][name]
    assert np.isfinite(ref).all()
    assert np.array_equal(ref.view(np.uint32), b2.view(np.uint32)), \
        f"{name}: {int((ref != b2).sum())} of {ref.size} differ, max |diff| {np.abs(ref - b2).max()}"


def test_generate_is_repeatable(runs):
    # three generate calls on one model object return the same logits (the
    # shim's cached tables and staging buffers are reused correctly)
    assert bool(runs["b2"]["repeatable"][0]) and bool(runs["ref"]["repeatable"][0])


def test_error_behaviour_identical(runs):
    ref, b2 = list(runs["ref"]["errors"]), list(runs["b2"]["errors"])
    assert ref == b2
    assert ref[0].startswith("1:") and "empty input" in ref[0]
    assert ref[1].startswith("1:") and "vocabulary" in ref[1]
