"""The reference-side C++ binding (aps2026_b200/shim/tensor_ops_b2.cu)
compiles against the reference's own include/tensor.h and config.h and
defines exactly the tensor_ops functions it replaces, with the reference's
signatures (checked through the mangled symbol names); the MoE hook edit
(aps2026_b200/shim/apply_moe_hook.py) replaces exactly the routing and
un-permute launches of moe_forward_grouped_gpu."""
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_INCLUDE = Path("/root/reference/include")
REF_TENSOR = Path("/root/reference/src/tensor.cu")
HOOKS = {
    "b2_dropin::moe_route(float const*, unsigned long, unsigned char*, unsigned int*, unsigned int*, unsigned int*, "
    "unsigned int*, unsigned int*, unsigned int*, unsigned int*, unsigned int*)",
    "b2_dropin::moe_combine(float const*, unsigned long, unsigned char const*, unsigned int const*, float*, "
    "unsigned long, unsigned long)",
}

EXPECTED = {
    "tensor_ops::add_inplace_gpu(Tensor&, Tensor const&)",
    "tensor_ops::silu_mul_gpu(Tensor const&, Tensor const&, Tensor&)",
    "tensor_ops::layer_norm_gpu(Tensor const&, Tensor const&, Tensor const&, float, Tensor&)",
    "tensor_ops::add_layer_norm_gpu(Tensor&, Tensor const&, Tensor const&, Tensor const&, float, Tensor&)",
    "tensor_ops::apply_rope_gpu(Tensor&, Tensor&, std::vector<unsigned long, std::allocator<unsigned long> > const&, "
    "unsigned long, unsigned long, unsigned long, float)",
    "tensor_ops::apply_rope_tree_gpu(Tensor&, Tensor&, unsigned int const*, unsigned long, unsigned long, "
    "unsigned long, unsigned long, unsigned long, float)",
    "tensor_ops::gather_rows_gpu(Tensor const&, std::vector<unsigned long, std::allocator<unsigned long> > const&, "
    "Tensor&)",
    "tensor_ops::gather_rows_gpu(Tensor const&, tensor_ops::RowIndexBuffer const&, Tensor&)",
    "tensor_ops::attention_gpu(Tensor const&, Tensor const&, Tensor const&, Tensor&, "
    "std::vector<unsigned long, std::allocator<unsigned long> > const&, unsigned long, unsigned long, unsigned long)",
    "tensor_ops::attention_tree_gpu(Tensor const&, Tensor const&, Tensor const&, Tensor&, unsigned int const*, "
    "unsigned int const*, unsigned long, unsigned long, unsigned long, unsigned long, unsigned long, unsigned long)",
}


@pytest.mark.skipif(not (REF_INCLUDE / "tensor.h").exists(), reason="reference headers not present")
def test_shim_compiles_against_reference_headers(tmp_path):
    obj = tmp_path / "shim.o"
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-c",
                    str(ROOT / "aps2026_b200/shim/tensor_ops_b2.cu"), f"-I{REF_INCLUDE}", f"-I{ROOT / 'include'}",
                    "-o", str(obj)], check=True, capture_output=True)
    nm = subprocess.run(["nm", "-C", "--defined-only", str(obj)], capture_output=True, text=True, check=True).stdout
    defined = {line.split(" T ", 1)[1] for line in nm.splitlines() if " T tensor_ops::" in line
               and "(anonymous namespace)" not in line}
    assert defined == EXPECTED
    hooks = {line.split(" T ", 1)[1] for line in nm.splitlines() if " T b2_dropin::" in line}
    assert hooks == HOOKS


def _moe_body(src: str) -> str:
    m = re.search(r"void\s+moe_forward_grouped_gpu\s*\([^;{]*\)\s*\{", src)
    depth, i = 0, m.end() - 1
    while True:
        depth += {"{": 1, "}": -1}.get(src[i], 0)
        i += 1
        if depth == 0:
            return src[m.end():i]


@pytest.mark.skipif(not REF_TENSOR.exists(), reason="reference source not present")
def test_moe_hook_edit_replaces_routing_and_combine_only():
    sys.path.insert(0, str(ROOT / "aps2026_b200" / "shim"))
    import apply_moe_hook

    src = REF_TENSOR.read_text()
    out = apply_moe_hook.patch(src)
    before, after = _moe_body(src), _moe_body(out)
    launches = lambda body: re.findall(r"(\w+)\s*<<<", body)  # noqa: E731
    gone = {"k_moe_top2", "k_moe_offsets_work", "k_moe_fill_stable", "k_moe_combine"}
    assert gone <= set(launches(before))
    assert not gone & set(launches(after))
    # every other launch of the function (the expert GEMMs) is untouched
    assert [k for k in launches(before) if k not in gone] == launches(after)
    assert after.count("b2_dropin::moe_route(") == 1 and after.count("b2_dropin::moe_combine(") == 1
    assert "cudaMemsetAsync" not in after
    # outside the function nothing changes but the hook header include
    assert out.replace(after, before, 1) == '#include "moe_hook.h"\n' + src


DROPIN_B2 = ROOT / "oracle" / "_ref" / "libdropin_b2.so"


@pytest.mark.skipif(not DROPIN_B2.exists(), reason="drop-in library not built (needs the reference tree)")
def test_dropin_library_takes_the_shim_functions():
    """oracle/_ref/libdropin_b2.so (the reference model code with the shim in
    place of the replaced tensor_ops functions): each replaced function is
    defined once under its own name (the shim's) and once renamed out of the
    reference's tensor.cu, and the shim's calls go to libaps2026_b200.so."""
    nm = subprocess.run(["nm", "-C", "--defined-only", str(DROPIN_B2)], capture_output=True, text=True,
                        check=True).stdout
    defined = {line.split(" T ", 1)[1] for line in nm.splitlines() if " T tensor_ops::" in line}
    for sig in EXPECTED:
        assert sig in defined
        assert sig.replace("tensor_ops::", "tensor_ops::ref_replaced_", 1) in defined
    undefined = subprocess.run(["nm", "-u", str(DROPIN_B2)], capture_output=True, text=True, check=True).stdout
    for sym in ("b2_layer_norm", "b2_attention_tree_compact", "b2_moe_route", "b2_moe_combine"):
        assert sym in undefined
    needed = subprocess.run(["readelf", "-d", str(DROPIN_B2)], capture_output=True, text=True, check=True).stdout
    assert "libaps2026_b200.so" in needed
