"""The C-ABI library loads without a GPU, exports every symbol the header
declares, and its host entry points (no device work) behave as specified."""
import ctypes as C
import subprocess

import numpy as np
import pytest

import oracle
from aps2026_b200 import _lib


def test_library_exports_every_declared_symbol():
    declared = _lib.declared_functions()
    assert len(declared) >= 16
    handle = _lib.lib()
    for name in declared:
        assert hasattr(handle, name), f"{name} declared in include/aps2026_b200.h but not exported"
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                        check=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    assert set(declared) <= exported


@pytest.mark.parametrize("cmd", [["gcc", "-std=c99", "-x", "c"], ["g++", "-std=c++17", "-x", "c++"]])
def test_header_is_plain_c_and_cpp(cmd):
    """The ABI header compiles warning-free as C99 (what a cgo / ctypes /
    N-API binding includes) and as C++."""
    from pathlib import Path

    header = Path(__file__).resolve().parents[1] / "include" / "aps2026_b200.h"
    r = subprocess.run(cmd + ["-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only", str(header)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_binding_table_covers_header():
    assert set(_lib.declared_functions()) == set(_lib.SIGNATURES)


def test_version():
    assert _lib.lib().b2_version().decode().startswith("aps2026_b200")


def test_null_pointer_arguments_are_rejected_before_any_device_work():
    lib = _lib.lib()
    assert lib.b2_layer_norm(None, None, None, None, 4, 16, 1e-5, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert "null" in _lib.last_error()
    assert lib.b2_gather_rows(None, 1, 4, None, 3, None, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert lib.b2_moe_route(None, 8, 33, 1e-3, 2e-2, *([None] * 10), 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert "E must be" in _lib.last_error()
    assert lib.b2_causal_softmax(None, None, 1, 8, 4, 1.0, 8, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    # zero-sized work is a no-op that succeeds (the reference's empty RowIndexBuffer path)
    assert lib.b2_gather_rows(None, 0, 4, None, 0, None, None) == _lib.B2_OK
    assert lib.b2_layer_norm(None, None, None, None, 0, 16, 1e-5, 0, None) == _lib.B2_OK


def test_route_workspace_size():
    n = C.c_size_t(0)
    assert _lib.lib().b2_moe_route_workspace_size(8192, 16, C.addressof(n)) == 0
    assert n.value == 32 * 16 * 4
    assert _lib.lib().b2_moe_route_workspace_size(1000, 13, C.addressof(n)) == 0
    assert n.value == 4 * 16 * 4  # experts padded to a power of two


@pytest.mark.parametrize("max_seq,head_dim,theta", [(4096, 128, 10000.0), (17, 64, 500000.0), (3, 2, 10.0)])
def test_rope_table_bitexact_vs_oracle(max_seq, head_dim, theta):
    from aps2026_b200 import ops

    c, s = ops.rope_table_host(max_seq, head_dim, theta)
    oc, os_ = oracle.rope_table(max_seq, head_dim, theta)
    oracle.assert_bitexact(c.numpy(), oc, "cos")
    oracle.assert_bitexact(s.numpy(), os_, "sin")


def test_rope_table_rejects_odd_head_dim():
    buf = np.empty(16, np.float32)
    assert _lib.lib().b2_rope_table(2, 3, 1e4, buf.ctypes.data, buf.ctypes.data) == _lib.B2_ERR_INVALID_ARGUMENT
