"""ctypes binding of libaps2026_b200.so (the C ABI in include/aps2026_b200.h).

Loading fails loudly when the shared library has not been built: there is no
CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libaps2026_b200.so"
HEADER = HERE.parent / "include" / "aps2026_b200.h"

B2_OK = 0
B2_ERR_INVALID_ARGUMENT = 1
B2_ERR_CUDA = 2
B2_ERR_DEVICE_CHECK = 3
B2_ERR_TIMEOUT = 4
B2_ERR_UNSUPPORTED = 5
B2_ERR_IO = 6
B2_FLAG_EXACT_ORDER = 1

B2_CHECK_GATHER = 1
B2_CHECK_ROPE = 2
B2_CHECK_COMBINE = 4
B2_CHECK_ATTENTION = 8

_vp, _sz, _f32, _u32 = C.c_void_p, C.c_size_t, C.c_float, C.c_uint32

# name -> (restype, argtypes); every pointer is passed as a void* address.
SIGNATURES: dict[str, tuple] = {
    "b2_version": (C.c_char_p, []),
    "b2_last_error": (C.c_char_p, []),
    "b2_device_status": (C.c_int, [_vp, _vp]),
    "b2_gather_rows": (C.c_int, [_vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    "b2_moe_gather_compact": (C.c_int, [_vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    "b2_prefix_trie_device_workspace_size": (C.c_int, [_sz, _vp]),
    "b2_prefix_trie_device": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "b2_layer_norm": (C.c_int, [_vp, _vp, _vp, _vp, _sz, _sz, _f32, _u32, _vp]),
    "b2_add_layer_norm": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _f32, _u32, _vp]),
    "b2_layer_norm_stats": (C.c_int, [_vp, _sz, _sz, _f32, _u32, _vp, _vp, _vp]),
    "b2_moe_combine_add_layer_norm": (
        C.c_int, [_vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _f32, _u32, _vp]),
    "b2_rope_table": (C.c_int, [_sz, _sz, _f32, _vp, _vp]),
    "b2_rope": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _sz, _vp]),
    "b2_causal_softmax": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _f32, _sz, _u32, _vp]),
    "b2_attention_tree": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _u32, _vp]),
    "b2_attention_tree_compact": (C.c_int, [_vp] * 7 + [_sz, _vp] + [_sz] * 7 + [_u32, _vp]),
    "b2_moe_route_workspace_size": (C.c_int, [_sz, _sz, _vp]),
    "b2_moe_route": (C.c_int, [_vp, _sz, _sz, _f32, _f32] + [_vp] * 10 + [_sz, _vp]),
    "b2_moe_route_noalloc": (C.c_int, [_vp, _sz, _sz, _f32, _f32] + [_vp] * 9 + [_vp]),
    "b2_silu_mul": (C.c_int, [_vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _vp]),
    "b2_silu_mul_flags": (C.c_int, [_vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _u32, _vp]),
    "b2_moe_combine": (C.c_int, [_vp, _sz, _vp, _vp, _vp, _sz, _sz, _vp]),
    "b2_add": (C.c_int, [_vp, _vp, _sz, _vp]),
    "b2_prefix_trie_build": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _sz, _vp]),
    "b2_read_inputs": (C.c_int, [C.c_char_p, _sz, _vp, _vp, _vp, _vp, _sz, _vp, _sz]),
    "b2_write_outputs": (C.c_int, [C.c_char_p, _vp, _sz, _sz, C.c_int, _vp]),
    "b2_selfcheck_exp": (C.c_int, [_u32, _u32, _vp, _vp, _vp]),
    "b2_selfcheck_wait": (C.c_int, [C.c_uint64]),
    # struct arguments (b2_prefill_shape / _layer / _work) are passed by address
    "b2_prefill_layers": (C.c_int, [_vp, _vp, _sz, _vp, _vp, _vp, _vp, _sz, _vp, _sz, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp]),
}


def declared_functions(header: Path = HEADER) -> list[str]:
    """Names of the functions include/aps2026_b200.h declares."""
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library with argument types set; raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m aps2026_b200.build` "
                "(there is no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().b2_last_error().decode()
