"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU oracle and of the
reference-built checker library.

- ``liboracle.so`` (oracle/oracle.cpp): CPU restatement of the reference
  kernels' arithmetic; every function cites the reference file:line it
  follows.
- ``_ref/libref.so`` (oracle/ref_harness.cu): the reference's own
  src/tensor.cu compiled from where it lies; its kernels run on a GPU, its
  host ops anywhere.
- ``_ref/libio_ref.so`` (oracle/io_harness.cu): the reference harness's own
  prompt-file reader and output-file writer (src/main.cpp:144-192); host
  only.
- ``outputs_bytes`` / ``parse_inputs`` below: numpy restatements of those two
  file formats.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm may use this package. The aps2026_b200 package never imports it.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref.so"
IO_REF_SO = HERE / "_ref" / "libio_ref.so"

_vp, _sz, _f32, _i = C.c_void_p, C.c_size_t, C.c_float, C.c_int


def build() -> None:
    """Builds liboracle.so and, when the reference tree exists, _ref/libref.so."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_orc = None
_ref = None


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def lib() -> C.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            build()
        h = C.CDLL(str(ORACLE_SO))
        sig = {
            "orc_num_threads": (_i, []),
            "orc_set_num_threads": (None, [_i]),
            "orc_gather_rows": (None, [_vp, _sz, _vp, _sz, _vp]),
            "orc_layer_norm": (None, [_vp, _vp, _vp, _vp, _sz, _sz, _f32]),
            "orc_add_layer_norm": (None, [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _f32]),
            "orc_rope_table": (None, [_sz, _sz, _f32, _vp, _vp]),
            "orc_rope": (None, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp]),
            "orc_causal_softmax": (None, [_vp, _vp, _sz, _sz, _sz, _f32, _sz]),
            "orc_moe_route": (None, [_vp, _sz, _sz, _f32, _f32] + [_vp] * 9),
            "orc_silu_mul": (None, [_vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz]),
            "orc_moe_combine": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
            "orc_moe_combine_add_layer_norm": (None, [_vp] * 8 + [_sz, _sz, _f32]),
            "orc_add": (None, [_vp, _vp, _sz]),
            "orc_prefix_trie": (C.c_longlong, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, _sz]),
            "orc_attention_tree": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(h, name)
            fn.restype, fn.argtypes = res, args
        _orc = h
    return _orc


def ref_available() -> bool:
    return REF_SO.exists()


def ref() -> C.CDLL:
    """The reference-built checker; raises if it was never built."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference tree)")
        h = C.CDLL(str(REF_SO))
        sig = {
            "ref_k_gather_rows": [_vp, _vp, _vp, _sz, _sz, _vp],
            "ref_k_layer_norm": [_vp, _vp, _vp, _vp, _sz, _sz, _f32, _vp],
            "ref_k_add_layer_norm": [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _f32, _vp],
            "ref_k_rope": [_vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _vp],
            "ref_k_moe_route": [_vp, _sz] + [_vp] * 10,
            "ref_k_silu_mul": [_vp, _vp, _vp, _sz, _vp],
            "ref_k_moe_combine": [_vp, _vp, _vp, _vp, _sz, _sz, _vp],
            "ref_k_add": [_vp, _vp, _sz, _vp],
            "ref_k_moe_gather_compact": [_vp, _vp, _vp, _sz, _sz, _vp],
            "ref_k_attention_tree": [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp],
            "ref_k_attention_grouped": [_vp] * 6 + [_sz] * 5 + [_vp],
            "ref_sliding_window": [],
            "ref_cpu_layer_norm": [_vp, _vp, _vp, _vp, _sz, _sz, _f32, _vp],
            "ref_cpu_apply_rope": [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _f32, _vp],
            "ref_cpu_silu_mul": [_vp, _vp, _vp, _sz, _vp],
            "ref_cpu_add_inplace": [_vp, _vp, _sz, _vp],
        }
        for name, args in sig.items():
            fn = getattr(h, name)
            fn.restype, fn.argtypes = _i, args
        _ref = h
    return _ref


_io_ref = None


def io_ref_available() -> bool:
    return IO_REF_SO.exists()


def io_ref() -> C.CDLL:
    """The reference's own read_inputs / write_outputs (src/main.cpp:144-192)
    behind io_harness.cu; raises if it was never built."""
    global _io_ref
    if _io_ref is None:
        if not IO_REF_SO.exists():
            raise FileNotFoundError(f"{IO_REF_SO} not built (needs the reference tree)")
        h = C.CDLL(str(IO_REF_SO))
        h.io_ref_error.restype, h.io_ref_error.argtypes = C.c_char_p, []
        h.io_ref_write_outputs.restype = _i
        h.io_ref_write_outputs.argtypes = [C.c_char_p, _vp, _sz, _sz]
        h.io_ref_read_inputs.restype = _i
        h.io_ref_read_inputs.argtypes = [C.c_char_p, _vp, _vp, _vp, _vp, _sz, _vp, _sz]
        _io_ref = h
    return _io_ref


def outputs_bytes(logits) -> bytes:
    """The output file write_outputs (src/main.cpp:183-192) makes of a
    [batch, vocab] fp32 matrix: uint32 batch, uint32 vocab, the floats
    row-major, all little-endian."""
    a = np.ascontiguousarray(logits, dtype="<f4")
    return np.array(a.shape, dtype="<u4").tobytes() + a.tobytes()


def inputs_bytes(prompts, max_seq_len=None) -> bytes:
    """The prompt file read_inputs (src/main.cpp:144-181) reads: uint32 batch,
    uint32 max_seq_len, then per prompt uint32 length and int32 ids."""
    m = max(len(p) for p in prompts) if max_seq_len is None else max_seq_len
    out = [np.array([len(prompts), m], dtype="<u4").tobytes()]
    for p in prompts:
        out.append(np.array([len(p)], dtype="<u4").tobytes() + np.asarray(p, dtype="<i4").tobytes())
    return b"".join(out)


def parse_inputs(data: bytes, max_len: int = 4096):
    """read_inputs (src/main.cpp:152-181) restated over the file's bytes:
    returns (prompts as lists, max_seq_len), or raises RuntimeError with the
    reference's message, its checks taken in its order."""
    if len(data) < 8:
        raise RuntimeError("invalid input header")
    batch, max_seq = np.frombuffer(data[:8], dtype="<u4").tolist()
    if batch == 0 or max_seq == 0 or max_seq > max_len:
        raise RuntimeError("invalid input header")
    pos, prompts = 8, []
    for _ in range(batch):
        if len(data) - pos < 4:
            raise RuntimeError("invalid sequence length in input")
        n = int(np.frombuffer(data[pos:pos + 4], dtype="<u4")[0])
        pos += 4
        if n == 0 or n > max_seq:
            raise RuntimeError("invalid sequence length in input")
        if len(data) - pos < 4 * n:
            raise RuntimeError("truncated input")
        prompts.append(np.frombuffer(data[pos:pos + 4 * n], dtype="<i4").tolist())
        pos += 4 * n
    return prompts, max_seq


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


# ---- oracle ops (numpy in, numpy out) ------------------------------------------


def gather_rows(x, rows):
    x, rows = f32(x), u32(rows)
    h = x.shape[-1]
    out = np.empty((rows.size, h), np.float32)
    lib().orc_gather_rows(_p(x), h, _p(rows), rows.size, _p(out))
    return out


def layer_norm(x, w, b, eps=1e-5):
    x, w, b = f32(x), f32(w), f32(b)
    h = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_layer_norm(_p(x), _p(w), _p(b), _p(y), x.size // h, h, eps)
    return y


def add_layer_norm(x, res, w, b, eps=1e-5):
    """Returns (x + res, LayerNorm(x + res))."""
    x, res, w, b = f32(x).copy(), f32(res), f32(w), f32(b)
    h = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_add_layer_norm(_p(x), _p(res), _p(w), _p(b), _p(y), x.size // h, h, eps)
    return x, y


def rope_table(max_seq, head_dim, theta=10000.0):
    half = head_dim // 2
    c = np.empty((max_seq, half), np.float32)
    s = np.empty((max_seq, half), np.float32)
    lib().orc_rope_table(max_seq, head_dim, theta, _p(c), _p(s))
    return c, s


def rope(q, k, row_pos, q_heads, kv_heads, head_dim, cos, sin):
    """Returns rotated copies of q and k."""
    q, k, row_pos, cos, sin = f32(q).copy(), f32(k).copy(), u32(row_pos), f32(cos), f32(sin)
    lib().orc_rope(_p(q), _p(k), _p(row_pos), row_pos.size, q_heads, kv_heads, head_dim, _p(cos), _p(sin))
    return q, k


def causal_softmax(scores, scale, window):
    scores = f32(scores)
    heads, T, ld = scores.shape
    probs = np.zeros_like(scores)
    lib().orc_causal_softmax(_p(scores), _p(probs), heads, T, ld, scale, window)
    return probs


def moe_route(logits, quantum=1e-3, tie_eps=2e-2):
    """Returns a dict with the reference routing outputs."""
    logits = f32(logits)
    T, E = logits.shape
    n64, n128 = (2 * T + 63) // 64 + E, (2 * T + 127) // 128 + E
    out = dict(routes=np.empty((T, 2), np.uint8), counts=np.empty(E, np.uint32),
               offsets=np.empty(E + 1, np.uint32), assignment_rows=np.empty(2 * T, np.uint32),
               route_positions=np.empty(2 * T, np.uint32), work_expert64=np.empty(n64, np.uint32),
               work_start64=np.empty(n64, np.uint32), work_expert128=np.empty(n128, np.uint32),
               work_start128=np.empty(n128, np.uint32))
    lib().orc_moe_route(_p(logits), T, E, quantum, tie_eps, *[_p(out[k]) for k in (
        "routes", "counts", "offsets", "assignment_rows", "route_positions", "work_expert64",
        "work_start64", "work_expert128", "work_start128")])
    return out


def attention_tree(q, k, v, row_pos, anc, q_heads, kv_heads, head_dim, window):
    """Prefix-tree GQA attention of k_attention_tree_gqa4; anc is
    [rows, anc_stride]."""
    q, k, v, row_pos, anc = f32(q), f32(k), f32(v), u32(row_pos), u32(anc)
    rows = row_pos.size
    out = np.empty((rows, q_heads * head_dim), np.float32)
    lib().orc_attention_tree(_p(q), _p(k), _p(v), _p(out), _p(row_pos), _p(anc), anc.shape[1], rows, q_heads,
                             kv_heads, head_dim, window)
    return out


def silu_mul(gate, up):
    gate, up = f32(gate), f32(up)
    rows, cols = gate.shape
    out = np.empty_like(gate)
    lib().orc_silu_mul(_p(gate), cols, _p(up), cols, _p(out), cols, rows, cols)
    return out


def moe_combine(expert_out, routes, route_positions, T):
    expert_out, routes, rp = f32(expert_out), np.ascontiguousarray(routes, np.uint8), u32(route_positions)
    h = expert_out.shape[-1]
    out = np.empty((T, h), np.float32)
    lib().orc_moe_combine(_p(expert_out), _p(routes), _p(rp), _p(out), T, h)
    return out


def moe_combine_add_layer_norm(expert_out, routes, route_positions, carry, w, b, eps=1e-5):
    """Returns (x_out, y)."""
    expert_out, carry, w, b = f32(expert_out), f32(carry), f32(w), f32(b)
    routes, rp = np.ascontiguousarray(routes, np.uint8), u32(route_positions)
    T, h = carry.shape
    x_out = np.empty_like(carry)
    y = np.empty_like(carry)
    lib().orc_moe_combine_add_layer_norm(_p(expert_out), _p(routes), _p(rp), _p(carry), _p(w), _p(b),
                                         _p(x_out), _p(y), T, h, eps)
    return x_out, y


def add(a, b):
    a, b = f32(a).copy(), f32(b)
    lib().orc_add(_p(a), _p(b), a.size)
    return a


def prefix_trie(prompts, vocab=32064, with_ancestors=True):
    lens = u32([len(p) for p in prompts])
    ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]), np.int32)
    total, stride = int(lens.sum()), int(lens.max())
    token_node = np.empty(total, np.uint32)
    node_token = np.empty(total, np.uint32)
    node_depth = np.empty(total, np.uint32)
    anc = np.empty(total * stride, np.uint32) if with_ancestors else None
    n = lib().orc_prefix_trie(_p(ids), _p(lens), len(prompts), vocab, _p(token_node), _p(node_token),
                              _p(node_depth), _p(anc), stride)
    if n < 0:
        raise ValueError("token out of vocabulary")
    return dict(token_node=token_node, node_token=node_token[:n], node_depth=node_depth[:n],
                node_anc=anc[: n * stride].reshape(n, stride) if anc is not None else None, nodes=n)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(n)


# ---- comparisons ----------------------------------------------------------------------

ATOL = 1e-6
RTOL = 1e-5


def close_mask(got, want, atol=ATOL, rtol=RTOL):
    """Elementwise pass mask of the north_star tolerance: |d| <= atol OR
    |d| / |want| <= rtol (the OR form of the reference's validation,
    src/main.cpp:341-343); NaN fails."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = np.abs(got - want)
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = d / np.abs(want)
    ok = (d <= atol) | (rel <= rtol)
    return ok & ~np.isnan(got) & ~np.isnan(want)


def assert_close(got, want, atol=ATOL, rtol=RTOL, what=""):
    ok = close_mask(got, want, atol, rtol)
    if not ok.all():
        bad = np.flatnonzero(~ok.ravel())
        i = bad[0]
        g, w = np.asarray(got).ravel()[i], np.asarray(want).ravel()[i]
        raise AssertionError(f"{what}: {bad.size} / {ok.size} elements outside tolerance; "
                             f"first at {i}: got {g!r} want {w!r}")


def assert_bitexact(got, want, what=""):
    got, want = np.ascontiguousarray(got), np.ascontiguousarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    gb, wb = got.view(np.uint8), want.view(np.uint8)
    if not np.array_equal(gb, wb):
        diff = np.flatnonzero(got.ravel().view(np.uint8 if got.dtype.itemsize == 1 else f"u{got.dtype.itemsize}")
                              != want.ravel().view(np.uint8 if want.dtype.itemsize == 1 else f"u{want.dtype.itemsize}"))
        i = diff[0]
        raise AssertionError(f"{what}: {diff.size} elements differ; first at {i}: "
                             f"got {got.ravel()[i]!r} want {want.ravel()[i]!r}")


# ---- layer pipeline ------------------------------------------------------------------------


def prefill_layers(emb, node_token, node_depth, standins, ln1, ln2, final, layers, q_heads=16, kv_heads=4,
                   head_dim=128, inter=448, eps=1e-5, theta=10000.0):
    """The non-GEMM layer loop of PhiDecoderLayer::forward_carry
    (src/layer.cu:273-300) and the final add + LayerNorm of
    PhiTinyMoEModel::generate (src/model.cu:119-150) with the oracle ops, in
    the reference's unfused order (k_moe_combine into x, then
    k_add_layer_norm with the carry). `standins` is a list of dicts of host
    arrays (q, k, attn, logits, gate_up, expert_out), layer l using
    standins[l % len]; q, k and attn are updated in place as on the GPU.
    Returns (final_x, final_out)."""
    node_depth = u32(node_depth)
    x = gather_rows(emb, node_token)
    rows, h = x.shape
    cos, sin = rope_table(int(node_depth.max()) + 1, head_dim, theta)
    carry = None
    routing = None
    prev = None
    for l in range(layers):
        s = standins[l % len(standins)]
        if l == 0:
            normed = layer_norm(x, ln1[l][0], ln1[l][1], eps)
        else:
            x = moe_combine(prev["expert_out"], routing["routes"], routing["route_positions"], rows)
            x, normed = add_layer_norm(x, carry, ln1[l][0], ln1[l][1], eps)
        q, k = rope(s["q"], s["k"], node_depth, q_heads, kv_heads, head_dim, cos, sin)
        s["q"][...] = q
        s["k"][...] = k
        attn, post = add_layer_norm(s["attn"], x, ln2[l][0], ln2[l][1], eps)
        s["attn"][...] = attn
        routing = route = moe_route(s["logits"])
        act = silu_mul(s["gate_up"][:, :inter], s["gate_up"][:, inter:])
        carry = s["attn"].copy()
        prev = s
        del normed, post, act, route
    x = moe_combine(prev["expert_out"], routing["routes"], routing["route_positions"], rows)
    return add_layer_norm(x, carry, final[0], final[1], eps)
