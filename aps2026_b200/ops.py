"""Host-side mirror of the reference's ``tensor_ops`` GPU ops on torch tensors.

Each function keeps the reference's name, argument meaning and error
behaviour (ezzy0654/aps2026 include/tensor.h:63-161): shapes that the
reference reads from ``Tensor::size()`` come from the torch tensors, a shape
mismatch raises ``ValueError`` where the reference throws
``std::invalid_argument``, and a CUDA failure raises ``RuntimeError`` where
its ``check_cuda`` throws ``std::runtime_error``. Every call goes through the
C ABI of libaps2026_b200.so on the current torch CUDA stream; tensors must be
contiguous fp32 (uint8 / int32 for index data) CUDA tensors.

PyTorch is used only for device memory and streams here.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib
from ._lib import B2_FLAG_EXACT_ORDER

NUM_EXPERTS = 16
ROUTER_SCORE_QUANTUM = 1.0e-3
ROUTER_TIE_EPS = 2.0e-2
SLIDING_WINDOW = 2047
ROPE_THETA = 10000.0
NORM_EPS = 1.0e-5


class InvalidArgument(ValueError):
    """The reference's std::invalid_argument."""


class CudaError(RuntimeError):
    """The reference's std::runtime_error from check_cuda."""


class FileError(RuntimeError):
    """The reference's std::runtime_error from the harness's file reader and
    writer (src/main.cpp:144-192)."""


def _check(rc: int, what: str) -> None:
    if rc == _lib.B2_OK:
        return
    msg = f"{what}: {_lib.last_error()}"
    if rc == _lib.B2_ERR_INVALID_ARGUMENT:
        raise InvalidArgument(msg)
    if rc == _lib.B2_ERR_UNSUPPORTED:
        raise InvalidArgument(f"unsupported: {msg}")
    if rc == _lib.B2_ERR_IO:
        raise FileError(msg)
    raise CudaError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise InvalidArgument("tensor is not on a CUDA device")
    if not t.is_contiguous():
        raise InvalidArgument("tensor is not contiguous")
    return t.data_ptr()


def _f32(t: torch.Tensor) -> int:
    if t.dtype != torch.float32:
        raise InvalidArgument(f"expected float32, got {t.dtype}")
    return _ptr(t)


def _u32(t: torch.Tensor) -> int:
    if t.dtype not in (torch.int32, torch.uint32):
        raise InvalidArgument(f"expected 32-bit indices, got {t.dtype}")
    return _ptr(t)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _flags(exact: bool) -> int:
    return B2_FLAG_EXACT_ORDER if exact else 0


def _rows_h(x: torch.Tensor) -> tuple[int, int]:
    h = x.shape[-1]
    return (x.numel() // h if h else 0), h


# ---- gather ---------------------------------------------------------------


def gather_rows_gpu(x: torch.Tensor, rows, out: torch.Tensor) -> None:
    """out[i, :] = x[rows[i], :]; rows: device int32 tensor or host sequence
    (tensor_ops::gather_rows_gpu, include/tensor.h:115-116, :138)."""
    x_rows, h = _rows_h(x)
    if not isinstance(rows, torch.Tensor):
        rows = torch.tensor(list(rows), dtype=torch.int32, device=x.device)
    count = rows.numel()
    if out.numel() != count * h:
        raise InvalidArgument("gather_rows shape")
    _check(_lib.lib().b2_gather_rows(_f32(x), x_rows, h, _u32(rows), count, _f32(out), _stream()),
           "gather_rows_gpu")


def moe_gather_compact_gpu(x: torch.Tensor, assignment_rows: torch.Tensor, out: torch.Tensor) -> None:
    """out[i, :] = x[assignment_rows[i], :], the expert-ordered input of the
    grouped expert GEMM (k_moe_gather_compact, src/tensor.cu:1420-1428)."""
    x_rows, h = _rows_h(x)
    count = assignment_rows.numel()
    if out.numel() != count * h:
        raise InvalidArgument("moe_gather_compact shape")
    _check(_lib.lib().b2_moe_gather_compact(_f32(x), x_rows, h, _u32(assignment_rows), count, _f32(out), _stream()),
           "moe_gather_compact_gpu")


# ---- LayerNorm ------------------------------------------------------------------


def layer_norm_gpu(x, weight, bias, eps: float, y, exact: bool = False) -> None:
    """tensor_ops::layer_norm_gpu (include/tensor.h:86-87)."""
    rows, h = _rows_h(x)
    if weight.numel() != h or bias.numel() != h or y.numel() != x.numel():
        raise InvalidArgument("layer norm shape")
    _check(_lib.lib().b2_layer_norm(_f32(x), _f32(weight), _f32(bias), _f32(y), rows, h, eps,
                                    _flags(exact), _stream()), "layer_norm_gpu")


def layer_norm_stats_gpu(x, eps: float, exact: bool = False):
    """Per-row mean and 1/std of x [rows, h] as b2_layer_norm forms them
    (b2_layer_norm_stats; the operand statistics of a GEMM prologue that
    applies b2_fusion::layer_norm_value). Returns (mean, inv), fp32 [rows]."""
    rows, h = _rows_h(x)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    inv = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(_lib.lib().b2_layer_norm_stats(_f32(x), rows, h, eps, _flags(exact), _ptr(mean), _ptr(inv), _stream()),
           "layer_norm_stats_gpu")
    return mean, inv


def add_layer_norm_gpu(x, residual, weight, bias, eps: float, y, exact: bool = False) -> None:
    """x += residual; y = LayerNorm(x) (tensor_ops::add_layer_norm_gpu,
    include/tensor.h:88-90)."""
    rows, h = _rows_h(x)
    if residual.numel() != x.numel() or weight.numel() != h or bias.numel() != h or y.numel() != x.numel():
        raise InvalidArgument("add layer norm shape")
    _check(_lib.lib().b2_add_layer_norm(_f32(x), _f32(residual), _f32(weight), _f32(bias), _f32(y),
                                        rows, h, eps, _flags(exact), _stream()), "add_layer_norm_gpu")


def moe_combine_add_layer_norm_gpu(expert_out, routes, route_positions, carry, weight, bias,
                                   eps: float, x_out, y, exact: bool = False) -> None:
    """x_out = combine(expert_out) + carry; y = LayerNorm(x_out): the MoE
    un-permute fused with the next layer's carried add + LN."""
    rows, h = _rows_h(carry)
    if x_out.numel() != carry.numel() or y.numel() != carry.numel() or routes.numel() != 2 * rows \
            or route_positions.numel() != 2 * rows or weight.numel() != h or bias.numel() != h:
        raise InvalidArgument("combine add layer norm shape")
    if routes.dtype != torch.uint8:
        raise InvalidArgument("routes must be uint8")
    expert_rows = expert_out.numel() // h
    _check(_lib.lib().b2_moe_combine_add_layer_norm(
        _f32(expert_out), expert_rows, _ptr(routes), _u32(route_positions), _f32(carry),
        _f32(weight), _f32(bias), _f32(x_out), _f32(y), rows, h, eps, _flags(exact), _stream()),
        "moe_combine_add_layer_norm_gpu")


# ---- RoPE ---------------------------------------------------------------------------


def rope_table_host(max_seq: int, head_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [max_seq, head_dim/2] built on the host exactly as the
    reference's rope_table (src/tensor.cu:2716-2724)."""
    half = head_dim // 2
    cos = torch.empty((max_seq, half), dtype=torch.float32)
    sin = torch.empty((max_seq, half), dtype=torch.float32)
    _check(_lib.lib().b2_rope_table(max_seq, head_dim, theta, cos.data_ptr(), sin.data_ptr()),
           "rope_table")
    return cos, sin


_ROPE_TABLES: dict = {}


def rope_table_gpu(max_seq: int, head_dim: int, theta: float, device=None):
    """Device copy of the table, cached per (device, head_dim, theta) and grown
    to the largest max_seq seen, as the reference caches its static table."""
    device = torch.device(device or torch.cuda.current_device())
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    key = (device, head_dim, float(theta))
    hit = _ROPE_TABLES.get(key)
    if hit is None or hit[0].shape[0] < max_seq:
        cos, sin = rope_table_host(max_seq, head_dim, theta)
        hit = (cos.to(device), sin.to(device))
        _ROPE_TABLES[key] = hit
    return hit


def apply_rope_tree_gpu(q, k, row_pos, rows: int, max_seq: int, q_heads: int, kv_heads: int,
                        head_dim: int, theta: float) -> None:
    """RoPE on trie rows: row r at position row_pos[r]
    (tensor_ops::apply_rope_tree_gpu, include/tensor.h:104-108)."""
    if q.numel() != rows * q_heads * head_dim or k.numel() != rows * kv_heads * head_dim:
        raise InvalidArgument("rope shape")
    cos, sin = rope_table_gpu(max_seq, head_dim, theta, q.device)
    _check(_lib.lib().b2_rope(_f32(q), _f32(k), _u32(row_pos), rows, q_heads, kv_heads, head_dim,
                              _f32(cos), _f32(sin), cos.shape[0], _stream()), "apply_rope_tree_gpu")


def apply_rope_gpu(q, k, seq_lens: Sequence[int], q_heads: int, kv_heads: int, head_dim: int,
                   theta: float) -> None:
    """RoPE over packed segments, position resetting per segment
    (tensor_ops::apply_rope_gpu, include/tensor.h:91-94)."""
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in seq_lens]).to(q.device)
    apply_rope_tree_gpu(q, k, pos, pos.numel(), max(seq_lens), q_heads, kv_heads, head_dim, theta)


# ---- softmax --------------------------------------------------------------------------


def causal_softmax_gpu(scores, probs, scale: float, window: int = SLIDING_WINDOW,
                       exact: bool = False) -> None:
    """probs = causal sliding-window softmax(scores * scale) over the last
    dim of [heads, T, T] (the softmax of k_attention_tree_gqa4)."""
    if scores.dim() != 3 or scores.shape[1] != scores.shape[2] or probs.shape != scores.shape:
        raise InvalidArgument("causal softmax shape")
    heads, T, _ = scores.shape
    _check(_lib.lib().b2_causal_softmax(_f32(scores), _f32(probs), heads, T, T, scale, window,
                                        _flags(exact), _stream()), "causal_softmax_gpu")


def attention_tree_gpu(q, k, v, out, row_pos, anc, anc_stride: int, rows: int, q_heads: int, kv_heads: int,
                       head_dim: int, window: int = SLIDING_WINDOW, exact: bool = False) -> None:
    """Prefix-tree GQA-4 attention on trie rows (tensor_ops::attention_tree_gpu,
    include/tensor.h:109-114); anc: device int32 [rows, anc_stride]."""
    if q_heads != 4 * kv_heads:
        raise InvalidArgument("attention_tree_gpu expects GQA-4")
    if (q.numel() != rows * q_heads * head_dim or out.numel() != q.numel()
            or k.numel() != rows * kv_heads * head_dim or v.numel() != k.numel()
            or row_pos.numel() != rows or anc.numel() != rows * anc_stride):
        raise InvalidArgument("attention shape")
    _check(_lib.lib().b2_attention_tree(_f32(q), _f32(k), _f32(v), _f32(out), _u32(row_pos), _u32(anc), anc_stride,
                                        rows, q_heads, kv_heads, head_dim, window, _flags(exact), _stream()),
           "attention_tree_gpu")


def attention_tree_compact_gpu(q, k, v, out, row_pos, node_prompt, prompt_offsets, token_node, max_len: int,
                               rows: int, q_heads: int, kv_heads: int, head_dim: int,
                               window: int = SLIDING_WINDOW, exact: bool = False) -> None:
    """attention_tree_gpu with compact ancestor chains (the node witnesses of
    prefix_trie_device): row r's chain is token_node[prompt_offsets[p]:][:pos + 1],
    p = node_prompt[r]."""
    if q_heads != 4 * kv_heads:
        raise InvalidArgument("attention_tree_gpu expects GQA-4")
    prompts = prompt_offsets.numel() - 1
    if (q.numel() != rows * q_heads * head_dim or out.numel() != q.numel()
            or k.numel() != rows * kv_heads * head_dim or v.numel() != k.numel()
            or row_pos.numel() != rows or node_prompt.numel() != rows or prompts < 1):
        raise InvalidArgument("attention shape")
    _check(_lib.lib().b2_attention_tree_compact(
        _f32(q), _f32(k), _f32(v), _f32(out), _u32(row_pos), _u32(node_prompt), _u32(prompt_offsets), prompts,
        _u32(token_node), token_node.numel(), max_len, rows, q_heads, kv_heads, head_dim, window, _flags(exact),
        _stream()), "attention_tree_compact_gpu")


# ---- MoE ----------------------------------------------------------------------------------


@dataclass
class MoeRouting:
    """Outputs of the routing step of moe_forward_grouped_gpu."""
    routes: torch.Tensor            # uint8 [T, 2]
    counts: torch.Tensor            # int32 [E]
    offsets: torch.Tensor           # int32 [E+1]
    assignment_rows: torch.Tensor   # int32 [2T]
    route_positions: torch.Tensor   # int32 [2T]
    work_expert64: torch.Tensor
    work_start64: torch.Tensor
    work_expert128: torch.Tensor
    work_start128: torch.Tensor


def queue_lengths(T: int, E: int) -> tuple[int, int]:
    return (2 * T + 63) // 64 + E, (2 * T + 127) // 128 + E


class RouteWorkspace:
    """Caller-owned routing scratch (per-tile expert histograms)."""

    def __init__(self, T: int, E: int, device):
        n = C.c_size_t(0)
        _check(_lib.lib().b2_moe_route_workspace_size(T, E, C.addressof(n)), "workspace size")
        self.bytes = n.value
        self.buf = torch.empty(max(self.bytes, 16), dtype=torch.uint8, device=device)


def alloc_routing(T: int, E: int, device) -> MoeRouting:
    n64, n128 = queue_lengths(T, E)
    z = lambda n, dt=torch.int32: torch.empty(n, dtype=dt, device=device)  # noqa: E731
    return MoeRouting(z(2 * T, torch.uint8).view(T, 2), z(E), z(E + 1), z(2 * T), z(2 * T),
                      z(n64), z(n64), z(n128), z(n128))


def moe_route_gpu(logits, out: MoeRouting | None = None, ws: RouteWorkspace | None = None,
                  quantum: float = ROUTER_SCORE_QUANTUM, tie_eps: float = ROUTER_TIE_EPS) -> MoeRouting:
    """Top-2 routing + stable token->expert permutation of router logits [T, E]
    (k_moe_top2 / k_moe_offsets_work / k_moe_fill_stable)."""
    if logits.dim() != 2:
        raise InvalidArgument("grouped MoE shape or handle")
    T, E = logits.shape
    out = out or alloc_routing(T, E, logits.device)
    ws = ws or RouteWorkspace(T, E, logits.device)
    _check(_lib.lib().b2_moe_route(
        _f32(logits), T, E, quantum, tie_eps, _ptr(out.routes), _u32(out.counts), _u32(out.offsets),
        _u32(out.assignment_rows), _u32(out.route_positions), _u32(out.work_expert64),
        _u32(out.work_start64), _u32(out.work_expert128), _u32(out.work_start128),
        _ptr(ws.buf), ws.bytes, _stream()), "moe_route_gpu")
    return out


def silu_mul_gpu(gate, up, out, exact: bool = True) -> None:
    """out = silu(gate) * up (tensor_ops::silu_mul_gpu, include/tensor.h:85).
    2-D views with a row stride (e.g. halves of a [2T, 896] gate|up buffer)
    are accepted. exact=True (the reference's contract) is bit-exact;
    exact=False is the tree-order mode's expf form (b2_silu_mul_flags)."""
    if gate.shape != up.shape or out.shape != gate.shape:
        raise InvalidArgument("silu_mul shape")
    if gate.dim() == 1:
        gate, up, out = gate.view(1, -1), up.view(1, -1), out.view(1, -1)
    for t in (gate, up, out):
        if t.dim() != 2 or t.stride(1) != 1 or not t.is_cuda or t.dtype != torch.float32:
            raise InvalidArgument("silu_mul layout")
    rows, cols = gate.shape
    if exact:
        rc = _lib.lib().b2_silu_mul(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0),
                                    out.data_ptr(), out.stride(0), rows, cols, _stream())
    else:
        rc = _lib.lib().b2_silu_mul_flags(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0),
                                          out.data_ptr(), out.stride(0), rows, cols, 0, _stream())
    _check(rc, "silu_mul_gpu")


def moe_combine_gpu(expert_out, routes, route_positions, out) -> None:
    """out[t] = 0.5 * E[lo] + 0.5 * E[hi] (k_moe_combine)."""
    T, h = _rows_h(out)
    if routes.numel() != 2 * T or route_positions.numel() != 2 * T or expert_out.shape[-1] != h:
        raise InvalidArgument("moe combine shape")
    _check(_lib.lib().b2_moe_combine(_f32(expert_out), expert_out.numel() // h, _ptr(routes),
                                     _u32(route_positions), _f32(out), T, h, _stream()), "moe_combine_gpu")


def add_inplace_gpu(a, b) -> None:
    """a += b (tensor_ops::add_inplace_gpu, include/tensor.h:83)."""
    if a.numel() != b.numel():
        raise InvalidArgument("add shape")
    _check(_lib.lib().b2_add(_f32(a), _f32(b), a.numel(), _stream()), "add_inplace_gpu")


def device_status() -> int:
    """Reads and clears the in-kernel bounds-check word (B2_CHECK_* bits)."""
    v = C.c_uint32(0)
    _check(_lib.lib().b2_device_status(C.addressof(v), _stream()), "device_status")
    return v.value


# ---- prefix trie (host) ------------------------------------------------------------------------


@dataclass
class PrefixTrie:
    token_node: "object"   # numpy uint32 [total tokens]
    node_token: "object"   # numpy uint32 [nodes]
    node_depth: "object"   # numpy uint32 [nodes]
    node_anc: "object"     # numpy uint32 [nodes, anc_stride] or None
    anc_stride: int
    nodes: int


def prefix_trie(prompts: Sequence[Sequence[int]], vocab: int = 32064, max_len: int = 4096,
                with_ancestors: bool = False) -> PrefixTrie:
    """Prefix-trie dedup of a prompt batch, numbered as
    PhiTinyMoEModel::generate numbers it (src/model.cu:64-117)."""
    import numpy as np

    lens = np.array([len(p) for p in prompts], dtype=np.uint32)
    ids = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts])
                               if len(prompts) else np.zeros(0, np.int32))
    total = int(lens.sum())
    stride = int(lens.max()) if len(prompts) else 0
    token_node = np.empty(total, np.uint32)
    node_token = np.empty(max(total, 1), np.uint32)
    node_depth = np.empty(max(total, 1), np.uint32)
    anc = np.empty(max(total, 1) * stride, np.uint32) if with_ancestors else None
    nodes = C.c_size_t(0)
    _check(_lib.lib().b2_prefix_trie_build(
        ids.ctypes.data, lens.ctypes.data, len(prompts), vocab, max_len, token_node.ctypes.data,
        node_token.ctypes.data, node_depth.ctypes.data, anc.ctypes.data if anc is not None else None,
        stride, C.addressof(nodes)), "prefix_trie")
    n = nodes.value
    return PrefixTrie(token_node, node_token[:n].copy(), node_depth[:n].copy(),
                      anc[: n * stride].reshape(n, stride).copy() if anc is not None else None,
                      stride, n)


@dataclass
class DeviceTrie:
    """Outputs of b2_prefix_trie_device (int32 device tensors)."""
    token_node: torch.Tensor   # [total]
    node_token: torch.Tensor   # [nodes]
    node_depth: torch.Tensor   # [nodes]
    node_prompt: torch.Tensor  # [nodes]: a prompt containing the node
    nodes: int


class TrieWorkspace:
    """Caller-owned scratch of b2_prefix_trie_device."""

    def __init__(self, batch: int, device):
        n = C.c_size_t(0)
        _check(_lib.lib().b2_prefix_trie_device_workspace_size(batch, C.addressof(n)), "workspace size")
        self.bytes = n.value
        self.buf = torch.empty(max(1, (self.bytes + 3) // 4), dtype=torch.int32, device=device)


def prefix_trie_device(ids: torch.Tensor, offsets: torch.Tensor, vocab: int = 32064, max_len: int = 4096,
                       ws: "TrieWorkspace | None" = None) -> DeviceTrie:
    """The prefix trie of the prompts ids[offsets[b]:offsets[b+1]] (int32
    device tensors) built on the GPU and numbered as PhiTinyMoEModel::generate
    numbers it (src/model.cu:64-117); reads the node count back (a 4-byte
    copy, which waits for the build)."""
    batch, total = offsets.numel() - 1, ids.numel()
    if batch < 1:
        raise InvalidArgument("generate received an empty input batch")
    dev = ids.device
    e = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=dev)  # noqa: E731
    token_node, node_token, node_depth, node_prompt, count = e(total), e(total), e(total), e(total), e(1)
    ws = ws or TrieWorkspace(batch, dev)
    _check(_lib.lib().b2_prefix_trie_device(_u32(ids), _u32(offsets), batch, total, vocab, max_len, _u32(token_node),
                                            _u32(node_token), _u32(node_depth), _u32(node_prompt), _u32(count),
                                            ws.buf.data_ptr(), ws.bytes, _stream()), "prefix_trie_device")
    n = int(count[0].item())
    return DeviceTrie(token_node[:total], node_token[:n], node_depth[:n], node_prompt[:n], n)


# ---- input and output files of the prefill harness --------------------------------------------


@dataclass
class InputBatch:
    """The prompts of an inputs.bin file in file order, packed back to back
    as b2_prefix_trie_build takes them."""
    ids: "object"       # numpy int32 [total tokens]
    seq_lens: "object"  # numpy uint32 [batch]
    max_seq_len: int    # the file's header field

    def prompts(self) -> list[list[int]]:
        import numpy as np

        ends = np.cumsum(self.seq_lens, dtype=np.int64)
        return [self.ids[e - n:e].tolist() for n, e in zip(self.seq_lens.tolist(), ends.tolist())]


def read_inputs(path, max_len: int = 4096) -> InputBatch:
    """Reads a variable-length prompt file as read_inputs does
    (src/main.cpp:144-181): same checks, same messages (FileError)."""
    import numpy as np

    b, m, total = C.c_uint32(0), C.c_uint32(0), C.c_size_t(0)
    raw = str(path).encode()
    L = _lib.lib()
    _check(L.b2_read_inputs(raw, max_len, C.addressof(b), C.addressof(m), C.addressof(total),
                            None, 0, None, 0), "read_inputs")
    lens = np.empty(b.value, np.uint32)
    ids = np.empty(max(total.value, 1), np.int32)
    _check(L.b2_read_inputs(raw, max_len, None, None, None, lens.ctypes.data, lens.size, ids.ctypes.data,
                            ids.size), "read_inputs")
    return InputBatch(ids[: total.value], lens, m.value)


def write_outputs(path, logits) -> None:
    """Writes [batch, vocab] fp32 logits as write_outputs does
    (src/main.cpp:183-192), byte for byte. A CUDA tensor is streamed from the
    device on the current stream (after the work already on it); a CPU tensor
    or numpy array is written directly."""
    import numpy as np

    if isinstance(logits, torch.Tensor):
        if logits.dtype != torch.float32 or logits.dim() != 2 or not logits.is_contiguous():
            raise InvalidArgument("logits must be a contiguous 2-D float32 tensor")
        on_dev = logits.is_cuda
        batch, vocab = logits.shape
        ptr = logits.data_ptr() if logits.numel() else None
        keep = logits
    else:
        keep = np.ascontiguousarray(logits, dtype=np.float32)
        if keep.ndim != 2:
            raise InvalidArgument("logits must be 2-D")
        on_dev = False
        batch, vocab = keep.shape
        ptr = keep.ctypes.data if keep.size else None
    _check(_lib.lib().b2_write_outputs(str(path).encode(), ptr, batch, vocab, int(on_dev),
                                       _stream() if on_dev else None), "write_outputs")
    del keep
