"""Non-GEMM prefill pipeline: prefix-trie dedup, the per-layer op sequence of
PhiDecoderLayer::forward_carry over all layers, the final add + LayerNorm,
and prompt sharding across GPUs with one NCCL gather of the final hidden
states.

The GEMM outputs of each layer (q/k projections, attention + o_proj, router
logits, expert gate/up and W2 outputs) are supplied as seeded stand-in
tensors of the config.h shapes (``StandIns``): the projections are outside
this path. Everything on the path itself runs through the C ABI
(``b2_prefill_layers`` for the layer loop, ``b2_prefix_trie_build`` or, for
end-to-end steps, ``b2_prefix_trie_device`` for the trie, ``b2_gather_rows``
for the expansion back to token rows).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np
import torch

from . import _lib, ops

VOCAB = 32064
HIDDEN = 4096
LAYERS = 32
Q_HEADS = 16
KV_HEADS = 4
HEAD_DIM = 128
EXPERTS = 16
INTER = 448
MAX_POS = 4096


class Shape(C.Structure):
    _fields_ = [("rows", C.c_size_t), ("hidden", C.c_size_t), ("q_heads", C.c_size_t),
                ("kv_heads", C.c_size_t), ("head_dim", C.c_size_t), ("experts", C.c_size_t),
                ("intermediate", C.c_size_t), ("eps", C.c_float), ("router_quantum", C.c_float),
                ("router_tie_eps", C.c_float), ("flags", C.c_uint32)]


class Layer(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("attn", C.c_void_p), ("router_logits", C.c_void_p),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("ld_gate_up", C.c_size_t),
                ("expert_out", C.c_void_p), ("ln1_gamma", C.c_void_p), ("ln1_beta", C.c_void_p),
                ("ln2_gamma", C.c_void_p), ("ln2_beta", C.c_void_p)]


class Work(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "normed", "post", "act", "routes", "counts", "offsets",
                                          "assignment_rows", "route_positions", "work_expert64",
                                          "work_start64", "work_expert128", "work_start128", "route_ws")] + [
        ("route_ws_bytes", C.c_size_t)]


def launches_per_run(layers: int) -> int:
    """Kernel launches of one b2_prefill_layers call (B2_PREFILL_LAUNCHES):
    gather + LN0 + per layer RoPE, add+LN, routing (2 kernels), SiLU, and the
    31 + 1 fused un-permute + add + LN launches."""
    return 2 + 6 * layers


# ---- synthetic inputs (BASELINE configs 4 and 5) -------------------------------------


def prompts_config4(seed: int = 3, batch: int = 16, length: int = 1024, shared: int = 256) -> list[np.ndarray]:
    """16 prompts x 1024 tokens whose first 256 tokens are identical; ids
    uniform over the vocabulary."""
    g = np.random.default_rng(seed)
    prefix = g.integers(0, VOCAB, shared)
    return [np.concatenate([prefix, g.integers(0, VOCAB, length - shared)]).astype(np.int32) for _ in range(batch)]


def prompts_config5(seed: int = 4, batch: int = 64, length: int = 2048) -> list[np.ndarray]:
    """64 prompts x 2048 tokens, ids uniform over the vocabulary."""
    g = np.random.default_rng(seed)
    return [g.integers(0, VOCAB, length).astype(np.int32) for _ in range(batch)]


def _randn(shape, gen, device, mean=0.0, std=1.0):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t


@dataclass
class Weights:
    """Embedding table and LayerNorm parameters (random init of the
    architecture: emb ~ N(0, 0.02), gamma ~ N(1, 0.1), beta ~ N(0, 0.1))."""
    emb: torch.Tensor
    ln1: list  # [(gamma, beta)] per layer (input_layernorm)
    ln2: list  # post_attention_layernorm
    final: tuple

    @staticmethod
    def make(device, seed: int, layers: int = LAYERS, vocab: int = VOCAB, hidden: int = HIDDEN) -> "Weights":
        gen = torch.Generator(device=device).manual_seed(seed)
        emb = _randn((vocab, hidden), gen, device, std=0.02)
        ln = lambda: (_randn(hidden, gen, device, 1.0, 0.1), _randn(hidden, gen, device, 0.0, 0.1))  # noqa: E731
        return Weights(emb, [ln() for _ in range(layers)], [ln() for _ in range(layers)], ln())


@dataclass
class StandIns:
    """Seeded N(0,1) stand-ins for one layer's GEMM outputs (config.h shapes)."""
    q: torch.Tensor           # [rows, q_heads*head_dim]
    k: torch.Tensor           # [rows, kv_heads*head_dim]
    attn: torch.Tensor        # [rows, hidden]
    logits: torch.Tensor      # [rows, experts]
    gate_up: torch.Tensor     # [2*rows, 2*intermediate]: gate | up per row
    expert_out: torch.Tensor  # [2*rows, hidden]

    @staticmethod
    def make(rows: int, device, gen, hidden=HIDDEN, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
             experts=EXPERTS, inter=INTER) -> "StandIns":
        return StandIns(_randn((rows, q_heads * head_dim), gen, device), _randn((rows, kv_heads * head_dim), gen, device),
                        _randn((rows, hidden), gen, device), _randn((rows, experts), gen, device),
                        _randn((2 * rows, 2 * inter), gen, device), _randn((2 * rows, hidden), gen, device))

    def nbytes(self) -> int:
        return sum(t.numel() * 4 for t in (self.q, self.k, self.attn, self.logits, self.gate_up, self.expert_out))


def standin_bytes(rows: int) -> int:
    return 4 * rows * (Q_HEADS * HEAD_DIM + KV_HEADS * HEAD_DIM + HIDDEN + EXPERTS + 2 * 2 * INTER + 2 * HIDDEN)


# ---- the batch on one GPU ------------------------------------------------------------------


@dataclass
class Batch:
    """A prompt batch deduplicated onto prefix-trie nodes, with its index
    arrays on the device."""
    prompts: list
    trie: "ops.PrefixTrie | None"  # the host trie; None when it was built on the device
    node_token: torch.Tensor    # int32 [nodes] on device
    node_depth: torch.Tensor    # int32 [nodes]
    token_node: torch.Tensor    # int32 [tokens]
    last_rows: torch.Tensor     # int32 [batch]: node of each prompt's last token
    max_len: int
    rows: int                   # trie nodes
    tokens: int

    @staticmethod
    def build(prompts: Sequence[np.ndarray], device, pinned: bool = False, stream=None) -> "Batch":
        trie = ops.prefix_trie(prompts)
        lens = np.array([len(p) for p in prompts])
        ends = np.cumsum(lens) - 1
        last = trie.token_node[ends].astype(np.int32)

        def up(a):
            t = torch.from_numpy(a.view(np.int32))
            if pinned:
                t = t.pin_memory()
            return t.to(device, non_blocking=pinned)

        return Batch(list(prompts), trie, up(trie.node_token), up(trie.node_depth), up(trie.token_node),
                     up(last), int(lens.max()), trie.nodes, int(lens.sum()))


class Pipeline:
    """Owns the working buffers of one GPU's share of the batch and runs the
    non-GEMM layer loop through ``b2_prefill_layers``."""

    def __init__(self, batch: Batch, weights: Weights, device, exact: bool = False,
                 hidden=HIDDEN, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM, experts=EXPERTS,
                 inter=INTER, eps=1e-5):
        self.batch, self.weights, self.device = batch, weights, device
        R = batch.rows
        self.shape = Shape(R, hidden, q_heads, kv_heads, head_dim, experts, inter, eps, ops.ROUTER_SCORE_QUANTUM,
                           ops.ROUTER_TIE_EPS, ops.B2_FLAG_EXACT_ORDER if exact else 0)
        e = lambda *s, dt=torch.float32: torch.empty(s, dtype=dt, device=device)  # noqa: E731
        self.x, self.normed, self.post = e(R, hidden), e(R, hidden), e(R, hidden)
        self.act = e(2 * R, inter)
        self.final_x, self.final_out = e(R, hidden), e(R, hidden)
        self.routing = ops.alloc_routing(R, experts, device)
        self.route_ws = ops.RouteWorkspace(R, experts, device)
        self.cos, self.sin = ops.rope_table_gpu(max(batch.max_len, 1), head_dim, ops.ROPE_THETA, device)
        r = self.routing
        self.work = Work(self.x.data_ptr(), self.normed.data_ptr(), self.post.data_ptr(), self.act.data_ptr(),
                         r.routes.data_ptr(), r.counts.data_ptr(), r.offsets.data_ptr(), r.assignment_rows.data_ptr(),
                         r.route_positions.data_ptr(), r.work_expert64.data_ptr(), r.work_start64.data_ptr(),
                         r.work_expert128.data_ptr(), r.work_start128.data_ptr(), self.route_ws.buf.data_ptr(),
                         self.route_ws.bytes)
        self._fn = _lib.lib().b2_prefill_layers
        self._layers = None
        self._layer_key = None

    def bind_layers(self, standins: Sequence[StandIns], layers: int | None = None) -> None:
        """Layer l uses stand-in set standins[l % len(standins)]."""
        layers = layers or len(self.weights.ln1)
        w = self.weights
        arr = (Layer * layers)()
        for l in range(layers):
            s = standins[l % len(standins)]
            inter = self.shape.intermediate
            arr[l] = Layer(s.q.data_ptr(), s.k.data_ptr(), s.attn.data_ptr(), s.logits.data_ptr(),
                           s.gate_up.data_ptr(), s.gate_up.data_ptr() + 4 * inter, s.gate_up.stride(0),
                           s.expert_out.data_ptr(), w.ln1[l][0].data_ptr(), w.ln1[l][1].data_ptr(),
                           w.ln2[l][0].data_ptr(), w.ln2[l][1].data_ptr())
        self._layers = arr
        self._standins = list(standins)

    def run(self, stream=None, timer: "StageTimer | None" = None, final_out: torch.Tensor | None = None) -> None:
        """Enqueues all layers + the final LayerNorm on `stream` (default:
        the current torch stream); `timer` records per-launch events;
        `final_out` redirects the final LayerNorm output (e.g. straight into
        a send buffer when node rows are token rows)."""
        if self._layers is None:
            raise RuntimeError("bind_layers() first")
        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
        w = self.weights
        ev = timer.handles() if timer is not None else None
        out = self.final_out if final_out is None else final_out
        if out.numel() != self.final_out.numel() or out.dtype != torch.float32 or not out.is_contiguous():
            raise ops.InvalidArgument("final_out shape")
        rc = self._fn(C.addressof(self.shape), w.emb.data_ptr(), w.emb.shape[0], self.batch.node_token.data_ptr(),
                      self.batch.node_depth.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(), self.cos.shape[0],
                      C.addressof(self._layers), len(self._layers), w.final[0].data_ptr(), w.final[1].data_ptr(),
                      C.addressof(self.work), self.final_x.data_ptr(), out.data_ptr(),
                      C.addressof(ev) if ev is not None else None, st)
        ops._check(rc, "b2_prefill_layers")

    def expand_to_tokens(self, out: torch.Tensor) -> None:
        """Final hidden states of every token row: out[t] = final_out[token_node[t]]."""
        ops.gather_rows_gpu(self.final_out, self.batch.token_node, out)

    def last_token_rows(self, out: torch.Tensor) -> None:
        """Final hidden state of each prompt's last token (the lm_head input)."""
        ops.gather_rows_gpu(self.final_out, self.batch.last_rows, out)


def identity_rows(batch: Batch) -> bool:
    """True when every token row is its own trie node in order (no shared
    prefixes): the final node rows are then already the token rows. (With as
    many nodes as tokens every token creates its node, and creation order is
    token order.)"""
    return batch.rows == batch.tokens


def slice_standins(s: StandIns, r0: int, rows: int) -> StandIns:
    """Row range [r0, r0 + rows) of a stand-in set (assignment-ordered
    tensors use rows [2 r0, 2 (r0 + rows)))."""
    return StandIns(s.q[r0:r0 + rows], s.k[r0:r0 + rows], s.attn[r0:r0 + rows], s.logits[r0:r0 + rows],
                    s.gate_up[2 * r0:2 * (r0 + rows)], s.expert_out[2 * r0:2 * (r0 + rows)])


class HostStage:
    """The host side of an end-to-end step: takes a chunk's prompts as host
    token ids and makes its Batch on the device.

    Device mode (default): packs [offsets | ids] into a pinned buffer, copies
    it up asynchronously and builds the trie on the GPU
    (b2_prefix_trie_device) on a high-priority stream of its own, so the
    build overlaps the previous step still running; only the node counts
    come back (the host needs them to size the launches), read once per step
    after every chunk's build is enqueued. Host mode: builds
    the trie on the host (b2_prefix_trie_build) and copies its index arrays
    up on the current stream.

    Every buffer exists twice and alternates by step, so preparing step k + 1
    waits only for step k - 1 (mark_used() records when a step is done with
    its buffers); all buffers are sized once, for the batches given
    (allocating pinned memory inside a timed loop would stall it)."""

    def __init__(self, device, batches: Sequence["Batch"], on_device: bool = True):
        self.device, self.on_device = device, on_device
        pin = lambda n: torch.empty(n, dtype=torch.int32, pin_memory=True)  # noqa: E731
        dev = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=device)  # noqa: E731
        if on_device:
            n = [2 * len(b.prompts) + 1 + b.tokens for b in batches]  # offsets | ids | last-token rows
            self.host = [[pin(k) for k in n] for _ in range(2)]
            # per slot and chunk: packed input, then token_node, node_token, node_depth, node_prompt
            self.dev_in = [[dev(k) for k in n] for _ in range(2)]
            self.dev_out = [[[dev(b.tokens) for _ in range(4)] for b in batches] for _ in range(2)]
            self.count_dev = [dev(len(batches)) for _ in range(2)]
            self.count_host = [pin(len(batches)) for _ in range(2)]
            self.ws = [ops.TrieWorkspace(len(b.prompts), device) for b in batches]
            _, high = torch.cuda.Stream.priority_range()
            self.stream = torch.cuda.Stream(device, priority=high)
        else:
            n = [2 * b.rows + b.tokens + len(b.prompts) for b in batches]
            self.host = [[pin(k) for k in n] for _ in range(2)]
        self.done = [[None] * len(batches) for _ in range(2)]  # the copy that last read host[slot][c]
        self.used = [None, None]                               # the step that last read slot's outputs
        self.slot = 0

    def mark_used(self) -> None:
        """Records, on the current stream, that the step just enqueued is the
        last reader of this slot's device buffers."""
        ev = torch.cuda.Event()
        ev.record()
        self.used[self.slot] = ev

    def upload_all(self, chunks: Sequence[Sequence[np.ndarray]]) -> "list[Batch]":
        """One Batch per chunk of prompts (the chunks the stage was sized
        for). Device mode launches every chunk's build before it reads the
        node counts back, so the host waits once per step."""
        self.slot ^= 1
        if not self.on_device:
            return [self._upload_host(c, ps) for c, ps in enumerate(chunks)]
        pending = [self._launch_device(c, ps) for c, ps in enumerate(chunks)]
        built = torch.cuda.Event()
        built.record(self.stream)
        built.synchronize()  # the node counts size the chunks' launches
        torch.cuda.current_stream(self.device).wait_event(built)
        out = []
        for c, (prompts, lens, total, last) in enumerate(pending):
            tn, nt, nd, _ = self.dev_out[self.slot][c]
            nodes = int(self.count_host[self.slot][c])
            out.append(Batch(list(prompts), None, nt[:nodes], nd[:nodes], tn[:total], last, int(lens.max()), nodes,
                             total))
        return out

    def _fill(self, c: int, parts) -> torch.Tensor:
        n = sum(int(a.size) for a in parts)
        if self.done[self.slot][c] is not None:
            self.done[self.slot][c].synchronize()
        buf = self.host[self.slot][c]
        if buf.numel() < n:
            raise ValueError("HostStage: a batch larger than the one it was sized for")
        view, k = buf.numpy(), 0
        for a in parts:
            view[k:k + a.size] = a.view(np.int32)
            k += a.size
        return buf[:n]

    def _upload_host(self, c: int, prompts) -> "Batch":
        trie = ops.prefix_trie(prompts)
        lens = np.array([len(p) for p in prompts])
        last = trie.token_node[np.cumsum(lens) - 1]
        parts = [trie.node_token, trie.node_depth, trie.token_node, last]
        src = self._fill(c, parts)
        dev = torch.empty(src.numel(), dtype=torch.int32, device=self.device)
        dev.copy_(src, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.done[self.slot][c] = ev
        out, k = [], 0
        for a in parts:
            out.append(dev[k:k + a.size])
            k += a.size
        return Batch(list(prompts), trie, out[0], out[1], out[2], out[3], int(lens.max()), trie.nodes,
                     int(lens.sum()))

    def _launch_device(self, c: int, prompts):
        s, slot = self.stream, self.slot
        lens = np.array([len(p) for p in prompts], dtype=np.int64)
        offs = np.zeros(len(prompts) + 1, np.int32)
        offs[1:] = np.cumsum(lens)
        total = int(offs[-1])
        ids = np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts])
        ends = offs[1:] - 1
        src = self._fill(c, [offs, ids, ends])
        dev_in = self.dev_in[slot][c]
        tn, nt, nd, npr = self.dev_out[slot][c]
        if self.used[slot] is not None:
            s.wait_event(self.used[slot])  # the step two back has finished with these buffers
        with torch.cuda.stream(s):
            dev_in[:src.numel()].copy_(src, non_blocking=True)
            done = torch.cuda.Event()
            done.record(s)
            self.done[slot][c] = done
            offsets, ids_d = dev_in[:offs.size], dev_in[offs.size:offs.size + total]
            ends_d = dev_in[offs.size + total:offs.size + total + ends.size]
            ws = self.ws[c]
            ops._check(ops._lib.lib().b2_prefix_trie_device(
                ids_d.data_ptr(), offsets.data_ptr(), len(prompts), total, VOCAB, 4096, tn.data_ptr(),
                nt.data_ptr(), nd.data_ptr(), npr.data_ptr(), self.count_dev[slot][c:c + 1].data_ptr(),
                ws.buf.data_ptr(), ws.bytes, s.cuda_stream), "prefix_trie_device")
            last = torch.index_select(tn, 0, ends_d)
            self.count_host[slot][c:c + 1].copy_(self.count_dev[slot][c:c + 1], non_blocking=True)
        return prompts, lens, total, last


def chunk_tokens(prompts: Sequence[np.ndarray], plan: list) -> list:
    """tokens[r][c]: token rows of rank r's chunk c under `plan`
    (shard.chunk_plan); every rank computes the same table."""
    return [[sum(len(prompts[i]) for i in part) for part in parts] for parts in plan]


class FinalGather:
    """Collects every rank's final hidden states (token rows, chunk by chunk)
    on rank 0 with point-to-point transfers: for chunk c each rank r > 0
    sends its rows to rank 0 and rank 0 receives them into a buffer of
    exactly that size, so ranks may hold different token counts and
    different numbers of chunks (prompts of unequal length shard unevenly).

    post(c, rows) issues chunk c's transfers as one batch
    (torch.distributed.batch_isend_irecv: a grouped ncclSend / ncclRecv on
    NCCL's stream, which first waits for the stream current at the call, so
    a chunk is sent once its rows are written). Every rank calls post for
    every c < chunks(), in order, including chunks it does not hold itself
    (rank 0 receives them). Transfers between two ranks are matched in
    posting order. Rank 0's own rows stay where they are."""

    def __init__(self, tokens: list, rank: int, hidden: int, device, dtype=None, group=None):
        import torch.distributed as dist

        self.dist, self.tokens, self.rank, self.group = dist, tokens, rank, group
        self.world = len(tokens)
        dtype = dtype or torch.float32
        self.recv = {}
        if rank == 0:
            for r in range(1, self.world):
                for c, n in enumerate(tokens[r]):
                    self.recv[(c, r)] = torch.empty((n, hidden), device=device, dtype=dtype)

    def chunks(self) -> int:
        return max(len(t) for t in self.tokens)

    def _peer(self, r: int) -> int:
        """Global rank of group rank r."""
        return r if self.group is None else self.dist.get_global_rank(self.group, r)

    def post(self, c: int, rows: "torch.Tensor | None") -> list:
        d = self.dist
        ops = []
        if self.rank == 0:
            for r in range(1, self.world):
                if c < len(self.tokens[r]):
                    ops.append(d.P2POp(d.irecv, self.recv[(c, r)], self._peer(r), self.group))
        elif c < len(self.tokens[self.rank]):
            if rows is None or rows.shape[0] != self.tokens[self.rank][c]:
                raise ValueError(f"FinalGather: chunk {c} of rank {self.rank} has the wrong row count")
            ops.append(d.P2POp(d.isend, rows, self._peer(0), self.group))
        return d.batch_isend_irecv(ops) if ops else []

    def rows(self, c: int, r: int, own: "torch.Tensor | None" = None) -> "torch.Tensor":
        """Rank 0, after the transfers completed: rank r's chunk c (`own` is
        rank 0's own rows for r == 0)."""
        return own if r == 0 else self.recv[(c, r)]


class ShardedPrefill:
    """One rank's share of a prompt batch on one GPU, split into `chunks`
    sub-batches. Each chunk runs all layers (b2_prefill_layers), writes its
    final hidden states as token rows, and -- with world > 1 -- is sent to
    rank 0 (FinalGather: NCCL send / recv on the collective's own stream)
    while the next chunk computes, so only the last chunk's transfer is
    exposed. Ranks may hold different token counts.

    With `concurrent` (default) the chunks run on their own streams, chunk 0
    at the highest priority: its launches take the SMs first, and the later
    chunks' CTAs fill the gaps it leaves (each launch's ramp and drain, which
    at a few thousand rows per launch cost as much as a tenth of the step).
    Chunk 0 still finishes first, so its gather still overlaps the rest."""

    def __init__(self, prompts: Sequence[np.ndarray], plan: list, weights: Weights, device,
                 standins: Sequence[StandIns], layers: int, rank: int = 0, exact: bool = False, group=None,
                 concurrent: bool = True, device_trie: bool = True):
        """`plan` is shard.chunk_plan(prompts, world, chunks): this rank runs
        plan[rank]; chunk sizes may differ between ranks."""
        self.device, self.world, self.rank, self.group = device, len(plan), rank, group
        world = self.world
        self.layers = layers
        self.plan = plan
        self.parts = plan[rank]
        self.prompts = [[prompts[i] for i in part] for part in self.parts]
        self.all_prompts = prompts
        self.batches = [Batch.build(ps, device) for ps in self.prompts]
        self.pipes, self.send, self.direct = [], [], []
        r0 = 0
        for b in self.batches:
            pipe = Pipeline(b, weights, device, exact=exact)
            pipe.bind_layers([slice_standins(s, r0, b.rows) for s in standins], layers)
            self.pipes.append(pipe)
            self.send.append(torch.empty((b.tokens, HIDDEN), device=device))
            self.direct.append(identity_rows(b))
            r0 += b.rows
        self.rows = r0
        self.tokens = sum(b.tokens for b in self.batches)
        self.gather = None
        if world > 1:
            self.gather = FinalGather(chunk_tokens(prompts, plan), rank, HIDDEN, device, group=group)
        self._stage = HostStage(device, self.batches, on_device=device_trie)
        self._last_idx = None
        self.streams = None
        if concurrent and len(self.pipes) > 1:
            _, high = torch.cuda.Stream.priority_range()  # (lowest, highest): lower value = higher priority
            self.streams = [torch.cuda.Stream(device, priority=min(high + c, 0)) for c in range(len(self.pipes))]

    @staticmethod
    def rows_needed(prompts: Sequence[np.ndarray], parts: list) -> int:
        return sum(ops.prefix_trie([prompts[i] for i in part]).nodes for part in parts)

    def launches_per_step(self) -> int:
        return sum(launches_per_run(self.layers) + (0 if d else 1) for d in self.direct)

    def step(self, timers=None) -> None:
        """Enqueues the whole share (+ the transfers to rank 0) after the work
        already on the current stream; on return the current stream is
        ordered after every chunk and every transfer."""
        cur = torch.cuda.current_stream(self.device)
        works = []
        for c, pipe in enumerate(self.pipes):
            s = self.streams[c] if self.streams else cur
            if s is not cur:
                s.wait_stream(cur)
            with torch.cuda.stream(s):
                if self.direct[c]:
                    pipe.run(stream=s, timer=timers[c] if timers else None, final_out=self.send[c])
                else:
                    pipe.run(stream=s, timer=timers[c] if timers else None)
                    pipe.expand_to_tokens(self.send[c])
                if self.gather is not None:  # NCCL's stream waits for s
                    works += self.gather.post(c, self.send[c])
        if self.gather is not None:  # chunks other ranks hold beyond this rank's own
            for c in range(len(self.pipes), self.gather.chunks()):
                works += self.gather.post(c, None)
        if self.streams:
            for s in self.streams:
                cur.wait_stream(s)
        for w in works:  # cur waits for the collective's stream
            w.wait()
        self._stage.mark_used()

    def rebuild(self) -> int:
        """The host part of an end-to-end step: every chunk's trie from host
        token ids (HostStage: built on the device from the uploaded ids by
        default, else on the host); returns the H2D bytes."""
        nbytes = 0
        for c, (ps, b) in enumerate(zip(self.prompts, self._stage.upload_all(self.prompts))):
            if b.rows != self.pipes[c].shape.rows:
                raise ValueError("rebuild: the prompts' trie differs from the one the pipeline was sized for")
            self.pipes[c].batch = b
            self.batches[c] = b
            if self._stage.on_device:
                nbytes += (2 * len(ps) + 1 + b.tokens) * 4
            else:
                nbytes += sum(int(t.numel()) * 4 for t in (b.node_token, b.node_depth, b.token_node, b.last_rows))
        return nbytes

    def last_token_rows(self, out: torch.Tensor) -> None:
        """Rank 0, after step(): the final hidden state of every prompt's last
        token, for all ranks' prompts, in shard.gather_order(plan) order
        (asynchronous: the row indices were uploaded once)."""
        if self._last_idx is None:
            self._last_idx = []
            for c in range(max(len(p) for p in self.plan)):
                for r in range(self.world):
                    if c >= len(self.plan[r]):
                        continue
                    ends = np.cumsum([len(self.all_prompts[i]) for i in self.plan[r][c]]) - 1
                    self._last_idx.append((c, r, torch.from_numpy(ends.astype(np.int32)).to(self.device)))
        k = 0
        for c, r, idx in self._last_idx:
            src = self.send[c] if r == 0 else self.gather.rows(c, r)
            ops.gather_rows_gpu(src, idx, out[k:k + idx.numel()])
            k += idx.numel()

    def release(self) -> None:
        """Drops the receive buffers (before the process group is destroyed)."""
        self.gather = None


class StageTimer:
    """CUDA event pairs around every launch of one b2_prefill_layers call
    (layout of the events argument in include/aps2026_b200.h)."""

    STAGES = ("rope", "add_ln", "route", "silu")

    def __init__(self, layers: int, kinds=None):
        """`kinds` (default: all) limits the records to those launch kinds
        ('ln0', 'fused', 'rope', 'add_ln', 'route', 'silu'): an event
        between two launches also serialises them, so fewer records
        disturb the run less."""
        self.layers = layers
        self.kinds = set(kinds) if kinds is not None else {"ln0", "fused", *self.STAGES}
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(2 * (5 * layers + 1))]
        for e in self.events:  # materialise the driver events
            e.record()
        torch.cuda.synchronize()
        handles = [e.cuda_event for e in self.events]
        for pair in range(5 * layers + 1):
            if self._kind(pair) not in self.kinds:
                handles[2 * pair] = handles[2 * pair + 1] = None
        self._arr = (C.c_void_p * len(self.events))(*handles)

    def _kind(self, pair: int) -> str:
        L = self.layers
        if pair == 0:
            return "ln0"
        if pair <= L:
            return "fused"
        return self.STAGES[(pair - L - 1) % 4]

    def handles(self):
        return self._arr

    def _ms(self, pair: int) -> float:
        return self.events[2 * pair].elapsed_time(self.events[2 * pair + 1])

    def durations(self) -> dict:
        """ms per launch of each recorded kind after the run has completed:
        'ln0', 'fused' (layers 1..L-1 and the final step), and the four
        per-layer stages."""
        L = self.layers
        out = {"ln0": [self._ms(0)], "fused": [self._ms(l) for l in range(1, L + 1)]}
        for s, name in enumerate(self.STAGES):
            out[name] = [self._ms(L + 1 + 4 * l + s) for l in range(L)]
        return {k: v for k, v in out.items() if k in self.kinds}


# ---- algorithmic bytes (per trie-node row) ----------------------------------------------------


def bytes_per_row(layers: int = LAYERS, hidden=HIDDEN, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                  experts=EXPERTS, inter=INTER) -> dict:
    """Bytes each kernel of the pipeline must move per node row (each tensor
    read or written once):
      gather 2h*4; LN h*4*2; fused un-permute+add+LN: 2 expert rows + carry
      read, x + normed written = 5h*4 plus 2 route ids + 2 positions;
      RoPE 2*(q+k)*4; add+LN 4h*4; routing E*4 logits + 2 route ids + 2*4
      positions + 2*4 assignment rows; SiLU 2 assignments * inter * 12."""
    f = 4
    d = dict(
        gather=2 * hidden * f,
        ln0=2 * hidden * f,
        fused=5 * hidden * f + 2 + 2 * 4,
        rope=2 * (q_heads + kv_heads) * head_dim * f,
        add_ln=4 * hidden * f,
        route=experts * f + 2 + 2 * 4 + 2 * 4,
        silu=2 * inter * 3 * f,
    )
    d["total"] = (d["gather"] + d["ln0"] + layers * (d["rope"] + d["add_ln"] + d["route"] + d["silu"])
                  + layers * d["fused"])
    return d
