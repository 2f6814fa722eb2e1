"""Drop-in run helpers (test infrastructure).

write_model(): a synthetic model.bin in the reference's loader format
(src/model_loader.cu:13-30: u32 count; per tensor u32 name length, name,
u32 ndim, u32 dims, u64 file offset, u64 bytes; then the float32 data) with
every tensor name PhiTinyMoEModel loads (src/model.cu:10-18, src/layer.cu).
The 32 layers' entries all point at ONE set of layer weights (the loader
reads each entry by its offset, so names may share data): a 1.5 GB file
instead of 15 GB. Weights are seeded N(0, 1/fan_in) so that every
projection, the router logits and the attention scores are O(1).

``python tests/_dropin.py <library> <model.bin> <out.npz>`` loads one of
oracle/_ref/libdropin_{ref,b2}.so in this process, runs the reference's
generate on PROMPTS and forward on FORWARD_PROMPT, and saves the logits and
wall times. Each library runs in its own process (both export the same
names and carry their own CUDA runtime).
"""
from __future__ import annotations

import ctypes as C
import struct
import sys
import time

import numpy as np

HIDDEN, VOCAB, LAYERS = 4096, 32064, 32
Q_DIM, KV_DIM, EXPERTS, INTER = 16 * 128, 4 * 128, 16, 448


def _tensors():
    """(name, shape, std, mean, shared-key) for every tensor the model loads."""
    out = [("model.embed_tokens.weight", (VOCAB, HIDDEN), 1.0, 0.0, "emb"),
           ("model.norm.weight", (HIDDEN,), 0.1, 1.0, "norm_w"),
           ("model.norm.bias", (HIDDEN,), 0.1, 0.0, "norm_b"),
           ("lm_head.weight", (VOCAB, HIDDEN), HIDDEN ** -0.5, 0.0, "lm_w"),
           ("lm_head.bias", (VOCAB,), 0.02, 0.0, "lm_b")]
    layer = [("input_layernorm.weight", (HIDDEN,), 0.1, 1.0),
             ("input_layernorm.bias", (HIDDEN,), 0.1, 0.0),
             ("post_attention_layernorm.weight", (HIDDEN,), 0.1, 1.0),
             ("post_attention_layernorm.bias", (HIDDEN,), 0.1, 0.0)]
    for proj, rows, cols in (("q", Q_DIM, HIDDEN), ("k", KV_DIM, HIDDEN), ("v", KV_DIM, HIDDEN),
                             ("o", HIDDEN, Q_DIM)):
        layer.append((f"self_attn.{proj}_proj.weight", (rows, cols), cols ** -0.5, 0.0))
        layer.append((f"self_attn.{proj}_proj.bias", (rows,), 0.02, 0.0))
    layer.append(("block_sparse_moe.gate.weight", (EXPERTS, HIDDEN), HIDDEN ** -0.5, 0.0))
    for e in range(EXPERTS):
        for w, shape in (("w1", (INTER, HIDDEN)), ("w2", (HIDDEN, INTER)), ("w3", (INTER, HIDDEN))):
            layer.append((f"block_sparse_moe.experts.{e}.{w}.weight", shape, shape[1] ** -0.5, 0.0))
    for i in range(LAYERS):
        for name, shape, std, mean in layer:
            out.append((f"model.layers.{i}.{name}", shape, std, mean, name))
    return out


def write_model(path, seed: int = 0) -> None:
    entries = _tensors()
    header = 4 + sum(4 + len(n) + 4 + 4 * len(s) + 16 for n, s, *_ in entries)
    g = np.random.default_rng(seed)
    blobs, where, offset = [], {}, header
    for _name, shape, std, mean, key in entries:
        if key in where:
            continue
        a = g.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)
        where[key] = offset
        blobs.append(a)
        offset += a.nbytes
    with open(path, "wb") as f:
        f.write(struct.pack("<I", len(entries)))
        for name, shape, _std, _mean, key in entries:
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape)))
            f.write(struct.pack(f"<{len(shape)}I", *shape))
            f.write(struct.pack("<QQ", where[key], 4 * int(np.prod(shape))))
        assert f.tell() == header
        for a in blobs:
            f.write(a.tobytes())


def prompts(seed: int = 5):
    """Five prompts with shared prefixes (one prompt a strict prefix of
    another, one repeated), so the trie dedups rows."""
    g = np.random.default_rng(seed)
    a = g.integers(0, VOCAB, 40)
    b = np.concatenate([a[:12], g.integers(0, VOCAB, 21)])
    c = a[:17].copy()
    d = g.integers(0, VOCAB, 9)
    return [a, b, c, d, a.copy()]


FORWARD_PROMPT_SEED = 6


def forward_prompt():
    return np.random.default_rng(FORWARD_PROMPT_SEED).integers(0, VOCAB, 37)


def _step(msg: str) -> None:
    print(f"[dropin] {msg}", file=sys.stderr, flush=True)


def _run(lib_path: str, model_path: str, out_path: str) -> None:
    lib = C.CDLL(lib_path)
    lib.dropin_error.restype = C.c_char_p
    lib.dropin_load.restype = C.c_void_p
    lib.dropin_load.argtypes = [C.c_char_p]
    lib.dropin_free.argtypes = [C.c_void_p]
    lib.dropin_generate.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                    C.POINTER(C.c_double)]
    lib.dropin_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_double)]
    t0 = time.time()
    model = lib.dropin_load(model_path.encode())
    if not model:
        raise RuntimeError(f"dropin_load: {lib.dropin_error().decode()}")
    load_s = time.time() - t0
    _step(f"loaded in {load_s:.1f} s")
    ps = prompts()
    ids = np.concatenate(ps).astype(np.int32)
    offs = np.zeros(len(ps) + 1, np.int32)
    offs[1:] = np.cumsum([len(p) for p in ps])
    gen = np.empty((len(ps), VOCAB), np.float32)
    times, first = [], None
    repeatable = True
    for _ in range(3):  # the first call includes one-time setup (tables, scratch)
        ms = C.c_double()
        rc = lib.dropin_generate(model, ids.ctypes.data, offs.ctypes.data, len(ps), gen.ctypes.data, C.byref(ms))
        if rc != 0:
            raise RuntimeError(f"dropin_generate rc={rc}: {lib.dropin_error().decode()}")
        times.append(ms.value)
        _step(f"generate {ms.value:.1f} ms")
        if first is None:
            first = gen.copy()
        repeatable &= bool(np.array_equal(first.view(np.uint32), gen.view(np.uint32)))
    fp = forward_prompt().astype(np.int32)
    fwd = np.empty(VOCAB, np.float32)
    ms = C.c_double()
    rc = lib.dropin_forward(model, fp.ctypes.data, len(fp), fwd.ctypes.data, C.byref(ms))
    if rc != 0:
        raise RuntimeError(f"dropin_forward rc={rc}: {lib.dropin_error().decode()}")
    _step(f"forward {ms.value:.1f} ms")
    # the packed ops of forward's GPU branch one by one, on seeded inputs
    lib.dropin_packed_attention.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_void_p]
    lib.dropin_add_inplace.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
    g = np.random.default_rng(7)
    lens = np.array([37, 5, 64], np.uint64)
    rows = int(lens.sum())
    pq = g.standard_normal((rows, Q_DIM), dtype=np.float32)
    pk = g.standard_normal((rows, KV_DIM), dtype=np.float32)
    pv = g.standard_normal((rows, KV_DIM), dtype=np.float32)
    pout = np.empty_like(pq)
    rc = lib.dropin_packed_attention(pq.ctypes.data, pk.ctypes.data, pv.ctypes.data, lens.ctypes.data, len(lens),
                                     pout.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"dropin_packed_attention rc={rc}: {lib.dropin_error().decode()}")
    aa = g.standard_normal(rows * HIDDEN, dtype=np.float32)
    ab = g.standard_normal(rows * HIDDEN, dtype=np.float32)
    rc = lib.dropin_add_inplace(aa.ctypes.data, ab.ctypes.data, aa.size)
    if rc != 0:
        raise RuntimeError(f"dropin_add_inplace rc={rc}: {lib.dropin_error().decode()}")
    _step("packed ops")
    # error behaviour: an empty prompt and an out-of-vocabulary token
    errs = []
    bad = [(np.zeros(1, np.int32), np.array([0, 0], np.int32)),
           (np.array([1, VOCAB], np.int32), np.array([0, 2], np.int32))]
    for bid, boff in bad:
        rc = lib.dropin_generate(model, bid.ctypes.data, boff.ctypes.data, 1, gen[:1].ctypes.data, None)
        errs.append(f"{rc}:{lib.dropin_error().decode()}")
    _step("errors checked")
    lib.dropin_free(C.c_void_p(model))
    _step("model freed")
    np.savez(out_path, generate=gen, forward=fwd, generate_ms=np.array(times), forward_ms=np.array([ms.value]),
             load_s=np.array([load_s]), errors=np.array(errs), repeatable=np.array([repeatable]),
             rope_q=pq, rope_k=pk, attention=pout, add=aa)


if __name__ == "__main__":
    import faulthandler
    import os

    faulthandler.enable()
    _run(sys.argv[1], sys.argv[2], sys.argv[3])
    _step("saved")
    # The unmodified reference library ends the process with SIGSEGV during
    # native static teardown at exit (its function-local device scratch is
    # destroyed after all work and after the results above were written);
    # leave without running the library's exit-time destructors.
    os._exit(0)
