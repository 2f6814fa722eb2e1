"""The prefill harness's files on the CPU: b2_read_inputs and b2_write_outputs
(host-memory logits) against the reference's own read_inputs / write_outputs
(src/main.cpp:144-192, built from its sources by oracle/Makefile into
oracle/_ref/libio_ref.so) and against the oracle's numpy restatement of the
two formats. Output files must be identical byte for byte; the reader must
return the same prompts and fail on the same malformed files with the same
messages, in the same order of checks."""
import ctypes as C

import numpy as np
import pytest

import oracle
from aps2026_b200 import _lib, ops
from tests._util import normal, rng

needs_ref = pytest.mark.skipif(not oracle.io_ref_available(), reason="reference I/O harness not built")


def _ref_write(path, logits):
    a = np.ascontiguousarray(logits, dtype=np.float32)
    rc = oracle.io_ref().io_ref_write_outputs(str(path).encode(), a.ctypes.data if a.size else None, *a.shape)
    assert rc == 0, oracle.io_ref().io_ref_error().decode()


def _ref_read(path):
    """(prompts, max_seq) from the reference reader, or its error message."""
    h = oracle.io_ref()
    b, m, t = C.c_uint32(0), C.c_uint32(0), C.c_size_t(0)
    lens = np.zeros(4096, np.uint32)
    ids = np.zeros(1 << 20, np.int32)
    rc = h.io_ref_read_inputs(str(path).encode(), C.addressof(b), C.addressof(m), C.addressof(t),
                              lens.ctypes.data, lens.size, ids.ctypes.data, ids.size)
    if rc != 0:
        return h.io_ref_error().decode()
    ends = np.cumsum(lens[: b.value], dtype=np.int64)
    return [ids[e - n:e].tolist() for n, e in zip(lens[: b.value].tolist(), ends.tolist())], m.value


@pytest.mark.parametrize("batch,vocab", [(64, 32064), (3, 5), (1, 1), (0, 7), (2, 1048577)])
def test_write_outputs_host(tmp_path, batch, vocab):
    g = rng(91)
    logits = normal(g, (batch, vocab))
    if logits.size:
        logits.flat[:: max(1, logits.size // 7)] = [np.nan, np.inf, -np.inf, -0.0, 1e-45, 3e38, 0.0][
            : len(logits.flat[:: max(1, logits.size // 7)])]
    path = tmp_path / "outputs.bin"
    ops.write_outputs(path, logits)
    got = path.read_bytes()
    assert got == oracle.outputs_bytes(logits)
    if oracle.io_ref_available():
        ref_path = tmp_path / "outputs_ref.bin"
        _ref_write(ref_path, logits)
        assert got == ref_path.read_bytes()


def test_write_outputs_overwrites(tmp_path):
    path = tmp_path / "o.bin"
    path.write_bytes(b"\xff" * 1000)
    ops.write_outputs(path, np.ones((2, 3), np.float32))
    assert path.read_bytes() == oracle.outputs_bytes(np.ones((2, 3), np.float32))


def test_write_outputs_errors(tmp_path):
    L = _lib.lib()
    bad = str(tmp_path / "no_such_dir" / "o.bin")
    buf = np.zeros(6, np.float32)
    assert L.b2_write_outputs(bad.encode(), buf.ctypes.data, 2, 3, 0, None) == _lib.B2_ERR_IO
    assert _lib.last_error() == f"cannot open output: {bad}"
    with pytest.raises(ops.FileError, match="cannot open output"):
        ops.write_outputs(bad, buf.reshape(2, 3))
    ok = str(tmp_path / "o.bin").encode()
    assert L.b2_write_outputs(None, buf.ctypes.data, 2, 3, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_write_outputs(ok, None, 2, 3, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_write_outputs(ok, buf.ctypes.data, 1 << 32, 1, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_write_outputs(ok, buf.ctypes.data, 1, 1 << 32, 0, None) == _lib.B2_ERR_INVALID_ARGUMENT
    # a full device fails the write with the reference's message
    assert L.b2_write_outputs(b"/dev/full", buf.ctypes.data, 2, 3, 0, None) == _lib.B2_ERR_IO
    assert _lib.last_error() == "failed while writing output: /dev/full"


def _prompts(g, batch, lo, hi, vocab=32064):
    return [g.integers(0, vocab, int(g.integers(lo, hi + 1))).astype(np.int32).tolist() for _ in range(batch)]


@pytest.mark.parametrize("batch,lo,hi", [(64, 2048, 2048), (17, 1, 300), (1, 1, 1), (3, 4096, 4096)])
def test_read_inputs(tmp_path, batch, lo, hi):
    g = rng(92 + batch)
    prompts = _prompts(g, batch, lo, hi)
    prompts[0][0] = -5  # ids are returned as stored; the trie checks the vocabulary
    path = tmp_path / "inputs.bin"
    data = oracle.inputs_bytes(prompts, max_seq_len=max(map(len, prompts)) + (batch % 3))
    path.write_bytes(data + b"\x01\x02\x03")  # trailing bytes are ignored
    got = ops.read_inputs(path)
    want, want_m = oracle.parse_inputs(path.read_bytes())
    assert got.prompts() == want == prompts
    assert got.max_seq_len == want_m
    assert got.ids.dtype == np.int32 and got.seq_lens.dtype == np.uint32
    if oracle.io_ref_available():
        assert _ref_read(path) == (want, want_m)


def _malformed():
    """(name, file bytes) of each way the reference's reader rejects a file."""
    u32 = lambda *v: np.array(v, dtype="<u4").tobytes()  # noqa: E731
    i32 = lambda *v: np.array(v, dtype="<i4").tobytes()  # noqa: E731
    return [
        ("empty", b""),
        ("half_header", u32(1)),
        ("header_7_bytes", u32(1) + b"\x04\x00\x00"),
        ("batch_0", u32(0, 4)),
        ("max_seq_0", u32(1, 0)),
        ("max_seq_above_4096", u32(1, 4097)),
        ("no_length", u32(1, 4)),
        ("length_cut", u32(1, 4) + b"\x02\x00"),
        ("length_0", u32(1, 4) + u32(0)),
        ("length_above_max_seq", u32(1, 4) + u32(5) + i32(1, 2, 3, 4, 5)),
        ("ids_cut", u32(1, 4) + u32(3) + i32(1, 2)),
        ("ids_cut_mid_word", u32(1, 4) + u32(2) + i32(7) + b"\x01"),
        ("second_prompt_missing", u32(2, 4) + u32(1) + i32(9)),
        ("second_prompt_cut", u32(2, 4) + u32(1) + i32(9) + u32(4) + i32(1, 2, 3)),
        ("header_batch_large", u32(1000, 4) + u32(1) + i32(9)),
    ]


@pytest.mark.parametrize("name,data", _malformed(), ids=[m[0] for m in _malformed()])
def test_read_inputs_rejects(tmp_path, name, data):
    path = tmp_path / f"{name}.bin"
    path.write_bytes(data)
    with pytest.raises(RuntimeError) as e:
        oracle.parse_inputs(data)
    want = str(e.value)
    with pytest.raises(ops.FileError) as got:
        ops.read_inputs(path)
    assert str(got.value) == f"read_inputs: {want}"
    if oracle.io_ref_available():
        assert _ref_read(path) == want


@needs_ref
def test_read_inputs_missing_file(tmp_path):
    path = tmp_path / "absent.bin"
    with pytest.raises(ops.FileError) as got:
        ops.read_inputs(path)
    assert str(got.value) == f"read_inputs: {_ref_read(path)}" == f"read_inputs: cannot open input: {path}"


def test_read_inputs_size_query_and_capacity(tmp_path):
    prompts = [[1, 2, 3], [4], [5, 6]]
    path = tmp_path / "in.bin"
    path.write_bytes(oracle.inputs_bytes(prompts))
    L = _lib.lib()
    b, m, t = C.c_uint32(0), C.c_uint32(0), C.c_size_t(0)
    raw = str(path).encode()
    assert L.b2_read_inputs(raw, 4096, C.addressof(b), C.addressof(m), C.addressof(t), None, 0, None, 0) == 0
    assert (b.value, m.value, t.value) == (3, 3, 6)
    lens, ids = np.zeros(3, np.uint32), np.zeros(6, np.int32)
    assert L.b2_read_inputs(raw, 4096, None, None, None, lens.ctypes.data, 2, ids.ctypes.data, 6) \
        == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_read_inputs(raw, 4096, None, None, None, lens.ctypes.data, 3, ids.ctypes.data, 5) \
        == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_read_inputs(raw, 4096, None, None, None, lens.ctypes.data, 3, None, 6) \
        == _lib.B2_ERR_INVALID_ARGUMENT
    assert L.b2_read_inputs(raw, 4096, None, None, None, lens.ctypes.data, 3, ids.ctypes.data, 6) == 0
    assert lens.tolist() == [3, 1, 2] and ids.tolist() == [1, 2, 3, 4, 5, 6]
    # max_len is the caller's MAX_POSITION_EMBEDDINGS
    assert L.b2_read_inputs(raw, 2, None, None, None, None, 0, None, 0) == _lib.B2_ERR_IO
    assert _lib.last_error() == "invalid input header"


def test_read_inputs_feeds_the_trie(tmp_path):
    g = rng(95)
    shared = g.integers(0, 32064, 40).tolist()
    prompts = [shared + g.integers(0, 32064, int(n)).tolist() for n in (5, 0, 17, 3)]
    path = tmp_path / "in.bin"
    path.write_bytes(oracle.inputs_bytes(prompts))
    batch = ops.read_inputs(path)
    got = ops.prefix_trie(batch.prompts())
    want = oracle.prefix_trie(prompts, with_ancestors=False)
    assert got.nodes == want["nodes"]
    oracle.assert_bitexact(got.token_node, want["token_node"], "token_node")
