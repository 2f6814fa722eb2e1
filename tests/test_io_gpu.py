"""b2_write_outputs from device memory: the file must be byte for byte the
one the reference's write_outputs (src/main.cpp:183-192) makes of the same
logits -- checked against the oracle's restatement of the format and, where
it was built, the reference's own writer. The logits come from a kernel
still running on a side stream when the call is made, so the copies must
order themselves after it; sizes cover one staging chunk, several full
chunks with a ragged last one, and an empty matrix."""
import pytest

import oracle
from aps2026_b200 import ops
from tests._util import normal, rng, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,vocab", [(64, 32064), (3, 5), (5, 1048583), (0, 32064)])
def test_write_outputs_device(tmp_path, cuda, batch, vocab):
    import torch

    g = rng(96)
    xh, yh = normal(g, (batch, vocab)), normal(g, (batch, vocab))
    logits, y = to_dev(xh, cuda), to_dev(yh, cuda)
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    path = tmp_path / "outputs.bin"
    with torch.cuda.stream(side):
        if batch:
            ops.add_inplace_gpu(logits, y)
        ops.write_outputs(path, logits)  # enqueued behind the add on `side`
    side.synchronize()
    host = to_host(logits)
    got = path.read_bytes()
    assert len(got) == 8 + 4 * batch * vocab
    assert got == oracle.outputs_bytes(host)
    assert got == oracle.outputs_bytes(oracle.add(xh, yh))  # the add's result, not its input
    if oracle.io_ref_available() and batch:
        ref_path = tmp_path / "outputs_ref.bin"
        rc = oracle.io_ref().io_ref_write_outputs(str(ref_path).encode(), host.ctypes.data, batch, vocab)
        assert rc == 0
        assert got == ref_path.read_bytes()
