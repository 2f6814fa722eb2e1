"""b2_moe_route_noalloc: routing for callers that cannot allocate device
memory (their host framework owns every allocation, or they must not call
cudaMalloc because it can synchronize the device). Its scratch is a fixed
array inside the library, so it takes no workspace argument.

Called through the C ABI and checked against b2_moe_route (caller
workspace) on the same logits: the outputs are integer indices, so they must
agree bit for bit -- on calls in a row, each smaller than the one before, so
stale scratch contents from the earlier calls are exercised. The cases reach
every padded expert width of the histogram reduction (E' = 4, 16, 32) and
the largest size the fixed scratch accepts (524,288 tokens at E = 16); one
case is also checked against the CPU oracle. This file is collected last on
purpose."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _route(lib, fn_name, logits, ws=None):
    import torch

    from aps2026_b200 import ops

    T, E = logits.shape
    out = ops.alloc_routing(T, E, logits.device)
    for t in (out.counts, out.offsets, out.assignment_rows, out.route_positions, out.work_expert64,
              out.work_start64, out.work_expert128, out.work_start128):
        t.fill_(-7)
    ptrs = [out.routes.data_ptr(), out.counts.data_ptr(), out.offsets.data_ptr(), out.assignment_rows.data_ptr(),
            out.route_positions.data_ptr(), out.work_expert64.data_ptr(), out.work_start64.data_ptr(),
            out.work_expert128.data_ptr(), out.work_start128.data_ptr()]
    stream = torch.cuda.current_stream().cuda_stream
    if ws is None:
        rc = getattr(lib, fn_name)(logits.data_ptr(), T, E, 1e-3, 2e-2, *ptrs, stream)
    else:
        rc = getattr(lib, fn_name)(logits.data_ptr(), T, E, 1e-3, 2e-2, *ptrs, ws.buf.data_ptr(), ws.bytes, stream)
    torch.cuda.synchronize()
    return rc, out


def test_noalloc_route_matches_workspace_route_twice(cuda):
    import torch

    import oracle
    from aps2026_b200 import _lib, ops

    lib = _lib.lib()
    g = np.random.default_rng(77)
    # largest first: 524,288 tokens at E = 16 fill the fixed scratch exactly
    # (2048 tiles x 16 words); E = 32 and E = 3 take the E' = 32 and E' = 4
    # histogram paths
    for T, E in ((524_288, 16), (100_003, 16), (70_001, 32), (5_000, 3), (3_000, 13)):
        logits = torch.from_numpy(g.standard_normal((T, E)).astype(np.float32)).to(cuda)
        rc_a, a = _route(lib, "b2_moe_route_noalloc", logits)
        assert rc_a == 0, _lib.last_error()
        rc_b, b = _route(lib, "b2_moe_route", logits, ops.RouteWorkspace(T, E, cuda))
        assert rc_b == 0, _lib.last_error()
        for name in ("routes", "counts", "offsets", "assignment_rows", "route_positions", "work_expert64",
                     "work_start64", "work_expert128", "work_start128"):
            assert torch.equal(getattr(a, name), getattr(b, name)), f"T={T} E={E}: {name} differs"
        if (T, E) == (5_000, 3):
            want = oracle.moe_route(logits.cpu().numpy())
            for name in ("assignment_rows", "route_positions"):
                assert np.array_equal(getattr(a, name).cpu().numpy().view(np.uint32), want[name]), name


def test_noalloc_route_rejects_sizes_beyond_its_scratch(cuda):
    import torch

    from aps2026_b200 import _lib

    lib = _lib.lib()
    T, E = 524_288 + 1, 16  # one tile more than the fixed scratch holds at E = 16
    logits = torch.zeros((T, E), device=cuda)
    rc, _ = _route(lib, "b2_moe_route_noalloc", logits)
    assert rc == _lib.B2_ERR_UNSUPPORTED
    assert "fixed scratch" in _lib.last_error()
