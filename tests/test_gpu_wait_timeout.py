"""The failure path of the kernels' bounded waits, driven to expiry on the GPU.

Every mbarrier wait of the library's pipelines gives up after a limit,
latches P3D_ERR_TIMEOUT in the context's device flag and lets the kernel
return, so a stuck pipeline reports an error instead of hanging the GPU.
p3d_wait_selftest runs that same wait routine with a short limit on a barrier
phase that nothing completes (and, as the control, on one that another warp
completes).  The test checks the latched status, that the wait lasted about
its limit, and that the context keeps working afterwards.  No fault, trap or
hang is involved: the waiting thread simply stops waiting.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000  # 50 ms


def _selftest(complete: int):
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    c = ops.ctx(0)
    out = (ctypes.c_int64 * 2)()
    rc = L.lib.p3d_wait_selftest(c.h, complete, LIMIT_NS, out)
    return rc, int(out[0]), int(out[1]), L.lib.p3d_last_error(c.h).decode()


def test_completed_wait_succeeds():
    rc, ok, ns, _ = _selftest(1)
    assert rc == 0 and ok == 1
    assert ns < LIMIT_NS


def test_expired_wait_latches_timeout_and_context_survives():
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    rc, ok, ns, msg = _selftest(0)
    assert rc == L.P3D_ERR_TIMEOUT, (rc, msg)
    assert "timed out" in msg
    assert ok == 0
    assert LIMIT_NS <= ns < LIMIT_NS + 1_000_000_000, ns  # gave up after about its limit
    # the flag was reported once and cleared; the context runs kernels again
    ops.ctx(0).sync_check()
    c = shell_coords(16, 5.0, 1.0)
    got = ops.neighbor_map27(torch.from_numpy(c).cuda()).cpu().numpy()
    ops.ctx(0).sync_check()
    np.testing.assert_array_equal(got, O.neighbor_map27(c))
    rc2, ok2, _, _ = _selftest(1)
    assert rc2 == 0 and ok2 == 1
