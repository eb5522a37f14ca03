"""GPU check of p3d_neighbor_map27_static, the neighbour map whose hash table
is a file-scope device array (no allocation in the call).

Called through the C ABI and compared bit for bit (integer output) with
p3d_neighbor_map27_ws on two calls in a row: a larger coordinate set, then a
smaller one, so stale keys of the first call would show in the second.  A
third case fills the table to its limit (exactly P3D_NBR_STATIC_MAX_POINTS
points, where the key slots reach the values region), and a fourth checks
that a call leaves the device's free memory unchanged.
Runs alone in a fresh process or after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from pixal3d.cpp_b200.workloads import shell_coords, batched

pytestmark = pytest.mark.gpu

MAX_POINTS = 524288  # P3D_NBR_STATIC_MAX_POINTS


def _ws_map(lib, c, coords):
    n = coords.shape[0]
    ws_bytes = int(lib.p3d_neighbor_map27_workspace(n))
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=coords.device)
    base = ws.data_ptr()
    aligned = (base + 255) // 256 * 256
    out = torch.empty((27, n), dtype=torch.int32, device=coords.device)
    c.check(lib.p3d_neighbor_map27_ws(c.h, ctypes.c_void_p(coords.data_ptr()), n, ctypes.c_void_p(aligned),
                                      ws_bytes, ctypes.c_void_p(out.data_ptr())))
    return out


def _static_map(lib, c, coords):
    n = coords.shape[0]
    out = torch.full((27, n), -7, dtype=torch.int32, device=coords.device)
    c.check(lib.p3d_neighbor_map27_static(c.h, ctypes.c_void_p(coords.data_ptr()), n,
                                          ctypes.c_void_p(out.data_ptr())))
    return out


def test_neighbor_map_static_matches_ws_twice():
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    lib = L.lib
    c = ops.ctx(0)
    dev = torch.device("cuda", 0)
    sets = [batched(shell_coords(), 2), shell_coords(40, 13.0, 1.3)]
    for i, cs in enumerate(sets):
        coords = torch.from_numpy(np.ascontiguousarray(cs)).to(dev)
        got = _static_map(lib, c, coords)
        exp = _ws_map(lib, c, coords)
        torch.cuda.synchronize()
        c.sync_check()
        n = cs.shape[0]
        assert int((exp < n).sum()) > n, "degenerate case: no neighbours found"
        assert torch.equal(got, exp), f"call {i}: static-table map differs from the workspace map (n={n})"


def test_neighbor_map_static_at_max_points():
    """n = 524,288: a dense 64 x 64 x 128 block (every interior point has all
    27 neighbours), so the table's 2^20 slots are all in use."""
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    c = ops.ctx(0)
    g = np.stack(np.meshgrid(np.arange(64), np.arange(64), np.arange(128), indexing="ij"), -1).reshape(-1, 3)
    cs = np.concatenate([np.zeros((g.shape[0], 1), np.int32), g.astype(np.int32)], axis=1)
    assert cs.shape[0] == MAX_POINTS
    coords = torch.from_numpy(np.ascontiguousarray(cs)).cuda()
    got = _static_map(L.lib, c, coords)
    exp = _ws_map(L.lib, c, coords)
    torch.cuda.synchronize()
    c.sync_check()
    # per axis of length L, (3L - 2) (point, offset) pairs stay inside the box
    assert int((exp < MAX_POINTS).sum()) == (3 * 64 - 2) * (3 * 64 - 2) * (3 * 128 - 2)
    assert bool((exp[:, 1 * 64 * 128 + 1 * 128 + 1] < MAX_POINTS).all()), "interior point lacks a neighbour"
    assert torch.equal(got, exp), "static-table map differs from the workspace map at the maximum size"


def test_neighbor_map_static_allocates_nothing():
    """After a first call (which may load device code), a second call leaves
    the device's free memory and torch's allocation unchanged."""
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    c = ops.ctx(0)
    coords = torch.from_numpy(np.ascontiguousarray(batched(shell_coords(), 2))).cuda()
    out = torch.empty((27, coords.shape[0]), dtype=torch.int32, device="cuda")

    def call():
        c.check(L.lib.p3d_neighbor_map27_static(c.h, ctypes.c_void_p(coords.data_ptr()), coords.shape[0],
                                                ctypes.c_void_p(out.data_ptr())))
        torch.cuda.synchronize()

    call()
    free0, _ = torch.cuda.mem_get_info(0)
    alloc0 = torch.cuda.memory_allocated(0)
    call()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    assert torch.cuda.memory_allocated(0) == alloc0
    c.sync_check()


def test_neighbor_map_static_rejects_oversize():
    from pixal3d.cpp_b200 import _lib as L
    from pixal3d.cpp_b200 import ops
    c = ops.ctx(0)
    coords = torch.zeros((1, 4), dtype=torch.int32, device="cuda")
    out = torch.zeros((27, 1), dtype=torch.int32, device="cuda")
    rc = L.lib.p3d_neighbor_map27_static(c.h, ctypes.c_void_p(coords.data_ptr()), MAX_POINTS + 1,
                                         ctypes.c_void_p(out.data_ptr()))
    assert rc == 1  # P3D_ERR_INVALID, checked on the host before any launch
    assert "maximum of 524288" in L.lib.p3d_last_error(c.h).decode()
