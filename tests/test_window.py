"""Shifted-window sparse self-attention (no reference implementation; the
config-3 SLat decoder's 8^3-window blocks).  Parity is against this repo's
own restatement in oracle/oracle.py:

- CPU: the full-grid partition (the C ABI's layout) agrees with the compact
  window_partition; a window that covers the whole grid reduces windowed
  attention to plain per-batch attention.
- GPU: p3d_window_partition bit-exact (perm and cu) against the oracle for
  shifts 0 and window/2, two batch items; p3d_window_attention within the
  north-star bound, with q/k/v as column views of one packed qkv buffer.
"""
import numpy as np
import pytest

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords, batched


def test_grid_partition_matches_compact_partition():
    c = batched(shell_coords(), 2)
    for shift in (0, 4):
        perm, cu = O.window_partition_grid(c, 2, 8, shift, (64, 64, 64))
        order, cc = O.window_partition(c, 8, shift)
        np.testing.assert_array_equal(perm, order)
        nz = np.r_[0, np.nonzero(np.diff(cu))[0] + 1]
        np.testing.assert_array_equal(cu[nz], cc)
        assert cu[-1] == c.shape[0] and np.diff(cu).max() <= 8 ** 3


def test_window_covering_grid_is_full_attention():
    rng = np.random.default_rng(3)
    c = batched(shell_coords(16, 5.0, 1.0), 2)
    n, H = c.shape[0], 2
    q, k, v = (rng.standard_normal((n, H * 64)).astype(np.float32) for _ in range(3))
    got = O.window_attention(q, k, v, c, 16, 0, H, 64, 0.125)
    cu = np.array([0, int((c[:, 0] == 0).sum()), n], np.int32)
    exp = O.varlen_attention(q, k, v, cu, cu, H, 64, 0.125)
    np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("shift", [0, 4])
def test_window_partition_bitexact(shift):
    import torch
    from pixal3d.cpp_b200 import ops
    c = batched(shell_coords(), 2)
    perm, cu = ops.window_partition(torch.from_numpy(c).cuda(), 2, 8, shift, (64, 64, 64))
    ep, ecu = O.window_partition_grid(c, 2, 8, shift, (64, 64, 64))
    np.testing.assert_array_equal(cu.cpu().numpy(), ecu)
    np.testing.assert_array_equal(perm.cpu().numpy(), ep)


@pytest.mark.gpu
@pytest.mark.parametrize("shift,dtype", [(0, "f16"), (4, "f16"), (4, "bf16")])
def test_window_attention_matches_oracle(shift, dtype):
    import torch
    from pixal3d.cpp_b200 import ops
    rng = np.random.default_rng(40 + shift)
    c = batched(shell_coords(32, 12.0, 1.5), 2)
    n, H = c.shape[0], 4
    C = H * 64
    qkv = rng.standard_normal((n, 3 * C)).astype(np.float32)
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    t = torch.from_numpy(qkv).cuda().to(td)
    r = t.float().cpu().numpy()
    coords = torch.from_numpy(c).cuda()
    perm, cu = ops.window_partition(coords, 2, 8, shift, (32, 32, 32))
    got = ops.window_attention(t[:, :C], t[:, C:2 * C], t[:, 2 * C:], perm, cu, 8, H, 0.125).float().cpu().numpy()
    exp = O.window_attention(r[:, :C], r[:, C:2 * C], r[:, 2 * C:], c, 8, shift, H, 64, 0.125)
    err = np.abs(got - exp)
    rel = float(np.linalg.norm(got - exp) / np.linalg.norm(exp))
    assert float(err.max()) <= 2e-2 and rel <= 5e-3, (float(err.max()), rel)
