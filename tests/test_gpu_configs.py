"""GPU parity at the BASELINE configurations' full sizes.

- The config-2 fine-level sparse conv (C = 1024 -> 1024, 43,532 rows, rows
  sorted by neighbour pattern, tile taps skipped: the dominant kernel as the
  flow runs it) against the numpy oracle on sampled rows and against a torch
  fp32 computation of every row, on the same f16-rounded operands.
- One config-1 sparse transformer block at N = 21,766 (C = 1024, 16 heads,
  1,029 condition tokens, t = 0.5) against the oracle's committed golden.
- One full config-2 SLat-flow forward (CFG batch 2 x 21,766 voxels, io
  resblocks, 24 blocks) against the oracle's committed golden.

The goldens come from tests/golden/make_golden.py --only configs (the oracle
on the CPU, inputs from tests/_configs.py).  Feature tolerance: the
north-star bound after one full SLat-flow forward, max-abs 2e-2 and
relative-L2 5e-3; integer outputs bit-exact.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests import _configs as K
from tests._fixtures import GOLDEN

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 5e-3


def errors(a, e):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    return float(np.abs(a - e).max()), float(np.linalg.norm(a - e) / np.linalg.norm(e))


def check(a, e, what, max_abs=MAX_ABS, rel_l2=REL_L2):
    mx, rl = errors(a, e)
    print(f"{what}: max_abs {mx:.3e} rel_l2 {rl:.3e}", flush=True)
    assert mx <= max_abs and rl <= rel_l2, f"{what}: max_abs {mx:.3e} (<= {max_abs}) rel_l2 {rl:.3e} (<= {rel_l2})"


def test_conv1024_fine_level_sorted_tap_skip():
    from pixal3d.cpp_b200 import ops
    cs, nbr, x, w, b = K.conv1024()
    n = cs.shape[0]
    dev = torch.device("cuda", 0)
    nbr_d = ops.neighbor_map27(torch.from_numpy(cs).to(dev))
    np.testing.assert_array_equal(nbr_d.cpu().numpy(), nbr)  # neighbour map bit-exact at full size
    taps = ops.conv_tile_taps(nbr_d)
    used = sum(bin(int(t)).count("1") for t in taps.cpu().numpy().astype(np.uint32))
    assert used < 27 * taps.numel(), "no tap is skipped: the test would not exercise skipping"
    x16 = torch.from_numpy(x).to(dev).to(torch.float16)
    w16 = torch.from_numpy(w).to(dev).to(torch.float16)
    bd = torch.from_numpy(b).to(dev)
    out_skip = torch.empty((n, K.C), device=dev)
    out_all = torch.empty((n, K.C), device=dev)
    ops.subm_conv3d(x16, nbr_d, w16, bd, out=out_skip, tile_taps=taps)
    ops.subm_conv3d(x16, nbr_d, w16, bd, out=out_all)
    torch.cuda.synchronize()
    ops.ctx(0).sync_check()
    # skipping taps whose gathered rows are all zero adds only zeros; the two
    # runs differ only in the last wave's tiles, which the split schedule cuts
    # at other steps (f32 partial sums added in another order)
    check(out_skip.cpu().numpy(), out_all.cpu().numpy(), "conv1024 tap skip vs all taps", max_abs=1e-3, rel_l2=1e-5)
    # the oracle on sampled rows (same f16-rounded operands, f32 math)
    rows = K.sample_rows(n, 512, seed=7)
    exp_rows = K.conv_rows(nbr, x, w, b, rows)
    check(out_skip[torch.from_numpy(rows).to(dev)].cpu().numpy(), exp_rows, "conv1024 sampled rows vs oracle",
          max_abs=1e-3, rel_l2=1e-4)
    # every row against torch fp32 (no TF32) on the same operands
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xz = torch.cat([x16.float(), torch.zeros((1, K.C), device=dev)])
        ref = bd.expand(n, K.C).clone()
        for k in range(27):
            ref += xz[nbr_d[k].long()] @ w16[k].float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    check(out_skip.cpu().numpy(), ref.cpu().numpy(), "conv1024 all rows vs torch fp32", max_abs=1e-3, rel_l2=1e-4)


def _flow(hp, w):
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    fields = {k: getattr(hp, k) for k in HParams.__dataclass_fields__ if hasattr(hp, k)}
    return FlowModel(HParams(**fields, operand_dtype="f16"), w)


def _golden(name, coords, x, ts, ctx, w):
    g = np.load(GOLDEN / f"{name}.npz")
    # the seeded inputs here are the bytes the oracle ran on
    np.testing.assert_allclose(K.fingerprint(coords, x, ts, ctx), g["inputs_fp"], rtol=1e-12, atol=0)
    np.testing.assert_allclose(K.weights_fingerprint(w), g["weights_fp"], rtol=1e-12, atol=0)
    return g["out"]


def test_config1_block_full_size():
    coords, x, ts, offs, ctx, hp, w = K.cfg1()
    exp = _golden("cfg1_block", coords, x, ts, ctx, w)
    model = _flow(hp, w)
    dev = torch.device("cuda", 0)
    model.prepare(torch.from_numpy(coords).to(dev), 1, (K.RES, K.RES, K.RES), offs)
    got = model.forward(torch.from_numpy(x).to(dev), torch.from_numpy(ts).to(dev), torch.from_numpy(ctx).to(dev))
    got = got.cpu().numpy()
    model.close()
    assert np.isfinite(got).all()
    check(got, exp, f"config-1 block N={coords.shape[0]} (f16 operands)")


def test_config2_forward_full_size():
    coords, x, ts, offs, ctx, hp, w = K.cfg2()
    exp = _golden("cfg2_forward", coords, x, ts, ctx, w)
    model = _flow(hp, w)
    del w
    dev = torch.device("cuda", 0)
    model.prepare(torch.from_numpy(coords).to(dev), 2, (K.RES, K.RES, K.RES), offs)
    got = model.forward(torch.from_numpy(x).to(dev), torch.from_numpy(ts).to(dev), torch.from_numpy(ctx).to(dev))
    got = got.cpu().numpy()
    model.close()
    assert np.isfinite(got).all()
    half = coords.shape[0] // 2
    check(got[:half], exp[:half], "config-2 forward, conditional item")
    check(got[half:], exp[half:], "config-2 forward, zeros-condition item")
    check(got, exp, f"config-2 forward 24 blocks N=2x{half} (f16 operands)")
