"""GPU parity of each kernel behind the C ABI against the pinned oracle.

Tolerances: integer/topology outputs bit-exact; feature outputs within the
north-star bound max-abs 2e-2 and relative-L2 5e-3 against the f32 oracle.
GEMM-class kernels are additionally checked tightly (relative-L2 2e-3... see
TIGHT) against a torch fp32 computation on the SAME bf16-rounded operands, so
an indexing or layout bug cannot hide inside the bf16 tolerance.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords, batched
from tests import _fixtures as FX

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 5e-3
TIGHT = 2e-3


def ops():
    from pixal3d.cpp_b200 import ops as _ops
    return _ops


def L():
    from pixal3d.cpp_b200 import _lib
    return _lib


def check(actual, expected, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (what, a.shape, e.shape)
    err = np.abs(a - e)
    mx = float(err.max()) if err.size else 0.0
    rl = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)) if err.size else 0.0
    assert mx <= max_abs and rl <= rel_l2, f"{what}: max_abs {mx:.3e} (<= {max_abs}) rel_l2 {rl:.3e} (<= {rel_l2})"
    return mx, rl


def bf16_out_tol(expected):
    """Max-abs bound for a bf16-STORED output: the north-star 2e-2 scaled by
    the output magnitude, since storing |y| ~ 4 in bf16 alone moves it by up
    to |y| * 2^-9."""
    return MAX_ABS * max(1.0, float(np.abs(expected).max()))


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def bf(a):
    return dev(a.astype(np.float32), torch.bfloat16)


def hf(a):
    return dev(a.astype(np.float32), torch.float16)


def rounded16(a):
    """float32 values of a after f16 rounding."""
    return np.ascontiguousarray(a.astype(np.float32)).astype(np.float16).astype(np.float32)


def rounded(a):
    """float32 values of a after bf16 rounding (what the kernel consumes)."""
    return torch.from_numpy(np.ascontiguousarray(a.astype(np.float32))).to(torch.bfloat16).float().numpy()


# ----------------------------------------------------------- topology

def test_neighbor_map_config0_bitexact():
    c = shell_coords()
    got = ops().neighbor_map27(dev(c)).cpu().numpy()
    np.testing.assert_array_equal(got, O.neighbor_map27(c))
    assert int((got < c.shape[0]).sum()) == 453614


def test_neighbor_map_golden_bitexact():
    v = np.load(FX.GOLDEN / "ref_vectors.npz")
    got = ops().neighbor_map27(dev(v["coords"])).cpu().numpy()
    np.testing.assert_array_equal(got, v["nbr"])


def test_neighbor_map_edge_cases():
    o = ops()
    one = np.array([[0, 5, 5, 5]], np.int32)
    got = o.neighbor_map27(dev(one)).cpu().numpy()
    exp = np.full((27, 1), 1, np.int32)
    exp[13, 0] = 0
    np.testing.assert_array_equal(got, exp)
    # a duplicated coordinate latches P3D_ERR_DUPLICATE
    dup = np.array([[0, 1, 1, 1], [0, 1, 1, 1]], np.int32)
    o.neighbor_map27(dev(dup))
    with pytest.raises(L().P3DError) as e:
        o.ctx().sync_check()
    assert e.value.status == L().P3D_ERR_DUPLICATE


def test_neighbor_map_key_range():
    """The hash key holds 16 bits per field.  At the edges of that range the
    map still equals the (full-width) oracle: the x+1 probe of x = 32767 is
    missing, not an alias of x = -32768.  A coordinate outside the range is
    refused (P3D_ERR_INVALID) rather than aliased."""
    o = ops()
    edge = np.array([[0, -32768, 0, 0], [0, -32767, 0, 0], [0, 32766, 5, 5], [0, 32767, 0, 0],
                     [65535, 0, 32767, -32768]], np.int32)
    got = o.neighbor_map27(dev(edge)).cpu().numpy()
    o.ctx().sync_check()
    np.testing.assert_array_equal(got, O.neighbor_map27(edge))
    assert got[2 * 9 + 4, 3] == edge.shape[0]  # (x+1) of x = 32767
    for bad in ([[0, 32768, 0, 0]], [[65536, 0, 0, 0]], [[-1, 0, 0, 0]], [[0, 0, -32769, 0]]):
        o.neighbor_map27(dev(np.array(bad, np.int32)))
        with pytest.raises(L().P3DError) as e:
            o.ctx().sync_check()
        assert e.value.status == L().P3D_ERR_INVALID, bad


def test_sparse_validate_matches_reference_order():
    """Device validity probe == the reference's sequential scan (first failing
    row and check) on crafted cases and on the config-0 shell with failures
    planted at random rows."""
    from tests.test_oracle_pin import validity_cases
    o = ops()
    for name, c, x in validity_cases():
        got = o.sparse_validate(dev(c), dev(x), 2, (4, 4, 4))
        assert got == O.validate_first(c, x, 2, (4, 4, 4)), name
    rng = np.random.default_rng(3)
    shell = batched(shell_coords(), 2)
    n = shell.shape[0]
    x = rng.standard_normal((n, 5)).astype(np.float32)
    assert o.sparse_validate(dev(shell), dev(x), 2, (64, 64, 64)) is None
    for trial in range(6):
        c = shell.copy()
        xx = x.copy()
        rows = rng.choice(n, 3, replace=False)
        c[rows[0], 1 + trial % 3] = 64 + trial            # outside the shape
        c[rows[1]] = c[rng.integers(0, n)]                # duplicate (or itself: no-op)
        xx[rows[2], trial % 5] = np.nan                   # non-finite
        got = o.sparse_validate(dev(c), dev(xx), 2, (64, 64, 64))
        assert got == O.validate_first(c, xx, 2, (64, 64, 64)), (trial, got)
    # coordinates only / features only
    assert o.sparse_validate(dev(shell), None, 2, (64, 64, 64)) is None
    assert o.sparse_validate(dev(shell), None, 1, (64, 64, 64)) == O.validate_first(shell, None, 1, (64, 64, 64))


def test_downsample_bitexact():
    o = ops()
    v = np.load(FX.GOLDEN / "ref_vectors.npz")
    c = v["coords"]
    oc, parent, child, m = o.downsample_topology(dev(c), 2, (16, 16, 16), 2)
    np.testing.assert_array_equal(oc.cpu().numpy(), v["down_coords"])
    feats = o.downsample_mean(dev(v["conv_x"]), child, 2).cpu().numpy()
    # f32 in octant order == reference summation order: bit-identical
    np.testing.assert_array_equal(feats, v["down_feats"])
    # config-0 shell, batch 2 (CFG pair)
    c2 = batched(shell_coords(), 2)
    oc2, parent2, _, m2 = o.downsample_topology(dev(c2), 2, (64, 64, 64), 2)
    rc, _, rp = O.downsample_mean(c2, np.zeros((c2.shape[0], 1), np.float32), 2)
    np.testing.assert_array_equal(oc2.cpu().numpy(), rc)
    np.testing.assert_array_equal(parent2.cpu().numpy(), rp)
    assert m2 == 2 * 4092


def test_c2s_bitexact():
    o = ops()
    v = np.load(FX.GOLDEN / "ref_vectors.npz")
    c = v["coords"]
    oc, sr, sc, m = o.c2s_topology(dev(c), 2, dev(v["c2s_mask"]))
    np.testing.assert_array_equal(oc.cpu().numpy(), v["c2s_coords"])
    feats = o.c2s_gather(dev(v["c2s_x"]), sr, sc, 3).cpu().numpy()
    np.testing.assert_array_equal(feats, v["c2s_feats"])
    # unmasked + the fixture's packed example
    d = FX.sparse_fixture()
    g = FX.parse_golden("sparse_numeric_fixture")
    oc, sr, sc, m = o.c2s_topology(dev(d["packed_coords"]), 2, dev(d["subdiv"]))
    np.testing.assert_array_equal(oc.cpu().numpy().ravel(), g["sparse_channel_to_spatial_coords"].astype(np.int32))
    np.testing.assert_allclose(o.c2s_gather(dev(d["packed"]), sr, sc, 2).cpu().numpy().ravel(),
                               g["sparse_channel_to_spatial_output"], atol=1e-7)
    oc, sr, sc, m = o.c2s_topology(dev(c), 2, None)
    assert m == 8 * c.shape[0]


# -------------------------------------------------------- contractions

@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (130, 8, 8), (300, 96, 72), (4133, 256, 64), (1000, 384, 1024),
                                   (777, 200, 136), (8192, 1024, 1024), (65, 100, 64)])
def test_linear_shapes(m, n, k):
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) * 0.1
    o = ops()
    y32 = o.linear(bf(x), bf(w), dev(b), out_dtype=torch.float32).cpu().numpy()
    tight = rounded(x) @ rounded(w).T + b
    check(y32, tight, max_abs=1e-3 * max(1, np.abs(tight).max()), rel_l2=1e-5, what="linear vs bf16-rounded fp32")
    check(y32, O.linear(x, w, b), what="linear vs oracle")
    y16 = o.linear(bf(x), bf(w), dev(b), out_dtype=torch.bfloat16).float().cpu().numpy()
    ref = O.linear(x, w, b)
    check(y16, ref, max_abs=bf16_out_tol(ref), what="linear bf16 out")


def test_linear_epilogues():
    rng = np.random.default_rng(3)
    m, n, k = 1000, 512, 256
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) * 0.1
    o = ops()
    ref = O.linear(x, w, b)
    g = o.linear(bf(x), bf(w), dev(b), out_dtype=torch.float32, epilogue=L().EPI_GELU_TANH).cpu().numpy()
    check(g, O.gelu_tanh(ref), what="gelu epilogue")
    s = o.linear(bf(x), bf(w), dev(b), out_dtype=torch.bfloat16, epilogue=L().EPI_SILU).float().cpu().numpy()
    check(s, O.silu(ref), max_abs=bf16_out_tol(O.silu(ref)), what="silu epilogue")
    # gated residual with two batch items split at row 600
    res = rng.standard_normal((m, n)).astype(np.float32)
    gate = rng.standard_normal((2, n)).astype(np.float32)
    offs = np.array([0, 600, m], np.int32)
    out = dev(res.copy())
    o.linear(bf(x), bf(w), dev(b), out=out, epilogue=L().EPI_RESIDUAL, gate=dev(gate), batch_offsets=dev(offs))
    bidx = np.where(np.arange(m) < 600, 0, 1)
    exp = res + gate[bidx] * ref
    check(out.cpu().numpy(), exp, max_abs=bf16_out_tol(exp) / 4, what="residual epilogue")


def test_linear_residual_output_view():
    """Gated residual into a column slice of a wider f32 buffer: ragged rows
    and columns (the TMA epilogue's boxes are clipped at the view's bounds),
    three batch items; columns outside the view stay untouched."""
    rng = np.random.default_rng(31)
    m, n, k, ld = 777, 200, 128, 256
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    big = rng.standard_normal((m, ld)).astype(np.float32)
    gate = rng.standard_normal((3, n)).astype(np.float32)
    offs = np.array([0, 100, 500, m], np.int32)
    buf = dev(big.copy())
    view = buf[:, 32:32 + n]
    o = ops()
    o.linear(bf(x), bf(w), dev(b), out=view, epilogue=L().EPI_RESIDUAL, gate=dev(gate), batch_offsets=dev(offs))
    got = buf.cpu().numpy()
    bidx = np.searchsorted(offs, np.arange(m), side="right") - 1
    exp = big[:, 32:32 + n] + gate[bidx] * (rounded(x) @ rounded(w).T + b)
    check(got[:, 32:32 + n], exp, max_abs=1e-3 * max(1.0, float(np.abs(exp).max())), rel_l2=1e-5,
          what="residual into a view")
    np.testing.assert_array_equal(got[:, :32], big[:, :32])
    np.testing.assert_array_equal(got[:, 32 + n:], big[:, 32 + n:])


def test_linear_direct_store_epilogue_subprocess(tmp_path):
    """The direct-store epilogue (P3D_GEMM_TMA_STORE=0, read once per process)
    agrees with the TMA epilogue on f32, 16-bit, residual and head-norm
    outputs: bit for bit where both round the same expression once; within
    one rounding where they differ (the residual: fused multiply-add against
    gate*v then the add in L2; the head norm's sum of squares order)."""
    import subprocess
    import sys
    import os
    code = r"""
import math, numpy as np, torch
from pixal3d.cpp_b200 import ops, _lib as L
from pixal3d.cpp_b200.workloads import shell_coords
rng = np.random.default_rng(44)
m, n, k = 1000, 384, 256
x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().half()
w = torch.from_numpy((rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)).cuda().half()
b = torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float32)).cuda()
res = torch.from_numpy(rng.standard_normal((m, n)).astype(np.float32)).cuda()
gate = torch.from_numpy(rng.standard_normal((2, n)).astype(np.float32)).cuda()
offs = torch.tensor([0, 600, m], dtype=torch.int32, device="cuda")
coords = torch.from_numpy(shell_coords(24, 8.0, 1.0)[:m]).cuda()
table = ops.rope_table(coords, 64)
gam = torch.from_numpy((1 + 0.1 * rng.standard_normal(2 * 128)).astype(np.float32)).cuda()
outs = [ops.linear(x, w, b, out_dtype=torch.float32), ops.linear(x, w, b, out_dtype=torch.float16, epilogue=L.EPI_GELU_TANH)]
r = res.clone(); ops.linear(x, w, b, out=r, epilogue=L.EPI_RESIDUAL, gate=gate, batch_offsets=offs); outs.append(r)
outs.append(ops.linear_headnorm(x, w, b, 128, gam, 256, table, out=torch.empty((m, n), device="cuda", dtype=torch.float16)))
# the trunk's residual shape with a partial last row tile (65 x 4 tiles)
m2, n2 = 8190, 1024
x2 = torch.from_numpy(rng.standard_normal((m2, 1024)).astype(np.float32)).cuda().half()
w2 = torch.from_numpy((rng.standard_normal((n2, 1024)) / 32).astype(np.float32)).cuda().half()
b2 = torch.from_numpy((rng.standard_normal(n2) * 0.1).astype(np.float32)).cuda()
g2 = torch.from_numpy(rng.standard_normal((2, n2)).astype(np.float32)).cuda()
o2 = torch.tensor([0, 5000, m2], dtype=torch.int32, device="cuda")
r2 = torch.from_numpy(rng.standard_normal((m2, n2)).astype(np.float32)).cuda()
ops.linear(x2, w2, b2, out=r2, epilogue=L.EPI_RESIDUAL, gate=g2, batch_offsets=o2); outs.append(r2)
torch.save([t.cpu() for t in outs], "OUT")
print("ok")
"""
    env = os.environ.copy()
    got = []
    for flag in ("1", "0"):
        out = tmp_path / f"epilogue_{flag}.pt"
        env["P3D_GEMM_TMA_STORE"] = flag
        r = subprocess.run([sys.executable, "-c", code.replace("OUT", str(out))], env=env, capture_output=True,
                           text=True, timeout=600, cwd=str(FX.GOLDEN.parent.parent))
        assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
        got.append(torch.load(out))
    tma, direct = got
    assert torch.equal(tma[0], direct[0]) and torch.equal(tma[1], direct[1])
    torch.testing.assert_close(tma[2], direct[2], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(tma[3].float(), direct[3].float(), rtol=1e-3, atol=1e-3)
    # trunk shape: TMA reduce-add vs read-modify-write of the residual
    torch.testing.assert_close(tma[4], direct[4], rtol=1e-5, atol=1e-4)


def test_linear_residual_trunk_shapes():
    """Gated-residual linears at the trunk's shapes (8,184 rows, or 8,190 with
    a partial last row tile; 1,024 output columns; K = 1,024 for the attention
    output projections, 4,096 for MLP down), residual batch segments split
    unevenly.  Against torch fp32 (no TF32) on the same f16 operands."""
    rng = np.random.default_rng(46)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for m, k in ((8184, 1024), (8190, 4096)):
            n = 1024
            x = hf(rng.standard_normal((m, k)))
            w = hf(rng.standard_normal((n, k)) / math.sqrt(k))
            b = dev((rng.standard_normal(n) * 0.1).astype(np.float32))
            res = dev(rng.standard_normal((m, n)).astype(np.float32))
            gate = dev(rng.standard_normal((2, n)).astype(np.float32))
            offs = torch.tensor([0, m // 3, m], dtype=torch.int32, device="cuda")
            out = res.clone()
            ops().linear(x, w, b, out=out, epilogue=L().EPI_RESIDUAL, gate=gate, batch_offsets=offs)
            g = torch.where(torch.arange(m, device="cuda")[:, None] < m // 3, gate[0], gate[1])
            exp = res + g * (x.float() @ w.float().T + b)
            check(out.cpu().numpy(), exp.cpu().numpy(), max_abs=1e-3, rel_l2=1e-5, what=f"trunk residual k={k}")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_linear_strided_input():
    """A column slice of a wider row (the attention output / qkv views)."""
    rng = np.random.default_rng(5)
    m, k, n = 513, 128, 192
    big = rng.standard_normal((m, 3 * k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)
    t = bf(big)
    y = ops().linear(t[:, k:2 * k], bf(w), None, out_dtype=torch.float32).cpu().numpy()
    check(y, rounded(big[:, k:2 * k]) @ rounded(w).T, max_abs=1e-3, rel_l2=1e-5, what="strided A")


def _conv_case(coords, cin, cout, seed):
    rng = np.random.default_rng(seed)
    n = coords.shape[0]
    x = rng.standard_normal((n, cin)).astype(np.float32)
    w = (rng.standard_normal((27, cout, cin)) / math.sqrt(27 * cin)).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("cin,cout", [(64, 64), (128, 384), (64, 8)])
def test_subm_conv3d(cin, cout):
    c = shell_coords() if cin == 64 and cout == 64 else shell_coords(40, 14.0, 1.3)
    x, w, b = _conv_case(c, cin, cout, cin + cout)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    got = o.subm_conv3d(bf(x), nbr, bf(w), dev(b), out_dtype=torch.float32).cpu().numpy()
    nb = O.neighbor_map27(c)
    tight = O.subm_conv3d(c, rounded(x), rounded(w), b, nb)
    check(got, tight, max_abs=2e-3, rel_l2=TIGHT * 0.05, what="conv vs bf16-rounded fp32")
    check(got, O.subm_conv3d(c, x, w, b, nb), what="conv vs oracle")


@pytest.mark.parametrize("cin,cout,npts", [(64, 512, None), (128, 256, None), (64, 512, 100)])
def test_subm_conv3d_pair_tiles(cin, cout, npts):
    """Cout a multiple of 256 runs the CTA-pair kernel (two N = 256 MMAs per
    pair tile when Cout % 512 == 0); 5,530 points leave the odd CTA of the last
    pair partly empty, 100 points leave it empty."""
    c = shell_coords(40, 14.0, 1.3)
    if npts is not None:
        c = np.ascontiguousarray(c[:npts])
    x, w, b = _conv_case(c, cin, cout, cin * 7 + cout)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    got = o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out_dtype=torch.float32).cpu().numpy()
    nb = O.neighbor_map27(c)
    tight = O.subm_conv3d(c, rounded16(x), rounded16(w), b, nb)
    check(got, tight, max_abs=1e-3, rel_l2=1e-4, what="pair conv vs f16-rounded fp32")
    res = np.random.default_rng(2).standard_normal(tight.shape).astype(np.float32)
    out = dev(res.copy())
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=out, epilogue=L().EPI_RESIDUAL)
    check(out.cpu().numpy(), res + tight, max_abs=1e-3, rel_l2=1e-4, what="pair conv residual")


def test_subm_conv3d_tile_taps_skip_is_exact():
    """Rows ordered by neighbour pattern (as the flow's fine level runs):
    the pair kernel skipping the taps no row of a 256-row tile uses gives the
    same bits as the full 27-tap loop, plain and with the residual epilogue."""
    c = shell_coords(40, 14.0, 1.3)
    nb = O.neighbor_map27(c)
    mask = np.zeros(c.shape[0], np.int64)
    for t in range(27):
        mask |= (nb[t] < c.shape[0]).astype(np.int64) << t
    c = np.ascontiguousarray(c[np.argsort(mask, kind="stable")])
    x, w, b = _conv_case(c, 128, 512, 3)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    taps = o.conv_tile_taps(nbr)
    tb = taps.cpu().numpy().astype(np.uint32)
    full = (1 << 27) - 1
    assert (tb != full).sum() > 0  # some tiles skip taps
    a = o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out_dtype=torch.float32)
    s = o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out_dtype=torch.float32, tile_taps=taps)
    assert torch.equal(a, s)
    res = dev(np.random.default_rng(1).standard_normal((c.shape[0], 512)).astype(np.float32))
    r1, r2 = res.clone(), res.clone()
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=r1, epilogue=L().EPI_RESIDUAL)
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=r2, epilogue=L().EPI_RESIDUAL, tile_taps=taps)
    assert torch.equal(r1, r2)
    # tile taps against the map: OR of each 256-row tile's neighbour patterns
    nbs = O.neighbor_map27(c)
    pat = np.zeros(c.shape[0], np.int64)
    for t in range(27):
        pat |= (nbs[t] < c.shape[0]).astype(np.int64) << t
    exp = [int(np.bitwise_or.reduce(pat[i:i + 256])) for i in range(0, c.shape[0], 256)]
    np.testing.assert_array_equal(tb.astype(np.int64), exp)



def test_subm_conv3d_residual_bf16():
    c = shell_coords(32, 10.0, 1.2)
    x, w, b = _conv_case(c, 64, 128, 9)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    ref = O.subm_conv3d(c, x, w, b)
    y16 = o.subm_conv3d(bf(x), nbr, bf(w), dev(b), out_dtype=torch.bfloat16).float().cpu().numpy()
    check(y16, ref, max_abs=bf16_out_tol(ref), what="conv bf16 out")
    res = np.random.default_rng(1).standard_normal(ref.shape).astype(np.float32)
    out = dev(res.copy())
    o.subm_conv3d(bf(x), nbr, bf(w), dev(b), out=out, epilogue=L().EPI_RESIDUAL)
    check(out.cpu().numpy(), res + ref, what="conv residual")


def test_sparse_fixture_ops_on_gpu():
    """The reference's sparse_numeric_fixture inputs through the GPU kernels
    (channels zero-padded to the kernels' granularity, as the host layer
    does) against the reference's own outputs."""
    d = FX.sparse_fixture()
    g = FX.parse_golden("sparse_numeric_fixture")
    o = ops()
    c = d["coords"]
    xp = np.zeros((10, 64), np.float32)
    xp[:, :3] = d["x"]
    wl = np.zeros((4, 8), np.float32)
    wl[:, :3] = d["lin_w"]
    y = o.linear(bf(xp[:, :8].copy()), bf(wl), dev(d["lin_b"]), out_dtype=torch.float32).cpu().numpy()
    check(y.ravel(), g["sparse_linear_output"], what="fixture linear")
    wc = np.zeros((27, 4, 64), np.float32)
    wc[:, :, :3] = d["conv_w"]
    nbr = o.neighbor_map27(dev(c))
    y = o.subm_conv3d(bf(xp), nbr, bf(wc), dev(d["conv_b"]), out_dtype=torch.float32).cpu().numpy()
    check(y.ravel(), g["sparse_conv_output"], what="fixture conv")
    y = o.layernorm_modulate(dev(d["x"]), 1e-5, dev(d["gamma"]), dev(d["beta"]), out_dtype=torch.float32)
    check(y.cpu().numpy().ravel(), g["sparse_norm_output"], max_abs=1e-5, rel_l2=1e-6, what="fixture layernorm")
    dc, parent, child, m = o.downsample_topology(dev(c), 2, (4, 4, 4), 2)
    np.testing.assert_array_equal(dc.cpu().numpy().ravel(), g["sparse_downsample_coords"].astype(np.int32))
    y = o.downsample_mean(dev(d["x"]), child, 2).cpu().numpy()
    check(y.ravel(), g["sparse_downsample_output"], max_abs=1e-6, rel_l2=1e-7, what="fixture downsample")


# ------------------------------------------------------------ elementwise

def test_layernorm_modulate():
    rng = np.random.default_rng(4)
    n, C = 3001, 1024
    x = (rng.standard_normal((n, C)) * 3 + 1).astype(np.float32)
    offs = np.array([0, 1500, n], np.int32)
    tmod = rng.standard_normal((2, 6 * C)).astype(np.float32) * 0.3
    bmod = rng.standard_normal(6 * C).astype(np.float32) * 0.1
    mod = (tmod + bmod[None, :]).astype(np.float32)
    bidx = np.where(np.arange(n) < 1500, 0, 1)
    o = ops()
    for off in (0, 3 * C):
        got = o.layernorm_modulate(dev(x), 1e-6, mod=dev(mod)[:, off:], batch_offsets=dev(offs)).float().cpu().numpy()
        exp = O.affine_modulate(O.layer_norm(x, 1e-6), bmod, tmod.ravel(), bidx, C, off)
        check(got, exp, what=f"ln+mod offset {off}")
    gam = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    bet = (rng.standard_normal(C) * 0.1).astype(np.float32)
    got = o.layernorm_modulate(dev(x), 1e-6, dev(gam), dev(bet), out_dtype=torch.float32).cpu().numpy()
    check(got, O.layer_norm(x, 1e-6, gam, bet), max_abs=1e-4, rel_l2=1e-6, what="ln affine f32")
    # odd channel count (no vector path)
    x3 = rng.standard_normal((17, 12)).astype(np.float32)
    got = o.layernorm_modulate(dev(x3), 1e-5, out_dtype=torch.float32).cpu().numpy()
    check(got, O.layer_norm(x3, 1e-5), max_abs=1e-5, rel_l2=1e-6, what="ln C=12")
    # C = 640: float4 loads but no register-resident instance; C = 384: register path, f16 out
    for cc, dt in ((640, torch.float32), (384, torch.float16)):
        xc = (rng.standard_normal((999, cc)) * 2).astype(np.float32)
        gc = (1 + rng.standard_normal(cc) * 0.1).astype(np.float32)
        bc = (rng.standard_normal(cc) * 0.1).astype(np.float32)
        got = o.layernorm_modulate(dev(xc), 1e-6, dev(gc), dev(bc), out_dtype=dt).float().cpu().numpy()
        tol = 1e-4 if dt == torch.float32 else 4e-3
        check(got, O.layer_norm(xc, 1e-6, gc, bc), max_abs=tol, rel_l2=1e-3, what=f"ln C={cc}")


def test_qk_rmsnorm_rope():
    rng = np.random.default_rng(8)
    c = batched(shell_coords(32, 11.0, 1.0), 2)
    n, H, hd = c.shape[0], 16, 64
    q = rng.standard_normal((n, 3 * H * hd)).astype(np.float32)
    gam = (1 + rng.standard_normal(H * hd) * 0.1).astype(np.float32)
    t = bf(q)
    o = ops()
    o.qk_rmsnorm_rope(t[:, :H * hd], H, hd, dev(gam), dev(c))
    o.qk_rmsnorm_rope(t[:, H * hd:2 * H * hd], H, hd, dev(gam), None)
    got = t.float().cpu().numpy()
    qr = rounded(q)
    check(got[:, :H * hd], O.rope(c, O.rms_norm_heads(qr[:, :H * hd], H, hd, gam), H, hd), what="rms+rope")
    check(got[:, H * hd:2 * H * hd], O.rms_norm_heads(qr[:, H * hd:2 * H * hd], H, hd, gam), what="rms only")
    np.testing.assert_array_equal(got[:, 2 * H * hd:], qr[:, 2 * H * hd:])
    # the fixture's RoPE (hd = 6, remainder pairs unrotated) and RMS outputs
    d = FX.sparse_fixture()
    g = FX.parse_golden("sparse_numeric_fixture")
    t = bf(d["q"])
    o.qk_rmsnorm_rope(t, 2, 6, None, dev(d["coords"]))
    check(t.float().cpu().numpy().ravel(), g["sparse_rope_output"], what="fixture rope")
    t = bf(d["q"])
    o.qk_rmsnorm_rope(t, 2, 6, dev(d["rms_gamma"]), None)
    check(t.float().cpu().numpy().ravel(), g["sparse_rms_output"], what="fixture rms")


def _attn_case(rng, lq, lk, H=4):
    q = rng.standard_normal((sum(lq), H * 64)).astype(np.float32)
    k = rng.standard_normal((sum(lk), H * 64)).astype(np.float32)
    v = rng.standard_normal((sum(lk), H * 64)).astype(np.float32)
    cq = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    ck = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    return q, k, v, cq, ck


@pytest.mark.parametrize("lq,lk", [([1, 77], [1, 77]), ([1000, 333], [1000, 333]), ([129], [1029]),
                                   ([2048, 2048], [1029, 1029])])
def test_varlen_attention(lq, lk):
    rng = np.random.default_rng(sum(lq) + sum(lk))
    H = 4
    q, k, v, cq, ck = _attn_case(rng, lq, lk, H)
    scale = 1.0 / 8.0
    got = ops().varlen_attention(bf(q), bf(k), bf(v), dev(cq), dev(ck), max(lq), H, scale).float().cpu().numpy()
    exp = O.varlen_attention(rounded(q), rounded(k), rounded(v), cq, ck, H, 64, scale)
    check(got, exp, what="attention")


def test_attention_strided_qkv_views():
    """q/k/v as column slices of one packed [n, 3C] buffer (the qkv GEMM output)."""
    rng = np.random.default_rng(12)
    H, n = 16, 700
    qkv = rng.standard_normal((n, 3 * H * 64)).astype(np.float32)
    cu = np.array([0, 300, n], np.int32)
    t = bf(qkv)
    C = H * 64
    got = ops().varlen_attention(t[:, :C], t[:, C:2 * C], t[:, 2 * C:], dev(cu), dev(cu), 400, H, 0.125)
    r = rounded(qkv)
    exp = O.varlen_attention(r[:, :C], r[:, C:2 * C], r[:, 2 * C:], cu, cu, H, 64, 0.125)
    check(got.float().cpu().numpy(), exp, what="strided attention")


@pytest.mark.parametrize("C,groups", [(256, 32), (1024, 32), (512, 2), (384, 4), (192, 8), (32, 32), (128, 64),
                                      (768, 32)])
def test_group_norm_silu(C, groups):
    """Group widths that take each reduction of the rows-layout stats kernel
    (shuffle over a power-of-two lane group, whole warp, per-lane atomics),
    channel counts outside its layout (C % 128 != 0, C = 768) and groups
    narrower than a float4 (1 and 2 channels: GroupNorm32 at C = 32); three
    batch items."""
    rng = np.random.default_rng(21 + C)
    c = batched(shell_coords(24, 8.0, 1.0), 3)
    n = c.shape[0]
    x = (rng.standard_normal((n, C)) * 2 + 0.5).astype(np.float32)
    gam = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    bet = (rng.standard_normal(C) * 0.1).astype(np.float32)
    o = ops()
    offs = o.batch_offsets_of(dev(c), 3)
    got = o.group_norm_silu(dev(x), groups, 1e-5, dev(gam), dev(bet), offs, True, torch.float32).cpu().numpy()
    exp = O.silu(O.group_norm(c[:, 0].astype(np.int64), x, groups, 1e-5, gam, bet))
    check(got, exp, max_abs=1e-4, rel_l2=1e-5, what="groupnorm+silu")
    h = o.group_norm_silu(dev(x), groups, 1e-5, dev(gam), dev(bet), offs, False, torch.float16).float().cpu().numpy()
    exp = O.group_norm(c[:, 0].astype(np.int64), x, groups, 1e-5, gam, bet)
    check(h, exp, max_abs=4e-3 * max(1.0, float(np.abs(exp).max())), what="groupnorm f16 out")


@pytest.mark.parametrize("g,gr", [(1.0, 0.0), (3.0, 0.0), (2.35, 0.41)])
def test_euler_cfg_step(g, gr):
    rng = np.random.default_rng(2)
    c = batched(shell_coords(16, 5.0, 1.0), 2)
    n = c.shape[0]
    x = rng.standard_normal((n, 8)).astype(np.float32)
    vp = rng.standard_normal((n, 8)).astype(np.float32)
    vn = rng.standard_normal((n, 8)).astype(np.float32)
    cfg = O.SamplerConfig(steps=4, sigma_min=0.031, guidance_strength=g, guidance_rescale=gr)
    t, tn = np.float32(0.7), np.float32(0.45)
    bidx = c[:, 0].astype(np.int64)
    pred = O.cfg_combine(x, t, vp, vn, np.float32(g), cfg, bidx, 2) if g != 1.0 else vp
    exp = x - (t - tn) * pred
    o = ops()
    xt = dev(x.copy())
    x0 = torch.empty_like(xt)
    o.euler_cfg_step(xt, dev(vp), dev(vn) if g != 1.0 else None, o.batch_offsets_of(dev(c), 2), float(t), float(tn),
                     g, gr, 0.031, x0_out=x0)
    check(xt.cpu().numpy(), exp, max_abs=1e-5, rel_l2=1e-6, what="euler/cfg")
    a = np.float32(1 - 0.031)
    check(x0.cpu().numpy(), a * x - (np.float32(0.031) + a * t) * pred, max_abs=1e-5, rel_l2=1e-6, what="x0 out")


# ------------------------------------------------------ f16 operand variants

@pytest.mark.parametrize("m,n,k", [(130, 8, 8), (4133, 256, 64), (2000, 1024, 1024)])
def test_linear_f16(m, n, k):
    rng = np.random.default_rng(m * 3 + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / math.sqrt(k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32) * 0.1
    o = ops()
    y = o.linear(hf(x), hf(w), dev(b), out_dtype=torch.float32).cpu().numpy()
    tight = rounded16(x) @ rounded16(w).T + b
    check(y, tight, max_abs=1e-3 * max(1, np.abs(tight).max()), rel_l2=1e-5, what="f16 linear vs rounded fp32")
    check(y, O.linear(x, w, b), max_abs=3e-3, rel_l2=1e-3, what="f16 linear vs oracle")
    y16 = o.linear(hf(x), hf(w), dev(b), out_dtype=torch.float16).float().cpu().numpy()
    check(y16, O.linear(x, w, b), max_abs=3e-3 * max(1, np.abs(tight).max()), rel_l2=1e-3, what="f16 out")


def test_subm_conv3d_f16():
    c = shell_coords()
    x, w, b = _conv_case(c, 64, 64, 77)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    got = o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out_dtype=torch.float32).cpu().numpy()
    nb = O.neighbor_map27(c)
    check(got, O.subm_conv3d(c, rounded16(x), rounded16(w), b, nb), max_abs=1e-3, rel_l2=1e-4, what="f16 conv tight")
    check(got, O.subm_conv3d(c, x, w, b, nb), max_abs=3e-3, rel_l2=1e-3, what="f16 conv vs oracle")


def test_varlen_attention_f16():
    rng = np.random.default_rng(99)
    H = 4
    q, k, v, cq, ck = _attn_case(rng, [700, 1300], [700, 1300], H)
    got = ops().varlen_attention(hf(q), hf(k), hf(v), dev(cq), dev(ck), 1300, H, 0.125).float().cpu().numpy()
    exp = O.varlen_attention(q, k, v, cq, ck, H, 64, 0.125)
    check(got, exp, max_abs=5e-3, rel_l2=1e-3, what="f16 attention")


def test_qk_rmsnorm_rope_f16():
    rng = np.random.default_rng(18)
    c = shell_coords(32, 11.0, 1.0)
    n, H, hd = c.shape[0], 16, 64
    q = rng.standard_normal((n, H * hd)).astype(np.float32)
    gam = (1 + rng.standard_normal(H * hd) * 0.1).astype(np.float32)
    t = hf(q)
    ops().qk_rmsnorm_rope(t, H, hd, dev(gam), dev(c))
    check(t.float().cpu().numpy(), O.rope(c, O.rms_norm_heads(q, H, hd, gam), H, hd), max_abs=1e-2, rel_l2=1e-3,
          what="f16 rms+rope")


# ------------------------------------------- fused per-head norm + RoPE GEMM

def test_rope_table():
    c = batched(shell_coords(32, 11.0, 1.0), 2)
    t = ops().rope_table(dev(c), 64, 1.0, 10000.0).cpu().numpy().transpose(1, 0, 2)  # pair-major -> [n, pairs, 2]
    cos, sin = O.rope_tables(c, 64, 1.0, 10000.0)
    check(t[..., 0], cos, max_abs=2e-5, rel_l2=1e-5, what="rope cos")
    check(t[..., 1], sin, max_abs=2e-5, rel_l2=1e-5, what="rope sin")


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("norm,rope", [(2, 2), (0, 2), (1, 0)])
def test_linear_headnorm(dtype, norm, rope):
    """qkv-style GEMM with the q/k head RMS norm and RoPE in the epilogue ==
    rope(rms_norm_heads(x W^T + b)) on the same rounded operands; columns
    past the fused range are the plain linear output."""
    rng = np.random.default_rng(31 + norm * 3 + rope)
    c = batched(shell_coords(24, 8.0, 1.2), 2)
    m, H, hd, k = c.shape[0], 4, 64, 256
    C = H * hd
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((3 * C, k)) / math.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal(3 * C) * 0.1).astype(np.float32)
    gam = (1 + rng.standard_normal(3 * C) * 0.1).astype(np.float32)
    to16, rnd = (hf, rounded16) if dtype == "f16" else (bf, rounded)
    o = ops()
    table = o.rope_table(dev(c), 64)
    got = o.linear_headnorm(to16(x), to16(w), dev(b), norm * C, dev(gam), rope * C, table).float().cpu().numpy()
    y = rnd(x) @ rnd(w).T + b
    exp = y.copy()
    if norm:
        exp[:, :norm * C] = O.rms_norm_heads(y[:, :norm * C], norm * H, hd, gam[:norm * C])
    for j in range(rope):
        exp[:, j * C:(j + 1) * C] = O.rope(c, exp[:, j * C:(j + 1) * C], H, hd)
    if dtype == "f16":
        check(got, exp, max_abs=4e-3 * max(1.0, float(np.abs(exp).max())), rel_l2=1e-3, what="f16 headnorm")
    else:
        check(got, exp, max_abs=bf16_out_tol(exp), rel_l2=REL_L2, what="bf16 headnorm")


def test_conv_row_order_matches_stable_sort():
    """p3d_conv_row_order (device radix sort) == numpy's stable argsort of
    (batch, row chunk, neighbour pattern), on the batch-2 config-0 shell and
    on a six-item ragged batch (chunks straddling items), for the flow's
    chunk, one chunk, and a small chunk; a chunk too small for a 64-bit key
    is refused."""
    from pixal3d.cpp_b200.workloads import image_shells, pack_cfg
    from tests._configs import pattern_order, CONV_ORDER_CHUNK_ROWS
    assert CONV_ORDER_CHUNK_ROWS == L().CONV_ORDER_CHUNK_ROWS
    o = ops()
    packed, _ = pack_cfg(image_shells(3, seed=5))
    for cs, batch in ((batched(shell_coords(), 2), 2), (packed, 6)):
        d = dev(cs)
        nb = O.neighbor_map27(cs)
        nbr = o.neighbor_map27(d)
        perm = o.conv_row_order(d, nbr, batch).cpu().numpy()
        np.testing.assert_array_equal(perm, pattern_order(cs, nb))
        for chunk in (0, 1000):
            perm = o.conv_row_order(d, nbr, batch, chunk).cpu().numpy()
            np.testing.assert_array_equal(perm, pattern_order(cs, nb, chunk))
    with pytest.raises(ValueError, match="64-bit key"):
        o.conv_row_order(d, nbr, 1 << 30, 1)


def test_flow_prepare_rejects_unordered_batches():
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    from tests._models import random_flow_weights
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=1,
                       num_heads=2, io_resblocks=1, groups=32)
    fields = {k: getattr(hp, k) for k in HParams.__dataclass_fields__ if hasattr(hp, k)}
    model = FlowModel(HParams(**fields), random_flow_weights(np.random.default_rng(0), hp))
    c = batched(shell_coords(16, 5.0, 1.0), 2)
    bad = np.ascontiguousarray(np.concatenate([c[c[:, 0] == 1], c[c[:, 0] == 0]]))
    with pytest.raises(L().P3DError, match="contiguous by batch"):
        model.prepare(dev(bad), 2, (16, 16, 16), [0, 10, 20])
    # the same flow prepares a valid set afterwards
    model.prepare(dev(c), 2, (16, 16, 16), [0, 10, 20])
    model.close()


def test_subm_conv3d_split_schedule_residual():
    """171 tiles of 128 rows on 148 SMs take the split schedule (tiles cut
    between two CTAs are summed by atomics); with a residual epilogue the
    output accumulates onto the caller's values, without one it starts from
    zero.  Both against the oracle on the same f16-rounded operands."""
    c = shell_coords()
    x, w, b = _conv_case(c, 64, 64, 21)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    ref = O.subm_conv3d(c, rounded16(x), rounded16(w), b, O.neighbor_map27(c))
    res = np.random.default_rng(2).standard_normal(ref.shape).astype(np.float32)
    out = dev(res.copy())
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=out, epilogue=L().EPI_RESIDUAL)
    check(out.cpu().numpy(), res + ref, max_abs=1e-3, rel_l2=1e-5, what="split conv residual")
    out2 = dev(np.full(ref.shape, 7.0, np.float32))
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=out2)
    check(out2.cpu().numpy(), ref, max_abs=1e-3, rel_l2=1e-5, what="split conv")


@pytest.mark.gpu
def test_subm_conv3d_pair_split_schedule():
    """The CTA-pair conv (C_out a multiple of 256) on 86 pair tiles of 256 rows
    takes the split schedule on the 74 SM pairs: each pair an equal share of
    all tiles' (used tap, K block) steps, cut tiles summed by atomics, bias
    once.  Rows in neighbour-pattern order with tap skipping, plain output
    (starts from zero whatever the buffer held) and residual epilogue, against
    the oracle on the same f16-rounded operands."""
    c = shell_coords()
    nb = O.neighbor_map27(c)
    mask = np.zeros(c.shape[0], np.int64)
    for t in range(27):
        mask |= (nb[t] < c.shape[0]).astype(np.int64) << t
    c = np.ascontiguousarray(c[np.argsort(mask, kind="stable")])
    x, w, b = _conv_case(c, 128, 256, 23)
    o = ops()
    nbr = o.neighbor_map27(dev(c))
    taps = o.conv_tile_taps(nbr)
    ref = O.subm_conv3d(c, rounded16(x), rounded16(w), b, O.neighbor_map27(c))
    out = dev(np.full(ref.shape, -3.0, np.float32))
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=out, tile_taps=taps)
    check(out.cpu().numpy(), ref, max_abs=1e-3, rel_l2=1e-5, what="pair split conv")
    res = np.random.default_rng(3).standard_normal(ref.shape).astype(np.float32)
    out2 = dev(res.copy())
    o.subm_conv3d(hf(x), nbr, hf(w), dev(b), out=out2, epilogue=L().EPI_RESIDUAL, tile_taps=taps)
    check(out2.cpu().numpy(), res + ref, max_abs=1e-3, rel_l2=1e-5, what="pair split conv residual")
