"""p3d_project_features (projection conditioning, src/projection.cpp) on the
GPU against the pinned restatement and the reference's own outputs.

The kernel computes in IEEE f32 in the reference's operation order with no
contraction, so features and validity flags are compared for EQUALITY with
the reference's outputs (tests/golden/projection_vectors.npz, produced by the
compiled reference) and with the oracle; the reference fixture's printed
values are checked with the reference comparator's tolerance (2e-5 max-abs,
2e-6 relative L2, scripts/compare_projection.py:23-29) since they are text.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords
from tests import _fixtures as FX
from tests.test_projection import TRANSLATED, close, fixture_map

pytestmark = pytest.mark.gpu

GOLD = FX.GOLDEN / "projection_vectors.npz"


def ops():
    from pixal3d.cpp_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def view(fmap, res, cam: O.ProjCamera):
    v = {"feature_map": dev(np.asarray(fmap, np.float32)), "image_resolution": res,
         "camera_angle_x": cam.camera_angle_x, "distance": cam.distance, "mesh_scale": cam.mesh_scale}
    if cam.transform is not None:
        v["transform"] = np.asarray(cam.transform, np.float32).reshape(16)
    return v


def run(views, grid, coords=None, out_dtype=torch.float32, **kw):
    o = ops()
    out, valid = o.project_features(views, grid, None if coords is None else dev(np.asarray(coords, np.int32)),
                                    out_dtype=out_dtype, **kw)
    o.ctx(0).sync_check()
    return out, valid


def test_reference_fixture_dense_grid():
    g = FX.parse_golden("projection_numeric_fixture")
    cam = O.ProjCamera(0.8, 2.25, 1.5)
    f, v = run([view(fixture_map(-0.5), 16, cam)], 4)
    close(f.cpu().numpy(), g["single_features"])
    np.testing.assert_array_equal(v.cpu().numpy(), g["single_valid"])
    moved = O.ProjCamera(0.8, 2.25, 1.5, TRANSLATED)
    f, v = run([view(fixture_map(-0.5), 16, cam), view(fixture_map(0.75), 16, moved)], 4)
    close(f.cpu().numpy(), g["average_features"])
    np.testing.assert_array_equal(v.cpu().numpy(), g["average_valid"])
    ef, ev = O.project_features_average([fixture_map(-0.5), fixture_map(0.75)], 4, 16, [cam, moved])
    np.testing.assert_array_equal(f.cpu().numpy(), ef)


def test_reference_vectors_bit_exact():
    v = np.load(GOLD)
    coords, fmap = v["coords"], v["fmap"]
    f, val = run([view(fmap, 518, O.ProjCamera(0.6, 2.0, 1.0))], 64, coords)
    np.testing.assert_array_equal(f.cpu().numpy(), v["front_feats"])
    np.testing.assert_array_equal(val.cpu().numpy(), v["front_valid"])
    f, val = run([view(fmap, 518, O.ProjCamera(0.9, 2.0, 0.8, v["moved_c2w"]))], 64, coords)
    np.testing.assert_array_equal(f.cpu().numpy(), v["moved_feats"])
    np.testing.assert_array_equal(val.cpu().numpy(), v["moved_valid"])
    cams = [O.ProjCamera(0.7, 2.2, 1.0), O.ProjCamera(0.7, 2.2, 1.0, v["avg_c2w"])]
    f, val = run([view(v["avg_map_a"], 64, cams[0]), view(v["avg_map_b"], 64, cams[1])], 8)  # C = 5: scalar path
    np.testing.assert_array_equal(f.cpu().numpy(), v["avg_feats"])
    np.testing.assert_array_equal(val.cpu().numpy(), v["avg_valid"])


def test_full_shell_dino_map_and_16bit_outputs():
    """The 64^3 shell (21,766 points) sampled from a 37 x 37 x 1024 map from
    three views; f16 / bf16 outputs are the f32 result rounded once."""
    rng = np.random.default_rng(5)
    coords = shell_coords()
    coords[:, 0] = 0
    maps = [rng.standard_normal((37, 37, 1024)).astype(np.float32) for _ in range(3)]
    rel = O.relative_calc_matrices([np.eye(4, dtype=np.float32).reshape(16), TRANSLATED,
                                    np.asarray(np.load(GOLD)["moved_c2w"], np.float32)], [2.0, 2.0, 2.0])
    cams = [O.ProjCamera(0.6, 2.0, 1.0, m) for m in rel]
    views = [view(m, 518, c) for m, c in zip(maps, cams)]
    f, val = run(views, 64, coords)
    ef, ev = O.project_features_average(maps, 64, 518, cams, coords)
    np.testing.assert_array_equal(val.cpu().numpy(), ev)
    np.testing.assert_array_equal(f.cpu().numpy(), ef)
    t = torch.from_numpy(ef).cuda()
    for dt in (torch.float16, torch.bfloat16):
        h, _ = run(views, 64, coords, out_dtype=dt)
        assert torch.equal(h, t.to(dt))


def test_channel_concatenation_and_unaligned_columns():
    """Two maps (8 and 5 channels) written side by side into one [n, 16] f32
    buffer at column offsets 0 and 9 (the second call takes the
    one-channel-per-lane path: its rows are not 16-byte aligned)."""
    rng = np.random.default_rng(9)
    coords = np.ascontiguousarray(shell_coords(24, 9.0, 1.2))
    coords[:, 0] = 0
    a = rng.standard_normal((20, 22, 8)).astype(np.float32)
    b = rng.standard_normal((11, 13, 5)).astype(np.float32)
    cam = O.ProjCamera(0.5, 1.8, 1.1)
    buf = torch.full((coords.shape[0], 16), 7.0, device="cuda")
    run([view(a, 256, cam)], 24, coords, out=buf[:, 0:8])
    run([view(b, 128, cam)], 24, coords, out=buf[:, 9:14])
    fa, _ = O.project_features_at_coords(a, 24, 256, cam, coords)
    fb, _ = O.project_features_at_coords(b, 24, 128, cam, coords)
    got = buf.cpu().numpy()
    np.testing.assert_array_equal(got[:, 0:8], fa)
    np.testing.assert_array_equal(got[:, 9:14], fb)
    assert np.all(got[:, 8] == 7.0) and np.all(got[:, 14:] == 7.0)


def test_errors():
    o = ops()
    m = np.zeros((4, 4, 4), np.float32)
    with pytest.raises(o.P3DError, match="camera_angle_x must be finite"):
        run([view(m, 16, O.ProjCamera(camera_angle_x=4.0))], 4)
    with pytest.raises(o.P3DError, match="camera transform matrix is singular"):
        run([view(m, 16, O.ProjCamera(transform=np.zeros(16, np.float32)))], 4)
    with pytest.raises(o.P3DError, match="grid_resolution must be positive"):
        run([view(m, 16, O.ProjCamera())], 0, np.zeros((1, 4), np.int32))
    with pytest.raises(o.P3DError, match="same channel count"):
        run([view(m, 16, O.ProjCamera()), view(np.zeros((4, 4, 3), np.float32), 16, O.ProjCamera())], 4)
    # a coordinate outside the grid is latched on the device and reported at
    # the next check; its row is zeros and later calls are unaffected
    bad = np.array([[0, 1, 1, 1], [0, 4, 0, 0], [1, 0, 0, 0]], np.int32)
    with pytest.raises(o.P3DError):
        run([view(np.ones((4, 4, 4), np.float32), 16, O.ProjCamera())], 4, bad)
    f, _ = run([view(np.ones((4, 4, 4), np.float32), 16, O.ProjCamera())], 4, bad[:1])
    assert torch.all(f == 1.0)


def test_host_api_transcript_equals_reference(tmp_path):
    """tests/cpp/projection_check.cpp built against this library's
    include/pixal3d/projection.h prints exactly what the same program built
    against the reference printed (tests/golden/projection_check_reference.txt:
    features to 9 significant digits, validity flags, bridge rows, and the
    refusal messages)."""
    import subprocess
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    pkg = repo / "pixal3d" / "cpp_b200"
    exe = tmp_path / "projection_check"
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{pkg / 'host' / 'include'}",
                    str(repo / "tests" / "cpp" / "projection_check.cpp"), f"-L{pkg}", "-lpixal3d_b200", "-lp3dcuda",
                    f"-Wl,-rpath,{pkg}", "-o", str(exe)], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    want = (FX.GOLDEN / "projection_check_reference.txt").read_text().splitlines()
    got = r.stdout.splitlines()
    assert len(got) == len(want)
    for g, w in zip(got, want):
        assert g == w, (g[:120], w[:120])
