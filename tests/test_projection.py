"""Projection conditioning (image_attn_mode=proj producer, src/projection.cpp)
on the CPU: the numpy restatement in oracle/oracle.py pinned to the
reference's fixture (tests/projection_numeric_fixture.cpp output, committed as
tests/golden/projection_numeric_fixture.txt), to its known-answer checks
(tests/test_projection.cpp), and to seeded vectors from the compiled reference
(tests/golden/projection_vectors.npz).  Tolerances are the reference
comparator's (scripts/compare_projection.py:23-29): features and matrices
2e-5 max-abs and 2e-6 relative L2; validity flags exact.  The CUDA kernel is
checked against the same restatement in tests/test_gpu_projection.py."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import _fixtures as FX

GOLD = FX.GOLDEN / "projection_vectors.npz"
ABS_TOL, L2_TOL = 2e-5, 2e-6


def close(a, b, abs_tol=ABS_TOL, l2_tol=L2_TOL):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    assert a.shape == b.shape, (a.shape, b.shape)
    d = a - b
    assert np.abs(d).max() <= abs_tol, np.abs(d).max()
    assert np.linalg.norm(d) <= l2_tol * max(np.linalg.norm(b), 1e-12)


def fixture_map(base):
    """The fixture's 5x4x3 map: base + 0.125 i + 0.03125 (i % 7), float32."""
    i = np.arange(60)
    v = (np.float32(base) + np.float32(0.125) * i.astype(np.float32)).astype(np.float32)
    return (v + np.float32(0.03125) * (i % 7).astype(np.float32)).astype(np.float32).reshape(5, 4, 3)


TRANSLATED = np.array([1, 0, 0, 0.5, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1], np.float32)


def test_reference_fixture():
    g = FX.parse_golden("projection_numeric_fixture")
    cam = O.ProjCamera(0.8, 2.25, 1.5)
    f, v = O.project_features_average([fixture_map(-0.5)], 4, 16, [cam])
    close(f, g["single_features"])
    np.testing.assert_array_equal(v, g["single_valid"])
    moved = O.ProjCamera(0.8, 2.25, 1.5, TRANSLATED)
    f, v = O.project_features_average([fixture_map(-0.5), fixture_map(0.75)], 4, 16, [cam, moved])
    close(f, g["average_features"])
    np.testing.assert_array_equal(v, g["average_valid"])
    eye = np.eye(4, dtype=np.float32).reshape(16)
    rel = O.relative_calc_matrices([eye, TRANSLATED], [2.25, 2.25])
    close(np.concatenate(rel), g["relative_matrices"])


def test_reference_known_answers():
    """The checks of tests/test_projection.cpp, restated."""
    const = np.full((2, 2, 3), 4.25, np.float32)
    f, _ = O.project_features_average([const], 3, 8, [O.ProjCamera(1.0, 2.0)])
    assert f.shape == (27, 3) and np.all(np.abs(f - 4.25) <= 1e-6)
    # sparse path == dense path at the requested cells, caller order kept
    m = np.array([[[100 * y + 10 * x + c for c in range(2)] for x in range(4)] for y in range(3)], np.float32)
    cam = O.ProjCamera(1.1, 2.3, 0.9)
    dense, dvalid = O.project_features_average([m], 4, 8, [cam])
    coords = np.array([[0, 3, 1, 2], [0, 0, 0, 0], [0, 3, 1, 2], [0, 2, 3, 1]], np.int32)
    sf, sv = O.project_features_at_coords(m, 4, 8, cam, coords)
    idx = (coords[:, 1] * 4 + coords[:, 2]) * 4 + coords[:, 3]
    np.testing.assert_array_equal(sf, dense[idx])
    np.testing.assert_array_equal(sv, dvalid[idx])
    # one-point grid samples the canonical image centre of a 2x2 map
    center, _ = O.project_features_average([np.array([0, 2, 4, 6], np.float32).reshape(2, 2, 1)], 1, 8,
                                           [O.ProjCamera(1.0, 2.0)])
    assert abs(center[0, 0] - 3.75) <= 1e-5
    a, b = np.full((2, 2, 1), 2.0, np.float32), np.full((2, 2, 1), 6.0, np.float32)
    avg, _ = O.project_features_average([a, b], 1, 8, [O.ProjCamera(1.0, 2.0)] * 2)
    assert abs(avg[0, 0] - 4.0) <= 1e-6
    eye = np.eye(4, dtype=np.float32).reshape(16)
    t = eye.copy()
    t[3] = 0.5
    rel = O.relative_calc_matrices([eye, t], [2.0, 2.0])
    np.testing.assert_allclose(rel[0], O.front_matrix(2.0), atol=1e-6)
    assert abs(rel[1][3] - 0.5) <= 1e-6
    with pytest.raises(ValueError, match="grid_resolution must be positive"):
        O.project_features_at_coords(m, 0, 8, cam, coords)


def test_restatement_errors():
    m = np.zeros((2, 2, 1), np.float32)
    with pytest.raises(ValueError, match="outside the requested grid"):
        O.project_features_at_coords(m, 4, 8, O.ProjCamera(), np.array([[1, 0, 0, 0]], np.int32))
    with pytest.raises(ValueError, match="outside the requested grid"):
        O.project_features_at_coords(m, 4, 8, O.ProjCamera(), np.array([[0, 0, 4, 0]], np.int32))
    with pytest.raises(ValueError, match="camera_angle_x"):
        O.projection_constants(O.ProjCamera(camera_angle_x=4.0), 8)
    with pytest.raises(ValueError, match="singular"):
        O.projection_constants(O.ProjCamera(transform=np.zeros(16, np.float32)), 8)
    with pytest.raises(ValueError, match="counts must match"):
        O.relative_calc_matrices([np.eye(4, dtype=np.float32).reshape(16)], [1.0, 2.0])


def test_reference_vectors():
    v = np.load(GOLD)
    coords, fmap = v["coords"], v["fmap"]
    f, val = O.project_features_at_coords(fmap, 64, 518, O.ProjCamera(0.6, 2.0, 1.0), coords)
    np.testing.assert_array_equal(f, v["front_feats"])
    np.testing.assert_array_equal(val, v["front_valid"])
    f, val = O.project_features_at_coords(fmap, 64, 518, O.ProjCamera(0.9, 2.0, 0.8, v["moved_c2w"]), coords)
    np.testing.assert_array_equal(f, v["moved_feats"])
    np.testing.assert_array_equal(val, v["moved_valid"])
    assert 0 < val.mean() < 1  # part of the shell behind the camera / outside the image
    cams = [O.ProjCamera(0.7, 2.2, 1.0), O.ProjCamera(0.7, 2.2, 1.0, v["avg_c2w"])]
    f, val = O.project_features_average([v["avg_map_a"], v["avg_map_b"]], 8, 64, cams)
    np.testing.assert_array_equal(f, v["avg_feats"])
    np.testing.assert_array_equal(val, v["avg_valid"])
    rel = O.relative_calc_matrices(list(v["rel_c2w"]), v["rel_dist"])
    close(np.stack(rel), v["rel_out"])


def test_relative_matrices_through_c_abi():
    """p3d_projection_relative_matrices is host math: callable without a GPU,
    bit-exact against the reference's relative matrices."""
    from pathlib import Path
    if not (Path(__file__).resolve().parent.parent / "pixal3d" / "cpp_b200" / "libp3dcuda.so").exists():
        pytest.skip("library not built")
    from pixal3d.cpp_b200 import ops
    v = np.load(GOLD)
    np.testing.assert_array_equal(ops.projection_relative_matrices(v["rel_c2w"], v["rel_dist"]), v["rel_out"])
    with pytest.raises(ops.P3DError):
        ops.projection_relative_matrices(np.zeros((1, 16), np.float32), [1.0])
