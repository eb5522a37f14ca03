"""SLat cascade glue (src/pipeline.cpp) on the CPU: the oracle's latent
(de)normalization and decoder-coordinate quantization against the
reference's known answers (tests/pipeline_utils_test.cpp, restated) and
against the compiled reference (oracle/_ref) on seeded inputs when that
library is present.  The CUDA kernels are checked in
tests/test_gpu_pipeline_glue.py."""
import numpy as np
import pytest

from oracle import oracle as O


def test_reference_known_answers():
    up = np.array([[0, 0, 0, 0], [0, 1, 1, 1], [0, 256, 256, 256], [0, 511, 511, 511]], np.int32)
    np.testing.assert_array_equal(O.quantize_slat_coords(up, 512), [[0, 0, 0, 0], [0, 32, 32, 32], [0, 63, 63, 63]])
    with pytest.raises(ValueError, match="must be 1024"):
        O.quantize_slat_coords(up, 512, 1536)
    with pytest.raises(ValueError, match="max_num_tokens"):
        O.quantize_slat_coords(up, 512, 1024, 2)
    x = np.array([[3.0, -1.0], [7.0, 5.0]], np.float32)
    np.testing.assert_allclose(O.normalize_slat(x, [1.0, 2.0], [2.0, 3.0]), [[1, -1], [3, 1]], atol=1e-6)
    with pytest.raises(ValueError, match="zero standard deviation"):
        O.normalize_slat(x, [1.0, 2.0], [2.0, 0.0])
    np.testing.assert_array_equal(O.denormalize_slat(O.normalize_slat(x, [1.0, 2.0], [2.0, 4.0]), [1.0, 2.0],
                                                     [2.0, 4.0]), x)


def _ref():
    from oracle import reflib
    if not reflib.available():
        pytest.skip("compiled reference (oracle/_ref) not built")
    return reflib


def test_against_compiled_reference():
    R = _ref()
    rng = np.random.default_rng(3)
    # two batch items of decoder coordinates at 256^3 (many collide on the 64^3 grid)
    c = np.concatenate([np.c_[np.zeros(3000, np.int32), rng.integers(0, 256, (3000, 3))],
                        np.c_[np.ones(2000, np.int32), rng.integers(0, 256, (2000, 3))]]).astype(np.int32)
    c = np.unique(c, axis=0).astype(np.int32)
    got = O.quantize_slat_coords(c, 256)
    np.testing.assert_array_equal(got, R.quantize_slat_coords(c, 256, batch=2, spatial=256))
    # odd low resolutions put mapped values on .5 boundaries
    for low in (63, 126, 127, 500):
        cc = np.unique(np.c_[np.zeros(4000, np.int32), rng.integers(0, low, (4000, 3))], axis=0).astype(np.int32)
        np.testing.assert_array_equal(O.quantize_slat_coords(cc, low), R.quantize_slat_coords(cc, low, spatial=low))
    x = (rng.standard_normal((c.shape[0], 8)) * 3).astype(np.float32)
    mean = rng.standard_normal(8).astype(np.float32)
    std = (np.abs(rng.standard_normal(8)) + 0.1).astype(np.float32)
    np.testing.assert_array_equal(O.normalize_slat(x, mean, std), R.normalize_slat(c, x, mean, std, batch=2,
                                                                                   shape=(256, 256, 256)))
