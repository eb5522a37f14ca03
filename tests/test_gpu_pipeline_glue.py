"""p3d_slat_normalize and p3d_quantize_slat_coords (the SLat cascade glue of
src/pipeline.cpp) on the GPU against the pinned oracle: both are exact
(integer coordinates; f32 arithmetic in the reference's order), so the
comparison is equality."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def ops():
    from pixal3d.cpp_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_quantize_known_answer_and_random():
    o = ops()
    up = np.array([[0, 0, 0, 0], [0, 1, 1, 1], [0, 256, 256, 256], [0, 511, 511, 511]], np.int32)
    np.testing.assert_array_equal(o.quantize_slat_coords(dev(up), 1, 512).cpu().numpy(),
                                  [[0, 0, 0, 0], [0, 32, 32, 32], [0, 63, 63, 63]])
    rng = np.random.default_rng(4)
    for low, batch in ((256, 2), (63, 1), (127, 3), (512, 4)):
        parts = [np.c_[np.full(6000, b, np.int32), rng.integers(0, low, (6000, 3))] for b in range(batch)]
        c = np.unique(np.concatenate(parts), axis=0).astype(np.int32)
        got = o.quantize_slat_coords(dev(c), batch, low).cpu().numpy()
        np.testing.assert_array_equal(got, O.quantize_slat_coords(c, low))


def test_quantize_refusals():
    o = ops()
    c = dev(np.array([[0, 1, 2, 3]], np.int32))
    with pytest.raises(o.P3DError, match="must be 1024"):
        o.quantize_slat_coords(c, 1, 512, resolution=1536)
    with pytest.raises(o.P3DError):  # maps to 126 on the 64-grid: latched on the device
        o.quantize_slat_coords(dev(np.array([[0, 200, 0, 0]], np.int32)), 1, 100)
    np.testing.assert_array_equal(o.quantize_slat_coords(c, 1, 64).cpu().numpy(), [[0, 1, 2, 3]])


def test_normalize_and_denormalize_bit_exact():
    o = ops()
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((50000, 8)) * 3).astype(np.float32)
    mean = rng.standard_normal(8).astype(np.float32)
    std = (np.abs(rng.standard_normal(8)) + 0.1).astype(np.float32)
    xt, mt, st = dev(x), dev(mean), dev(std)
    y = o.slat_normalize(xt, mt, st)
    np.testing.assert_array_equal(y.cpu().numpy(), O.normalize_slat(x, mean, std))
    z = o.slat_normalize(y, mt, st, denormalize=True, out=y)  # in place
    np.testing.assert_array_equal(z.cpu().numpy(), O.denormalize_slat(O.normalize_slat(x, mean, std), mean, std))
    o.ctx(0).sync_check()
    big = dev(np.full((4, 8), 3e38, np.float32))
    o.slat_normalize(big, mt, dev(np.full(8, 10.0, np.float32)), denormalize=True)
    with pytest.raises(o.P3DError):
        o.ctx(0).sync_check()
