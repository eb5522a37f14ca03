"""GPU parity of the config-3 shifted-window SLat decoder (SwinDecoder; no
reference implementation, checked against oracle.swin_decoder_forward).

A reduced configuration keeps the oracle to seconds: C0 = 128 (2 heads x
64), 2 blocks (shift 0 and 4), window 8^3 on a 32^3 shell, stages to 64 and
32 channels (the C = 32 stage exercises the zero-padded conv input and the
one-channel GroupNorm groups), 16 output channels, seeded Bernoulli(0.5)
subdivision masks.  Coordinates bit-exact; features within the north-star
bound (max-abs 2e-2, relative-L2 5e-3).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords

pytestmark = pytest.mark.gpu


def make_weights(rng):
    from pixal3d.cpp_b200.workloads import random_swin_weights
    return random_swin_weights(rng)


def test_swin_decoder_matches_restatement():
    from pixal3d.cpp_b200.swin_decoder import SwinDecoder
    rng = np.random.default_rng(5)
    cfg = {"model_channels": 128, "num_heads": 2, "window": 8, "spatial": 32, "groups": 32}
    w = make_weights(rng)
    coords = shell_coords(32, 10.0, 1.5)
    x = rng.standard_normal((coords.shape[0], 8)).astype(np.float32)
    m1 = (rng.random((coords.shape[0], 8)) < 0.5).astype(np.float32)
    n1 = int(m1.sum())
    m2 = (rng.random((n1, 8)) < 0.5).astype(np.float32)
    oc, out = O.swin_decoder_forward(coords, x, cfg, w, [m1, m2])
    d = SwinDecoder(cfg, w)
    gc, gout = d.run(torch.from_numpy(coords).cuda(), torch.from_numpy(x).cuda(), [m1, m2], batch=1)
    np.testing.assert_array_equal(gc.cpu().numpy(), oc)
    got = gout.cpu().numpy()
    assert got.shape == out.shape and got.shape[0] > 3 * coords.shape[0]
    err = np.abs(got - out)
    rel = float(np.linalg.norm(got - out) / np.linalg.norm(out))
    assert float(err.max()) <= 2e-2 and rel <= 5e-3, (float(err.max()), rel)
