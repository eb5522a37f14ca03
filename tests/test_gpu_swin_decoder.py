"""GPU parity of the config-3 shifted-window SLat decoder (SwinDecoder; no
reference implementation, checked against oracle.swin_decoder_forward).

A reduced configuration keeps the oracle to seconds: C0 = 128 (2 heads x
64), 2 blocks (shift 0 and 4), window 8^3 on a 32^3 shell, stages to 64 and
32 channels (the C = 32 stage exercises the zero-padded conv input and the
one-channel GroupNorm groups), 16 output channels, seeded Bernoulli(0.5)
subdivision masks.  Coordinates bit-exact; features within the north-star
bound (max-abs 2e-2, relative-L2 5e-3).
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords

pytestmark = pytest.mark.gpu


def make_weights(rng, c0=128, stages=(64, 32), latent=8, out=16, blocks=2, mlp_ratio=4):
    def xav(o, i):
        a = math.sqrt(6.0 / (o + i))
        return rng.uniform(-a, a, (o, i)).astype(np.float32)

    def vec(n, s=0.05, m=0.0):
        return (m + rng.standard_normal(n) * s).astype(np.float32)

    def conv(o, i):
        return (rng.standard_normal((27, o, i)) / math.sqrt(27 * i)).astype(np.float32)

    w = {"from_latent_w": xav(c0, latent), "from_latent_b": vec(c0), "blocks": [], "stages": []}
    for _ in range(blocks):
        w["blocks"].append({"norm1_w": vec(c0, 0.05, 1.0), "norm1_b": vec(c0), "qkv_w": xav(3 * c0, c0),
                            "qkv_b": vec(3 * c0), "out_w": xav(c0, c0), "out_b": vec(c0),
                            "norm2_w": vec(c0, 0.05, 1.0), "norm2_b": vec(c0), "mlp0_w": xav(mlp_ratio * c0, c0),
                            "mlp0_b": vec(mlp_ratio * c0), "mlp2_w": xav(c0, mlp_ratio * c0), "mlp2_b": vec(c0)})
    ci = c0
    for co in stages:
        w["stages"].append({"gn1_w": vec(ci, 0.05, 1.0), "gn1_b": vec(ci), "conv1_w": conv(co, ci), "conv1_b": vec(co),
                            "gn2_w": vec(co, 0.05, 1.0), "gn2_b": vec(co), "conv2_w": conv(co, co),
                            "conv2_b": vec(co), "skip_w": xav(co, ci), "skip_b": vec(co)})
        ci = co
    w["output_w"] = xav(out, ci)
    w["output_b"] = vec(out)
    return w


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
