"""GPU parity of the device-resident SLat decoder (p3d_decoder_*).

- The reference's decoder fixture (3 levels, predicted subdivision): output
  coordinates bit-exact, features and subdivision logits within the
  north-star bound, and the coordinates of slat_decoder_upsample_coords_f32
  after each level.
- A wider decoder (C = 128 -> 64 -> 32) on a sphere shell against the oracle.
  The first subdivision decision depends on logits computed with 16-bit
  operands, so that case runs with guided subdivision: the guides are the
  oracle's own predicted logits, and both sides take the same topology.
  Integer topology must then match exactly.
The predicted-subdivision path at this size is checked on its first level
only, the level-0 logits, before any topology divergence.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords
from tests import _fixtures as FX

pytestmark = pytest.mark.gpu


def check(a, e, what, max_abs=2e-2, rel_l2=5e-3):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    assert a.shape == e.shape, (what, a.shape, e.shape)
    mx = float(np.abs(a - e).max()) if a.size else 0.0
    rl = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)) if a.size else 0.0
    assert mx <= max_abs and rl <= rel_l2, f"{what}: max_abs {mx:.3e} rel_l2 {rl:.3e}"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_decoder_fixture_matches_reference():
    from pixal3d.cpp_b200.decoder import Decoder
    g = FX.parse_golden("slat_decoder_numeric_fixture")
    w, cfg, coords, x = FX.decoder_fixture()
    d = Decoder(cfg["model_channels"], cfg["num_blocks"], 3, cfg["out_channels"], w, pred_subdiv=True)
    oc, feats, preds = d.run(dev(coords), dev(x), 1, (2, 2, 2))
    np.testing.assert_array_equal(oc.cpu().numpy().ravel(), g["slat_decoder_coords"].astype(np.int32))
    check(feats.cpu().numpy().ravel(), g["slat_decoder_output"], "decoder output")
    check(preds[0].cpu().numpy().ravel(), g["slat_decoder_subdiv_0_output"], "subdiv 0")
    check(preds[1].cpu().numpy().ravel(), g["slat_decoder_subdiv_1_output"], "subdiv 1")
    for level in range(3):
        c, h, _ = d.run(dev(coords), dev(x), 1, (2, 2, 2), stop_level=level)
        np.testing.assert_array_equal(c.cpu().numpy().ravel(), g[f"slat_decoder_upsample_coords_{level}"].astype(np.int32))
    d.close()


def _wide_decoder(rng, chans=(128, 64, 32), latent=8, out=16, mlp_ratio=4):
    def xav(o, i):
        a = math.sqrt(6.0 / (o + i))
        return rng.uniform(-a, a, (o, i)).astype(np.float32)

    def conv(o, i):
        return (rng.standard_normal((27, o, i)) / math.sqrt(27 * i)).astype(np.float32)

    def vec(n, s=0.05, m=0.0):
        return (m + rng.standard_normal(n) * s).astype(np.float32)

    blocks = []
    for level, c in enumerate(chans):
        blocks.append({"norm_w": vec(c, 0.05, 1.0), "norm_b": vec(c), "conv_w": conv(c, c), "conv_b": vec(c),
                       "mlp0_w": xav(mlp_ratio * c, c), "mlp0_b": vec(mlp_ratio * c), "mlp2_w": xav(c, mlp_ratio * c),
                       "mlp2_b": vec(c)})
        if level + 1 < len(chans):
            o = chans[level + 1]
            blocks.append({"norm1_w": vec(c, 0.05, 1.0), "norm1_b": vec(c), "conv1_w": conv(8 * o, c),
                           "conv1_b": vec(8 * o), "conv2_w": conv(o, o), "conv2_b": vec(o),
                           "subdiv_w": xav(8, c), "subdiv_b": vec(8, 0.5)})
    w = {"from_latent_w": xav(chans[0], latent), "from_latent_b": vec(chans[0]), "output_w": xav(out, chans[-1]),
         "output_b": vec(out), "blocks": blocks}
    cfg = {"model_channels": list(chans), "num_blocks": [1] * len(chans), "norm_eps": 1e-6, "pred_subdiv": True,
           "out_channels": out}
    return w, cfg


def test_wide_decoder_guided_matches_oracle():
    from pixal3d.cpp_b200.decoder import Decoder
    rng = np.random.default_rng(11)
    w, cfg = _wide_decoder(rng)
    coords = shell_coords(16, 5.0, 1.0)
    x = rng.standard_normal((coords.shape[0], 8)).astype(np.float32)
    oc_ref, out_ref, preds_ref = O.decoder_forward(coords, x, cfg, w)
    # guided run: the oracle's predicted logits decide the subdivision on both sides
    cfg_g = dict(cfg, pred_subdiv=False)
    oc2, out2, _ = O.decoder_forward(coords, x, cfg_g, w, guides=preds_ref)
    np.testing.assert_array_equal(oc2, oc_ref)
    d = Decoder(cfg["model_channels"], cfg["num_blocks"], 8, cfg["out_channels"], w, pred_subdiv=False)
    oc, feats, _ = d.run(dev(coords), dev(x), 1, (16, 16, 16), guides=[dev(p) for p in preds_ref])
    np.testing.assert_array_equal(oc.cpu().numpy(), oc_ref)
    assert oc.shape[0] > 4 * coords.shape[0]
    check(feats.cpu().numpy(), out_ref, "wide decoder output")
    d.close()
    # predicted-subdivision path: level-0 logits agree before any topology divergence
    dp = Decoder(cfg["model_channels"], cfg["num_blocks"], 8, cfg["out_channels"], w, pred_subdiv=True)
    c1, h1, _ = dp.run(dev(coords), dev(x), 1, (16, 16, 16), stop_level=1)
    _, _, preds = dp.run(dev(coords), dev(x), 1, (16, 16, 16))
    check(preds[0].cpu().numpy(), preds_ref[0], "level-0 subdivision logits", max_abs=2e-2 * max(
        1.0, float(np.abs(preds_ref[0]).max())))
    # stopped run: the hidden state entering level 1 on the device's own topology
    assert c1.shape[0] == h1.shape[0] and h1.shape[1] == cfg["model_channels"][1]
    dp.close()
