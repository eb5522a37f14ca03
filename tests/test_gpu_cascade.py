"""The device-resident SLat cascade (pixal3d/cpp_b200/cascade.py: shape LR ->
decoder coordinate upsampling -> quantization to the 1024 grid -> shape HR
-> texture with the normalized shape latent as concat condition and
projected image features) against the oracle, stage by stage.

Each stage's oracle run starts from the device's own inputs for that stage
(coordinates, and for the texture stage the device's shape latent), so the
comparison measures one stage at a time: latents within the north-star
bound (max-abs 2e-2, relative-L2 5e-3), coordinates exact.  The decoder's
subdivision logits are its bias alone (zero weights), so the upsampled
coordinates do not depend on 16-bit rounding of the latent.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import shell_coords
from tests._models import random_flow_weights

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 5e-3


def check(a, e, what):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    mx = float(np.abs(a - e).max())
    rl = float(np.linalg.norm(a - e) / np.linalg.norm(e))
    assert mx <= MAX_ABS * max(1.0, float(np.abs(e).max())) and rl <= REL_L2, f"{what}: {mx:.3e} {rl:.3e}"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def flow(hp, seed):
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    w = random_flow_weights(np.random.default_rng(seed), hp)
    fields = {k: getattr(hp, k) for k in HParams.__dataclass_fields__ if hasattr(hp, k)}
    return w, FlowModel(HParams(**fields), w)


def decoder_weights(rng, chans, latent, out):
    def xav(o, i):
        a = math.sqrt(6.0 / (o + i))
        return rng.uniform(-a, a, (o, i)).astype(np.float32)

    def conv(o, i):
        return (rng.standard_normal((27, o, i)) / math.sqrt(27 * i)).astype(np.float32)

    def vec(n, s=0.05, m=0.0):
        return (m + rng.standard_normal(n) * s).astype(np.float32)

    keep = np.array([4, -4, 4, -4, -4, 4, -4, 4], np.float32)  # children kept: a fixed half
    blocks = []
    for level, c in enumerate(chans):
        blocks.append({"norm_w": vec(c, 0.05, 1.0), "norm_b": vec(c), "conv_w": conv(c, c), "conv_b": vec(c),
                       "mlp0_w": xav(4 * c, c), "mlp0_b": vec(4 * c), "mlp2_w": xav(c, 4 * c), "mlp2_b": vec(c)})
        if level + 1 < len(chans):
            o = chans[level + 1]
            blocks.append({"norm1_w": vec(c, 0.05, 1.0), "norm1_b": vec(c), "conv1_w": conv(8 * o, c),
                           "conv1_b": vec(8 * o), "conv2_w": conv(o, o), "conv2_b": vec(o),
                           "subdiv_w": np.zeros((8, c), np.float32), "subdiv_b": keep})
    w = {"from_latent_w": xav(chans[0], latent), "from_latent_b": vec(chans[0]), "output_w": xav(out, chans[-1]),
         "output_b": vec(out), "blocks": blocks}
    cfg = {"model_channels": list(chans), "num_blocks": [1] * len(chans), "norm_eps": 1e-6, "pred_subdiv": True,
           "out_channels": out}
    return w, cfg


def test_slat_cascade_stage_by_stage():
    from pixal3d.cpp_b200 import ops
    from pixal3d.cpp_b200.cascade import Normalization, SamplerSettings, SLatCascade, seeded_noise
    from pixal3d.cpp_b200.decoder import Decoder
    rng = np.random.default_rng(21)
    shp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=1,
                        num_heads=2)
    thp = O.FlowHParams(in_channels=16, out_channels=8, model_channels=128, cond_channels=64, num_blocks=1,
                        num_heads=2, proj_in_channels=8, image_attn_mode="proj")
    w_low, m_low = flow(shp, 31)
    w_high, m_high = flow(shp, 32)
    w_tex, m_tex = flow(thp, 33)
    dw, dcfg = decoder_weights(rng, [64, 32, 16], 8, 8)
    dec = Decoder(dcfg["model_channels"], dcfg["num_blocks"], 8, 8, dw)
    smean = rng.standard_normal(8).astype(np.float32)
    sstd = (np.abs(rng.standard_normal(8)) + 0.5).astype(np.float32)
    tmean = rng.standard_normal(8).astype(np.float32)
    tstd = (np.abs(rng.standard_normal(8)) + 0.5).astype(np.float32)
    tokens = rng.standard_normal((21, 64)).astype(np.float32)
    fmap = rng.standard_normal((37, 37, 8)).astype(np.float32)
    cam = O.ProjCamera(0.6, 2.0, 1.0)

    def condition(stage, coords, grid):
        proj = None
        if stage == "texture_slat":
            proj, _ = ops.project_features([{"feature_map": dev(fmap), "image_resolution": 518, "camera_angle_x": 0.6,
                                             "distance": 2.0, "mesh_scale": 1.0}], grid, coords)
        return dev(tokens), [0, 21], proj

    noise = seeded_noise(7)
    cas = SLatCascade(m_low, m_high, m_tex, dec, Normalization(dev(smean), dev(sstd)),
                      Normalization(dev(tmean), dev(tstd)), low_resolution=16, upsample_times=2)
    ss = SamplerSettings(steps=2, guidance_strength=2.0, rescale_t=3.0)
    ts = SamplerSettings(steps=2, guidance_strength=1.5, rescale_t=2.0)
    c0 = shell_coords(16, 5.5, 1.0)
    out = cas.run(dev(c0), noise, condition, ss, ts)

    one = np.array([0, 21], np.int64)
    zt = np.zeros_like(tokens)

    def sampled(hp, w, coords, x0, sc, proj=None, concat=None):
        def model(state, t, cond):
            xin = state if concat is None else np.concatenate([state, concat], 1).astype(np.float32)
            p = None if proj is None else (proj if cond else np.zeros_like(proj))
            return O.slat_flow_forward(coords, xin, np.array([t], np.float32), one, tokens if cond else zt, p, hp, w)
        return O.flow_euler_sample(x0, sc, model, coords[:, 0].astype(np.int64), 1)

    def oc(s):
        return O.SamplerConfig(steps=s.steps, sigma_min=s.sigma_min, rescale_t=s.rescale_t,
                               guidance_strength=s.guidance_strength, guidance_rescale=s.guidance_rescale,
                               guidance_interval_min=0.0, guidance_interval_max=1.0)

    # shape LR
    n_low = noise("shape_slat_low", dev(c0), 8, 16).cpu().numpy()
    exp = O.denormalize_slat(sampled(shp, w_low, c0, n_low, oc(ss)), smean, sstd)
    check(out["shape_slat_low"].cpu().numpy(), exp, "shape LR latent")
    # hand-off coordinates (bias-only subdivision: independent of the latent)
    dcfg2 = dict(dcfg)
    up_ref, _, _ = O.decoder_forward(c0, exp, dcfg2, dw)
    np.testing.assert_array_equal(out["shape_upsampled_coords"].cpu().numpy(), up_ref)
    high = O.quantize_slat_coords(up_ref, 64)
    np.testing.assert_array_equal(out["high_coords"].cpu().numpy(), high)
    assert high.shape[0] > 4 * c0.shape[0]
    # shape HR
    n_high = noise("shape_slat_high", dev(high), 8, 64).cpu().numpy()
    exp_h = O.denormalize_slat(sampled(shp, w_high, high, n_high, oc(ss)), smean, sstd)
    check(out["shape_slat_high"].cpu().numpy(), exp_h, "shape HR latent")
    # texture: concat = the device shape latent normalized; projected rows
    concat = O.normalize_slat(out["shape_slat_high"].cpu().numpy(), smean, sstd)
    proj, _ = O.project_features_at_coords(fmap, 64, 518, cam, high)
    n_tex = noise("texture_slat", dev(high), 8, 64).cpu().numpy()
    exp_t = O.denormalize_slat(sampled(thp, w_tex, high, n_tex, oc(ts), proj, concat), tmean, tstd)
    check(out["texture_slat"].cpu().numpy(), exp_t, "texture latent")
    for m in (m_low, m_high, m_tex):
        m.close()
    dec.close()
