"""Pin the numpy oracle (oracle/oracle.py) to the reference.

(a) Against the reference's own deterministic fixtures, whose outputs were
    produced by the compiled reference and committed in tests/golden/*.txt.
(b) Against seeded reference vectors in tests/golden/ref_vectors.npz.
(c) Against the compiled reference library (oracle/_ref) on fresh seeded
    inputs, when that library is present (it is built where the reference is
    mounted; the GPU box gets the prebuilt .so).

Tolerances follow the reference's own comparators: sparse ops 2e-5 max-abs
(scripts/compare_sparse.py:222), composite blocks / flow 5e-4
(scripts/compare_sparse_transformer.py:127), sampler 5e-6 relative scale
(scripts/compare_flow_sampler.py:108).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import _fixtures as FX

SPARSE_TOL = 2e-5
BLOCK_TOL = 5e-4


def close(a, b, tol):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    assert a.shape == b.shape, (a.shape, b.shape)
    err = np.abs(a - b).max() if a.size else 0.0
    assert err <= tol, f"max abs err {err} > {tol}"


# ---------------------------------------------------------------- (a) fixtures

def test_sparse_numeric_fixture():
    g = FX.parse_golden("sparse_numeric_fixture")
    d = FX.sparse_fixture()
    c = d["coords"]
    bidx = c[:, 0].astype(np.int64)
    close(O.linear(d["x"], d["lin_w"], d["lin_b"]), g["sparse_linear_output"], SPARSE_TOL)
    close(O.subm_conv3d(c, d["x"], d["conv_w"], d["conv_b"]), g["sparse_conv_output"], SPARSE_TOL)
    close(O.layer_norm(d["x"], 1e-5, d["gamma"], d["beta"]), g["sparse_norm_output"], SPARSE_TOL)
    dc, df, _ = O.downsample_mean(c, d["x"], 2)
    np.testing.assert_array_equal(dc.ravel(), g["sparse_downsample_coords"].astype(np.int32))
    close(df, g["sparse_downsample_output"], SPARSE_TOL)
    close(O.sdpa(bidx, d["q"], bidx, d["k"], d["v"], 2, 6, 0.37), g["sparse_attention_output"], SPARSE_TOL)
    close(O.rope(c, d["q"], 2, 6), g["sparse_rope_output"], SPARSE_TOL)
    close(O.rms_norm_heads(d["q"], 2, 6, d["rms_gamma"]), g["sparse_rms_output"], SPARSE_TOL)
    close(O.cross_attention(bidx, d["q"], d["ctx_offsets"], d["ctx_k"], d["ctx_v"], 2, 6, 0.29),
          g["sparse_cross_output"], SPARSE_TOL)
    cc, cf = O.channel_to_spatial(d["packed_coords"], d["packed"], 2, d["subdiv"])
    np.testing.assert_array_equal(cc.ravel(), g["sparse_channel_to_spatial_coords"].astype(np.int32))
    close(cf, g["sparse_channel_to_spatial_output"], SPARSE_TOL)


def test_sparse_transformer_fixture():
    g = FX.parse_golden("sparse_transformer_numeric_fixture")
    C = 12
    w = FX.block_params("", C, 5, 7, 18)
    cfg = O.BlockConfig(channels=C, num_heads=2, mlp_hidden=18, context_channels=5, proj_in_channels=7,
                        use_projection=True)
    x = FX.seq(120, -0.27, 0.013).reshape(10, C)
    proj = FX.seq(70, 0.19, -0.017).reshape(10, 7)
    ctx = FX.seq(25, -0.11, 0.021).reshape(5, 5)
    tmod = FX.seq(2 * 6 * C, 0.07, -0.009)
    out = O.transformer_block(FX.TEN_COORDS, x, tmod, np.array([0, 3, 5]), ctx, proj, cfg, w)
    close(out, g["sparse_transformer_output"], BLOCK_TOL)


def _fixture_flow_hp():
    return O.FlowHParams(in_channels=12, out_channels=12, model_channels=12, cond_channels=5, num_blocks=1,
                         num_heads=2, mlp_ratio=1.5, proj_in_channels=7, image_attn_mode="proj")


def test_slat_flow_fixture_forward_and_sample():
    g = FX.parse_golden("slat_flow_numeric_fixture")
    w, inp = FX.flow_fixture()
    hp = _fixture_flow_hp()
    c = inp["coords"]
    out = O.slat_flow_forward(c, inp["x"], inp["timesteps"], inp["ctx_offsets"], inp["ctx"], inp["proj"], hp, w)
    np.testing.assert_array_equal(c.ravel(), g["slat_flow_coords"].astype(np.int32))
    close(out, g["slat_flow_output"], BLOCK_TOL)

    sc = O.SamplerConfig(steps=4, sigma_min=0.031, rescale_t=2.7, guidance_strength=2.0, guidance_rescale=0.23,
                         guidance_interval_min=0.34, guidance_interval_max=0.91)
    zctx = np.zeros_like(inp["ctx"])
    zproj = np.zeros_like(inp["proj"])

    def model(state, t, cond):
        ts = np.full(2, t, np.float32)
        return O.slat_flow_forward(c, state, ts, inp["ctx_offsets"], inp["ctx"] if cond else zctx,
                                   inp["proj"] if cond else zproj, hp, w)

    x, x0 = O.flow_euler_sample(inp["x"], sc, model, c[:, 0].astype(np.int64), 2, record_x0=True)
    close(x, g["slat_flow_sample_direct"], BLOCK_TOL)
    close(x0, g["slat_flow_sample_direct_x0_last"], BLOCK_TOL)


def test_flow_sampler_fixture():
    g = FX.parse_golden("flow_sampler_numeric_fixture")
    coords = np.array([[0, 0, 0, 0], [0, 0, 1, 0], [0, 2, 1, 1], [1, 0, 0, 1], [1, 1, 2, 0]], np.int32)
    noise = FX.seq(15, -0.73, 0.091).reshape(5, 3)
    sc = O.SamplerConfig(steps=6, sigma_min=0.031, rescale_t=2.7, guidance_strength=2.35, guidance_rescale=0.41,
                         guidance_interval_min=0.34, guidance_interval_max=0.91)
    ch = np.tile(np.arange(3, dtype=np.float32), (5, 1))

    def model(state, t, cond):
        cv = np.float32(0.19) if cond else np.float32(-0.07)
        return (np.float32(0.043) * state + np.float32(0.00037) * t + np.float32(0.011) * ch + cv).astype(np.float32)

    x, x0 = O.flow_euler_sample(noise, sc, model, coords[:, 0].astype(np.int64), 2, record_x0=True)
    scale = max(1.0, np.abs(g["flow_sampler_samples"]).max())
    close(x, g["flow_sampler_samples"], 5e-6 * scale)
    close(x, g["flow_sampler_pred_x_t_last"], 5e-6 * scale)
    close(x0, g["flow_sampler_pred_x_0_last"], 5e-6 * scale)


def test_slat_decoder_fixture():
    g = FX.parse_golden("slat_decoder_numeric_fixture")
    w, cfg, coords, x = FX.decoder_fixture()
    oc, out, preds = O.decoder_forward(coords, x, cfg, w)
    np.testing.assert_array_equal(oc.ravel(), g["slat_decoder_coords"].astype(np.int32))
    close(out, g["slat_decoder_output"], 1e-4)
    assert len(preds) == 2
    # Level-1 subdivision logits live on the level-1 coordinates.
    np.testing.assert_array_equal((preds[0] > 0).astype(np.float64).ravel(), g["slat_decoder_subdiv_0_active"])
    close(preds[0], g["slat_decoder_subdiv_0_output"], 1e-4)
    close(preds[1], g["slat_decoder_subdiv_1_output"], 1e-4)
    np.testing.assert_array_equal((preds[1] > 0).astype(np.float64).ravel(), g["slat_decoder_subdiv_1_active"])
    # upsample_coords: the coordinates after `level` C2S stages
    # (slat_decoder_upsample_coords_f32, src/slat_decoder.cpp:378-445).
    for level in range(3):
        cc = coords
        h = O.linear(x, w["from_latent_w"], w["from_latent_b"])
        bi = 0
        for lv in range(level):
            for _ in range(cfg["num_blocks"][lv]):
                h = O.convnext_block(cc, h, w["blocks"][bi], 1e-6)
                bi += 1
            cc, h, _ = O.resblock_c2s(cc, h, w["blocks"][bi], 1e-6, cfg["model_channels"][lv + 1], True)
            bi += 1
        np.testing.assert_array_equal(cc.ravel(), g[f"slat_decoder_upsample_coords_{level}"].astype(np.int32))


def test_timestep_frequency_fixture():
    g = FX.parse_golden("flow_numeric_fixture")
    t = np.array([-1.25, 0.0, 0.75, 2.5], np.float32)
    close(O.timestep_embedding(t, 9), g["timestep_frequency"], 2e-6)


# ---------------------------------------------------------- (b) ref_vectors

def test_ref_vectors():
    v = np.load(FX.GOLDEN / "ref_vectors.npz")
    c = v["coords"]
    bidx = c[:, 0].astype(np.int64)
    np.testing.assert_array_equal(O.neighbor_map27(c), v["nbr"])
    assert O.coords_fingerprint(c) == int(v["fingerprint"][0])
    close(O.subm_conv3d(c, v["conv_x"], v["conv_w"], v["conv_b"]), v["conv_out"], SPARSE_TOL)
    dc, df, _ = O.downsample_mean(c, v["conv_x"], 2)
    np.testing.assert_array_equal(dc, v["down_coords"])
    close(df, v["down_feats"], SPARSE_TOL)
    cc, cf = O.channel_to_spatial(c, v["c2s_x"], 2, v["c2s_mask"])
    np.testing.assert_array_equal(cc, v["c2s_coords"])
    close(cf, v["c2s_feats"], 0)
    close(O.sdpa(bidx, v["attn_q"], bidx, v["attn_k"], v["attn_v"], 2, 8, 0.35), v["attn_out"], SPARSE_TOL)
    close(O.rope(c, v["attn_q"], 2, 8), v["rope_out"], SPARSE_TOL)
    close(O.rms_norm_heads(v["attn_q"], 2, 8, v["rms_gamma"]), v["rms_out"], SPARSE_TOL)


# ------------------------------------------------------- (c) live reference

reflib = pytest.importorskip("oracle.reflib")
needs_ref = pytest.mark.skipif(not reflib.available(), reason="oracle/_ref/libp3dref.so not built")


@needs_ref
def test_live_reference_block_and_flow():
    rng = np.random.default_rng(7)
    from pixal3d.cpp_b200.workloads import shell_coords, batched
    base = shell_coords(12, 4.0, 0.9)
    coords = batched(base, 2)
    n = coords.shape[0]
    C, H, ctxc, mlp = 32, 2, 24, 64
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=C, cond_channels=ctxc, num_blocks=2,
                       num_heads=H, mlp_ratio=2.0)
    from tests._models import random_flow_weights
    w = random_flow_weights(rng, hp)
    x = rng.standard_normal((n, 8)).astype(np.float32)
    offs = np.array([0, 7, 12], np.int64)
    ctx = rng.standard_normal((12, ctxc)).astype(np.float32)
    ts = np.array([500.0, 500.0], np.float32)
    ref = reflib.slat_flow_forward(coords, x, ts, offs, ctx, None, hp, w, 2, (12, 12, 12))
    mine = O.slat_flow_forward(coords, x, ts, offs, ctx, None, hp, w)
    close(mine, ref, BLOCK_TOL)
    # sampler with CFG + rescale, 3 steps
    sc = O.SamplerConfig(steps=3, guidance_strength=3.0, guidance_rescale=0.5)
    ref_s = reflib.slat_flow_sample(coords, x, offs, ctx, None, hp, w, sc, batch=2, shape=(12, 12, 12))
    zctx = np.zeros_like(ctx)

    def model(state, t, cond):
        return O.slat_flow_forward(coords, state, np.full(2, t, np.float32), offs, ctx if cond else zctx, None, hp, w)

    mine_s = O.flow_euler_sample(x, sc, model, coords[:, 0].astype(np.int64), 2)
    close(mine_s, ref_s, 1e-3)


@needs_ref
def test_live_reference_ops():
    rng = np.random.default_rng(11)
    from pixal3d.cpp_b200.workloads import shell_coords
    c = shell_coords(20, 7.0, 1.2)
    n = c.shape[0]
    x = rng.standard_normal((n, 16)).astype(np.float32)
    w = (rng.standard_normal((27, 16, 16)) / 20).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    close(O.subm_conv3d(c, x, w, b), reflib.subm_conv3d(c, x, w, b), SPARSE_TOL)
    np.testing.assert_array_equal(O.neighbor_map27(c), reflib.neighbor_map27(c))
    lw = rng.standard_normal((24, 16)).astype(np.float32)
    close(O.linear(x, lw, b[:24] if b.size >= 24 else np.zeros(24, np.float32)),
          reflib.sparse_linear(c, x, lw, np.zeros(24, np.float32) if b.size < 24 else b[:24]), SPARSE_TOL)
    close(O.layer_norm(x, 1e-6), reflib.layer_norm(c, x, 1e-6), SPARSE_TOL)
    t = np.array([0.0, 250.0, 999.0], np.float32)
    w0 = rng.standard_normal((32, 256)).astype(np.float32) * 0.05
    w2 = rng.standard_normal((32, 32)).astype(np.float32) * 0.1
    b0 = np.zeros(32, np.float32)
    close(O.timestep_embed_mlp(t, 32, w0, b0, w2, b0), reflib.timestep_embed_mlp(t, 32, w0, b0, w2, b0), 2e-5)
    oc, of, _ = O.downsample_mean(c, x, 2)
    rc, rf, _ = reflib.downsample_mean(c, x, 2)
    np.testing.assert_array_equal(oc, rc)
    close(of, rf, SPARSE_TOL)


def validity_cases():
    """Valid and invalid sparse tensors, including rows that fail different
    checks in different orders (the first failing row decides the error)."""
    rng = np.random.default_rng(21)
    base = FX.TEN_COORDS.copy()
    x = rng.standard_normal((10, 3)).astype(np.float32)
    cases = [("valid", base, x)]
    c = base.copy(); c[6] = c[2]
    cases.append(("duplicate", c, x))
    c = base.copy(); c[4, 2] = 9
    cases.append(("outside", c, x))
    c = base.copy(); c[3] = [1, 3, 3, 3]; c[4] = [0, 3, 2, 1]
    cases.append(("batch order", c, x))
    xx = x.copy(); xx[5, 1] = np.nan
    cases.append(("nan", base, xx))
    c = base.copy(); c[7, 3] = -1; c[5] = c[1]; xx = x.copy(); xx[2, 0] = np.inf
    cases.append(("inf before duplicate before outside", c, xx))
    c = base.copy(); c[2, 1] = 99; c[8] = c[0]
    cases.append(("outside before duplicate", c, x))
    return cases


@needs_ref
def test_validate_matches_reference():
    for name, c, x in validity_cases():
        assert O.validate(c, x, 2, (4, 4, 4)) == reflib.valid(c, x, 2, (4, 4, 4)), name
