"""The B200 build of the reference's C++ API (include/pixal3d/sparse.h,
sparse_transformer.h, flow_sampler.h, slat_flow.h) on the reference's own
numeric fixtures: tests/cpp/host_api_check.cpp makes the same calls as the
reference's tests/*_numeric_fixture.cpp, linked against libpixal3d_b200.so,
and its outputs are compared with the fixture outputs the reference printed
(tests/golden/).  Tolerance: the north-star bound (max-abs 2e-2, relative-L2
5e-3) for 16-bit-operand kernels; 1e-5 relative for the f32 sampler math.
"""
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from tests import _fixtures as FX

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "pixal3d" / "cpp_b200"


def _write(path, arrays):
    with open(path, "wb") as f:
        for name, a in arrays.items():
            a = np.ascontiguousarray(a)
            t = {np.dtype(np.float32): 0, np.dtype(np.int32): 1, np.dtype(np.int64): 2}[a.dtype]
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)) + nb + struct.pack("<BQ", t, a.size))
            f.write(a.tobytes())


def _read(path):
    out = {}
    data = Path(path).read_bytes()
    i = 0
    while i < len(data):
        (ln,) = struct.unpack_from("<I", data, i)
        i += 4
        name = data[i:i + ln].decode()
        i += ln
        t, count = struct.unpack_from("<BQ", data, i)
        i += 9
        assert t == 0
        out[name] = np.frombuffer(data, np.float32, count, i).copy()
        i += 4 * count
    return out


def _inputs():
    a = {}
    d = FX.sparse_fixture()
    for k in ("coords", "x", "lin_w", "lin_b", "conv_w", "conv_b", "gamma", "beta", "q", "k", "v", "rms_gamma",
              "ctx_k", "ctx_v", "packed_coords", "packed", "subdiv"):
        a["sp." + k] = d[k].astype(np.int32 if k.endswith("coords") else np.float32)
    C = 12
    for k, v in FX.block_params("", C, 5, 7, 18).items():
        a["blk.w." + k] = v.astype(np.float32)
    a["blk.x"] = FX.seq(120, -0.27, 0.013)
    a["blk.proj"] = FX.seq(70, 0.19, -0.017)
    a["blk.ctx"] = FX.seq(25, -0.11, 0.021)
    a["blk.tmod"] = FX.seq(2 * 6 * C, 0.07, -0.009)
    w, inp = FX.flow_fixture()
    for k, v in w.items():
        if k != "blocks":
            a["fl." + k] = v.astype(np.float32)
    for k, v in w["blocks"][0].items():
        a["fl.b0." + k] = v.astype(np.float32)
    for k in ("x", "proj", "ctx", "timesteps"):
        a["fl." + k] = inp[k].astype(np.float32)
    # a model shape served by the device-resident flow (64-wide heads)
    from tests._models import random_flow_weights
    from oracle import oracle as O
    from pixal3d.cpp_b200.workloads import shell_coords
    hp = _device_hp()
    bw = random_flow_weights(np.random.default_rng(5), hp)
    for k, v in bw.items():
        if k != "blocks":
            a["bf." + k] = np.asarray(v, np.float32)
    for i, b in enumerate(bw["blocks"]):
        for k, v in b.items():
            a[f"bf.b{i}." + k] = np.asarray(v, np.float32)
    rng = np.random.default_rng(6)
    a["bf.hparams"] = np.array([8, 8, 128, 64, 2, 4.0, 16], np.float32)
    a["bf.coords"] = shell_coords(16, 5.5, 1.0)
    a["bf.noise"] = rng.standard_normal((a["bf.coords"].shape[0], 8)).astype(np.float32)
    a["bf.ctx"] = rng.standard_normal((33, 64)).astype(np.float32)
    a["bf.timestep"] = np.array([640.0], np.float32)
    wd, cfgd, dcoords, dx = FX.decoder_fixture()
    for k in ("from_latent_w", "from_latent_b", "output_w", "output_b"):
        a["dec." + k] = wd[k].astype(np.float32)
    for i, b in enumerate(wd["blocks"]):
        for k, v in b.items():
            a[f"dec.b{i}.{k}"] = np.asarray(v, np.float32)
    a["dec.coords"] = dcoords.astype(np.int32)
    a["dec.x"] = dx.astype(np.float32)
    a["dec.h0"] = O.linear(dx, wd["from_latent_w"], wd["from_latent_b"])
    a["fs.coords"] = np.array([[0, 0, 0, 0], [0, 0, 1, 0], [0, 2, 1, 1], [1, 0, 0, 1], [1, 1, 2, 0]], np.int32)
    a["fs.noise"] = FX.seq(15, -0.73, 0.091)
    # texture stage (the reference's tests/slat_flow_concat_fixture.cpp inputs)
    a["tx.coords"] = FX.TEN_COORDS.astype(np.int32)
    a["tx.x"] = FX.seq(120, -0.27, 0.013)
    a["tx.concat"] = FX.seq(40, 0.07, -0.011)
    a["tx.proj"] = FX.seq(70, 0.19, -0.017)
    a["tx.ctx"] = FX.seq(320, -0.11, 0.021)
    return a


def _device_hp():
    from oracle import oracle as O
    return O.FlowHParams(in_channels=8, out_channels=8, model_channels=128, cond_channels=64, num_blocks=2,
                         num_heads=2)


def _pack_weights():
    """The bf.* model's weights and the values the test pack stores for them
    (MLP matrices BF16, other matrices F16, vectors F32)."""
    from tests._models import random_flow_weights
    from tests import gguf_pack as G
    w = random_flow_weights(np.random.default_rng(5), _device_hp())
    return w, G.stored_flow_weights(w, G.GGML_F16)


def _texture_hp():
    """A texture-stage model: 12 noise channels + 4 concat channels in,
    12 out, projection conditioning with 7 channels."""
    from oracle import oracle as O
    return O.FlowHParams(in_channels=16, out_channels=12, model_channels=128, cond_channels=64, num_blocks=2,
                         num_heads=2, proj_in_channels=7, image_attn_mode="proj")


def _texture_weights():
    from tests._models import random_flow_weights
    from tests import gguf_pack as G
    w = random_flow_weights(np.random.default_rng(11), _texture_hp())
    return w, G.stored_flow_weights(w, G.GGML_F16)


def _write_texture_pack(path):
    from tests import gguf_pack as G
    w, _ = _texture_weights()
    G.write_pack(path, G.flow_metadata("texture_flow_1024", _texture_hp(), resolution=16),
                 G.flow_tensors("tx1024", w, G.GGML_F16))


def _write_flow_pack(path):
    from tests import gguf_pack as G
    w, _ = _pack_weights()
    G.write_pack(path, G.flow_metadata("shape_flow_512", _device_hp(), resolution=16),
                 G.flow_tensors("sh512", w, G.GGML_F16))


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    d = tmp_path_factory.mktemp("host_api")
    exe = d / "host_api_check"
    cmd = ["g++", "-O2", "-std=c++17", f"-I{PKG / 'host' / 'include'}", str(REPO / "tests" / "cpp" / "host_api_check.cpp"),
           f"-L{PKG}", "-lpixal3d_b200", "-lp3dcuda", f"-Wl,-rpath,{PKG}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    _write(d / "in.bin", _inputs())
    _write_flow_pack(d / "flow.gguf")
    _write_texture_pack(d / "texture.gguf")
    r = subprocess.run([str(exe), str(d / "in.bin"), str(d / "out.bin"), str(d / "flow.gguf"), str(d / "texture.gguf")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return _read(d / "out.bin")


def _close(got, exp, what, max_abs=2e-2, rel_l2=5e-3):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    assert got.shape == exp.shape, (what, got.shape, exp.shape)
    mx = float(np.abs(got - exp).max())
    rl = float(np.linalg.norm(got - exp) / max(np.linalg.norm(exp), 1e-30))
    assert mx <= max_abs and rl <= rel_l2, f"{what}: max_abs {mx:.3e} rel_l2 {rl:.3e}"


def test_sparse_operators_match_reference_fixture(harness):
    g = FX.parse_golden("sparse_numeric_fixture")
    for k in ("sparse_linear_output", "sparse_conv_output", "sparse_norm_output", "sparse_downsample_output",
              "sparse_attention_output", "sparse_rope_output", "sparse_rms_output", "sparse_cross_output",
              "sparse_channel_to_spatial_output"):
        _close(harness[k], g[k], k)
    for k in ("sparse_downsample_coords", "sparse_channel_to_spatial_coords"):
        np.testing.assert_array_equal(harness[k], g[k])


def test_transformer_block_matches_reference_fixture(harness):
    g = FX.parse_golden("sparse_transformer_numeric_fixture")
    _close(harness["sparse_transformer_output"], g["sparse_transformer_output"], "block")


def test_slat_flow_matches_reference_fixture(harness):
    g = FX.parse_golden("slat_flow_numeric_fixture")
    np.testing.assert_array_equal(harness["slat_flow_coords"], g["slat_flow_coords"])
    _close(harness["slat_flow_output"], g["slat_flow_output"], "flow forward")
    _close(harness["slat_flow_model_forward"], g["slat_flow_output"], "SLatFlowModel::forward")
    _close(harness["slat_flow_sample_direct"], g["slat_flow_sample_direct"], "sample (trajectory loop)")
    _close(harness["slat_flow_sample_direct_x0_last"], g["slat_flow_sample_direct_x0_last"], "sample x0")
    _close(harness["slat_flow_sample_device"], g["slat_flow_sample_direct"], "sample (device loop)")


def test_flow_sampler_matches_reference_fixture(harness):
    g = FX.parse_golden("flow_sampler_numeric_fixture")
    scale = max(1.0, float(np.abs(g["flow_sampler_samples"]).max()))
    for k in ("flow_sampler_samples", "flow_sampler_pred_x_t_last", "flow_sampler_pred_x_0_last"):
        _close(harness[k], g[k], k, max_abs=1e-5 * scale, rel_l2=1e-5)


def test_device_resident_flow_through_host_api(harness):
    """SLatFlowModel::forward / ::sample on a model the device-resident flow
    serves (C = 128, 64-wide heads): batched-CFG device sampler == the
    oracle's flow_euler_sample with the zero condition."""
    from oracle import oracle as O
    from tests._models import random_flow_weights
    a = _inputs()
    hp = _device_hp()
    w = random_flow_weights(np.random.default_rng(5), hp)
    c, x, ctx = a["bf.coords"], a["bf.noise"], a["bf.ctx"]
    one = np.array([0, ctx.shape[0]], np.int64)
    exp = O.slat_flow_forward(c, x, a["bf.timestep"], one, ctx, None, hp, w)
    _close(harness["device_flow_forward"], exp.ravel(), "device forward")
    sc = O.SamplerConfig(steps=4, guidance_strength=3.0, rescale_t=3.0)
    zctx = np.zeros_like(ctx)

    def model(state, t, cond):
        return O.slat_flow_forward(c, state, np.array([t], np.float32), one, ctx if cond else zctx, None, hp, w)

    exp_s = O.flow_euler_sample(x, sc, model, c[:, 0].astype(np.int64), 1)
    _close(harness["device_flow_sample"], exp_s.ravel(), "device sample")


def test_slat_decoder_matches_reference_fixture(harness):
    """slat_decoder_forward_f32, SLatDecoderModel::decode / ::upsample_coords
    and the single-block functions through the host API."""
    from oracle import oracle as O
    g = FX.parse_golden("slat_decoder_numeric_fixture")
    np.testing.assert_array_equal(harness["slat_decoder_coords"], g["slat_decoder_coords"])
    _close(harness["slat_decoder_output"], g["slat_decoder_output"], "decoder output")
    _close(harness["slat_decoder_model_output"], g["slat_decoder_output"], "SLatDecoderModel::decode")
    _close(harness["slat_decoder_subdiv_0_output"], g["slat_decoder_subdiv_0_output"], "subdiv 0")
    _close(harness["slat_decoder_subdiv_1_output"], g["slat_decoder_subdiv_1_output"], "subdiv 1")
    for level in range(3):
        k = f"slat_decoder_upsample_coords_{level}"
        np.testing.assert_array_equal(harness[k], g[k])
    w, cfg, coords, x = FX.decoder_fixture()
    h0 = O.linear(x, w["from_latent_w"], w["from_latent_b"])
    _close(harness["dec_convnext_output"], O.convnext_block(coords, h0, w["blocks"][0], 1e-6).ravel(), "convnext")
    cc, hh, pp = O.resblock_c2s(coords, h0, w["blocks"][1], 1e-6, 8, True)
    np.testing.assert_array_equal(harness["dec_c2s_coords"], cc.ravel())
    _close(harness["dec_c2s_output"], hh.ravel(), "c2s block")
    _close(harness["dec_c2s_subdiv"], pp.ravel(), "c2s predicted subdivision")


def test_flow_gguf_pack_through_host_api(harness):
    """SLatFlowModel::load of a GGUF v3 pack (compact-v1 names, F16 matrices,
    F32 vectors): hyperparameters and tensor index from the header, loading
    without data refuses forward, a missing component is refused, and the
    loaded model's forward matches the oracle on the pack's stored values."""
    from oracle import oracle as O
    info = harness["gguf_info"]
    hp = _device_hp()
    n_tensors = 10 + 21 * hp.num_blocks  # cross mode: no proj_linear
    np.testing.assert_array_equal(info, [n_tensors, 0, 1, 1, 0, hp.model_channels, hp.num_blocks, hp.num_heads,
                                         hp.cond_channels, hp.mlp_ratio, 16])
    assert harness["gguf_no_data_forward_refused"][0] == 1
    assert harness["gguf_missing_component_refused"][0] == 1
    a = _inputs()
    _, st = _pack_weights()
    c, x, ctx = a["bf.coords"], a["bf.noise"], a["bf.ctx"]
    one = np.array([0, ctx.shape[0]], np.int64)
    exp = O.slat_flow_forward(c, x, a["bf.timestep"], one, ctx, None, hp, st)
    _close(harness["gguf_flow_forward"], exp.ravel(), "GGUF-loaded forward")


def test_texture_stage_concat_and_projection_through_host_api(harness):
    """The calls of the reference's tests/slat_flow_concat_fixture.cpp on a
    texture_flow_1024 pack (concat condition + projection mode): forward with
    [input | concat], then a 3-step sampler run, against the oracle on the
    pack's stored values."""
    from oracle import oracle as O
    hp = _texture_hp()
    _, st = _texture_weights()
    a = _inputs()
    c = a["tx.coords"]
    x = a["tx.x"].reshape(10, 12)
    cat = a["tx.concat"].reshape(10, 4)
    proj = a["tx.proj"].reshape(10, 7)
    ctx = a["tx.ctx"].reshape(5, 64)
    offs = np.array([0, 3, 5], np.int64)
    ts = np.array([0.17, -0.23], np.float32)
    exp = O.slat_flow_forward(c, np.concatenate([x, cat], 1), ts, offs, ctx, proj, hp, st)
    _close(harness["tx_concat_forward"], exp.ravel(), "texture forward with concat")
    sc = O.SamplerConfig(steps=3, sigma_min=0.031, rescale_t=2.7, guidance_strength=1.0, guidance_rescale=0.0,
                         guidance_interval_min=0.0, guidance_interval_max=1.0)

    def ref_model(state, t, cond):
        return O.slat_flow_forward(c, np.concatenate([state, cat], 1).astype(np.float32), np.array([t, t], np.float32),
                                   offs, ctx if cond else np.zeros_like(ctx), proj if cond else np.zeros_like(proj),
                                   hp, st)

    exp = O.flow_euler_sample(x, sc, ref_model, c[:, 0].astype(np.int64), 2)
    _close(harness["tx_concat_sample"], exp.ravel(), "texture sample with concat")
    # run_slat_stage_f32: the same sampling, then latent * std + mean
    mean = (0.25 * np.arange(12) - 1.0).astype(np.float32)
    std = (0.5 + 0.125 * np.arange(12)).astype(np.float32)
    got = harness["tx_stage_latent"].reshape(10, 12)
    np.testing.assert_array_equal(got, O.denormalize_slat(harness["tx_concat_sample"].reshape(10, 12), mean, std))
    _close(got.ravel(), O.denormalize_slat(exp, mean, std).ravel(), "texture stage latent")
    assert harness["tx_concat_mismatch_refused"][0] == 1


def test_pipeline_utils_reference_checks(harness):
    """tests/pipeline_utils_test.cpp's assertions through this library's
    pipeline.h: quantization known answer and refusals, normalization known
    answer and the zero-std refusal."""
    np.testing.assert_array_equal(harness["pipeline_utils"], np.ones(6, np.float32))
