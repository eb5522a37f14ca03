"""Inputs of the reference's deterministic numeric fixtures, restated.

The reference's fixtures (tests/*_numeric_fixture.cpp in Pixal3D.cpp) build
their inputs from closed-form sequences and a name-hash `stable_value`; the
functions here rebuild the same inputs so the oracle and the CUDA path can be
run on them and compared with the fixture outputs stored in tests/golden/.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
F32 = np.float32

TEN_COORDS = np.array([
    0, 0, 0, 0, 0, 0, 0, 1, 0, 0, 1, 0, 0, 1, 1, 1, 0, 2, 2, 2,
    1, 0, 0, 0, 1, 0, 1, 0, 1, 1, 1, 1, 1, 2, 1, 2, 1, 3, 3, 3,
], dtype=np.int32).reshape(10, 4)


def parse_golden(name: str) -> dict:
    """Parse `name count v0 v1 ...` lines of a fixture's stdout."""
    out = {}
    for line in (GOLDEN / f"{name}.txt").read_text().splitlines():
        parts = line.split()
        if not parts:
            continue
        count = int(parts[1])
        vals = np.array([float(v) for v in parts[2:]], dtype=np.float64)
        assert vals.size == count, line[:60]
        out[parts[0]] = vals
    return out


def seq(count: int, offset: float, step: float) -> np.ndarray:
    """offset + step * i in float32 (fixture `sequence`)."""
    i = np.arange(count, dtype=F32)
    return (F32(offset) + F32(step) * i).astype(F32)


def stable_value(name: str, index: np.ndarray, rule: str) -> np.ndarray:
    """Fixture parameter generator: ((index + sum((i+1)*ord(c))) % 29 - 14) * 0.018,
    with the gamma rule (|v| + 0.5 for names ending in 'gamma') used by the
    transformer/flow fixtures or the norm rule (+1 for names ending in
    'norm.weight') used by the decoder fixture."""
    stable = sum((i + 1) * ord(ch) for i, ch in enumerate(name))
    v = ((np.asarray(index, dtype=np.int64) + stable) % 29).astype(F32)
    v = ((v - F32(14.0)) * F32(0.018)).astype(F32)
    if rule == "gamma" and name.endswith("gamma"):
        v = (np.abs(v) + F32(0.5)).astype(F32)
    if rule == "norm" and name.endswith("norm.weight"):
        v = (v + F32(1.0)).astype(F32)
    return v


def param(name: str, count: int, rule: str = "gamma") -> np.ndarray:
    return stable_value(name, np.arange(count), rule)


def conv_param(name: str, cout: int, cin: int) -> np.ndarray:
    """Decoder fixture conv weights: torch [out, kd, kh, kw, in] order mapped
    to the compact [kernel, out, in] layout."""
    w = np.zeros((27, cout, cin), dtype=F32)
    for kd in range(3):
        for kh in range(3):
            for kw in range(3):
                k = kd * 9 + kh * 3 + kw
                o = np.arange(cout)[:, None]
                i = np.arange(cin)[None, :]
                src = ((o * 3 + kd) * 3 + kh) * 3 * cin + kw * cin + i
                w[k] = stable_value(name, src, "norm")
    return w


def block_params(prefix: str, C: int, ctx: int, proj: int, mlp: int) -> dict:
    """SparseTransformerBlockWeightsF32 of the transformer / flow fixtures."""
    cp = prefix + "cross_attn.cross_attn_block."
    return {
        "modulation": param(prefix + "modulation", 6 * C),
        "self_to_qkv_weight": param(prefix + "self_attn.to_qkv.weight", 3 * C * C).reshape(3 * C, C),
        "self_to_qkv_bias": param(prefix + "self_attn.to_qkv.bias", 3 * C),
        "self_q_gamma": param(prefix + "self_attn.q_rms_norm.gamma", C),
        "self_k_gamma": param(prefix + "self_attn.k_rms_norm.gamma", C),
        "self_to_out_weight": param(prefix + "self_attn.to_out.weight", C * C).reshape(C, C),
        "self_to_out_bias": param(prefix + "self_attn.to_out.bias", C),
        "norm2_weight": param(prefix + "norm2.weight", C),
        "norm2_bias": param(prefix + "norm2.bias", C),
        "cross_to_q_weight": param(cp + "to_q.weight", C * C).reshape(C, C),
        "cross_to_q_bias": param(cp + "to_q.bias", C),
        "cross_to_kv_weight": param(cp + "to_kv.weight", 2 * C * ctx).reshape(2 * C, ctx),
        "cross_to_kv_bias": param(cp + "to_kv.bias", 2 * C),
        "cross_q_gamma": param(cp + "q_rms_norm.gamma", C),
        "cross_k_gamma": param(cp + "k_rms_norm.gamma", C),
        "cross_to_out_weight": param(cp + "to_out.weight", C * C).reshape(C, C),
        "cross_to_out_bias": param(cp + "to_out.bias", C),
        "proj_weight": param(prefix + "cross_attn.proj_linear.weight", C * proj).reshape(C, proj),
        "proj_bias": param(prefix + "cross_attn.proj_linear.bias", C),
        "mlp0_weight": param(prefix + "mlp.mlp.0.weight", mlp * C).reshape(mlp, C),
        "mlp0_bias": param(prefix + "mlp.mlp.0.bias", mlp),
        "mlp2_weight": param(prefix + "mlp.mlp.2.weight", C * mlp).reshape(C, mlp),
        "mlp2_bias": param(prefix + "mlp.mlp.2.bias", C),
    }


def sparse_fixture():
    """Inputs of sparse_numeric_fixture.cpp (10 points, 2 batches, 4^3)."""
    d = {}
    d["coords"] = TEN_COORDS
    d["x"] = seq(30, -0.31, 0.047).reshape(10, 3)
    d["lin_w"] = seq(12, -0.11, 0.013).reshape(4, 3)
    d["lin_b"] = np.array([-0.07, 0.02, 0.11, 0.20], F32)
    d["conv_w"] = seq(27 * 12, -0.021, 0.0017).reshape(27, 4, 3)
    d["conv_b"] = np.array([-0.03, 0.01, 0.05, 0.09], F32)
    d["gamma"] = np.array([0.8, 1.1, 1.4], F32)
    d["beta"] = np.array([-0.2, 0.03, 0.17], F32)
    d["q"] = seq(120, -0.23, 0.017).reshape(10, 12)
    d["k"] = seq(120, 0.17, -0.021).reshape(10, 12)
    d["v"] = seq(120, -0.13, 0.031).reshape(10, 12)
    d["rms_gamma"] = seq(12, 0.7, 0.013)
    d["ctx_offsets"] = np.array([0, 3, 5], np.int64)
    d["ctx_k"] = seq(60, 0.09, -0.014).reshape(5, 12)
    d["ctx_v"] = seq(60, -0.18, 0.022).reshape(5, 12)
    d["packed_coords"] = np.array([0, 0, 0, 0, 0, 1, 0, 1, 1, 0, 1, 0], np.int32).reshape(3, 4)
    d["packed"] = seq(48, -0.17, 0.011).reshape(3, 16)
    d["subdiv"] = np.array([1, 0, 1, 0, 0, 1, 0, 0, 0, 1, 1, 0, 1, 0, 0, 1, 1, 1, 0, 0, 0, 0, 1, 0],
                           F32).reshape(3, 8)
    return d


def flow_fixture():
    """Inputs of slat_flow_numeric_fixture.cpp (one block, C=12, proj mode)."""
    C, ctx, proj, mlp = 12, 5, 7, 18
    w = {
        "input_weight": param("input_layer.weight", C * 12).reshape(C, 12),
        "input_bias": param("input_layer.bias", C),
        "timestep_weight0": param("t_embedder.mlp.0.weight", C * 256).reshape(C, 256),
        "timestep_bias0": param("t_embedder.mlp.0.bias", C),
        "timestep_weight2": param("t_embedder.mlp.2.weight", C * C).reshape(C, C),
        "timestep_bias2": param("t_embedder.mlp.2.bias", C),
        "modulation_weight": param("adaLN_modulation.1.weight", 6 * C * C).reshape(6 * C, C),
        "modulation_bias": param("adaLN_modulation.1.bias", 6 * C),
        "output_weight": param("out_layer.weight", 12 * C).reshape(12, C),
        "output_bias": param("out_layer.bias", 12),
        "blocks": [block_params("blocks.0.", C, ctx, proj, mlp)],
    }
    inputs = {
        "coords": TEN_COORDS,
        "x": seq(120, -0.27, 0.013).reshape(10, 12),
        "proj": seq(70, 0.19, -0.017).reshape(10, 7),
        "ctx_offsets": np.array([0, 3, 5], np.int64),
        "ctx": seq(25, -0.11, 0.021).reshape(5, 5),
        "timesteps": np.array([0.17, -0.23], F32),
    }
    return w, inputs


def decoder_fixture():
    """Inputs of slat_decoder_numeric_fixture.cpp (3 levels, pred_subdiv)."""
    def p(name, count):
        return stable_value(name, np.arange(count), "norm")

    def convnext(prefix, c, mlp):
        return {
            "norm_w": p(prefix + ".norm.weight", c), "norm_b": p(prefix + ".norm.bias", c),
            "conv_w": conv_param(prefix + ".conv.weight", c, c), "conv_b": p(prefix + ".conv.bias", c),
            "mlp0_w": p(prefix + ".mlp.0.weight", mlp * c).reshape(mlp, c), "mlp0_b": p(prefix + ".mlp.0.bias", mlp),
            "mlp2_w": p(prefix + ".mlp.2.weight", c * mlp).reshape(c, mlp), "mlp2_b": p(prefix + ".mlp.2.bias", c),
        }

    def c2s(prefix, c, co):
        return {
            "norm1_w": p(prefix + ".norm1.weight", c), "norm1_b": p(prefix + ".norm1.bias", c),
            "conv1_w": conv_param(prefix + ".conv1.weight", co * 8, c), "conv1_b": p(prefix + ".conv1.bias", co * 8),
            "conv2_w": conv_param(prefix + ".conv2.weight", co, co), "conv2_b": p(prefix + ".conv2.bias", co),
            "subdiv_w": p(prefix + ".to_subdiv.weight", 8 * c).reshape(8, c), "subdiv_b": p(prefix + ".to_subdiv.bias", 8),
        }

    w = {
        "from_latent_w": p("from_latent.weight", 8 * 3).reshape(8, 3), "from_latent_b": p("from_latent.bias", 8),
        "output_w": p("output_layer.weight", 3 * 4).reshape(3, 4), "output_b": p("output_layer.bias", 3),
        "blocks": [convnext("blocks.0.0", 8, 32), c2s("blocks.0.1", 8, 8), convnext("blocks.1.0", 8, 32),
                   c2s("blocks.1.1", 8, 4), convnext("blocks.2.0", 4, 16)],
    }
    cfg = {"model_channels": [8, 8, 4], "num_blocks": [1, 1, 1], "norm_eps": 1e-6, "pred_subdiv": True,
           "out_channels": 3}
    coords = np.array([[0, 0, 0, 0], [0, 1, 0, 1]], np.int32)
    x = seq(6, -0.21, 0.037).reshape(2, 3)
    return w, cfg, coords, x
