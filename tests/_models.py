"""Seeded random-init model weights for parity tests (the benchmark configs
use random init; no checkpoint is available)."""
from __future__ import annotations

import math

import numpy as np

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import xavier


def random_flow_weights(rng, hp: O.FlowHParams) -> dict:
    """Xavier-uniform linears, biases ~ N(0, 0.02), gammas ~ 1 + N(0, 0.05),
    block modulation ~ N(0, 0.1); io resblock convs ~ N(0, 1/sqrt(27 C))."""
    C = hp.model_channels
    mlp = int(C * hp.mlp_ratio)

    def bias(k):
        return (rng.standard_normal(k) * 0.02).astype(np.float32)

    def gamma(k):
        return (1.0 + rng.standard_normal(k) * 0.05).astype(np.float32)

    w = {
        "input_weight": xavier(rng, C, hp.in_channels), "input_bias": bias(C),
        "timestep_weight0": xavier(rng, C, 256), "timestep_bias0": bias(C),
        "timestep_weight2": xavier(rng, C, C), "timestep_bias2": bias(C),
        "modulation_weight": xavier(rng, 6 * C, C), "modulation_bias": bias(6 * C),
        "output_weight": xavier(rng, hp.out_channels, C), "output_bias": bias(hp.out_channels),
        "blocks": [],
    }
    proj = hp.image_attn_mode == "proj"
    for _ in range(hp.num_blocks):
        w["blocks"].append({
            "modulation": (rng.standard_normal(6 * C) * 0.1).astype(np.float32),
            "self_to_qkv_weight": xavier(rng, 3 * C, C), "self_to_qkv_bias": bias(3 * C),
            "self_q_gamma": gamma(C), "self_k_gamma": gamma(C),
            "self_to_out_weight": xavier(rng, C, C), "self_to_out_bias": bias(C),
            "norm2_weight": gamma(C), "norm2_bias": bias(C),
            "cross_to_q_weight": xavier(rng, C, C), "cross_to_q_bias": bias(C),
            "cross_to_kv_weight": xavier(rng, 2 * C, hp.cond_channels), "cross_to_kv_bias": bias(2 * C),
            "cross_q_gamma": gamma(C), "cross_k_gamma": gamma(C),
            "cross_to_out_weight": xavier(rng, C, C), "cross_to_out_bias": bias(C),
            "proj_weight": xavier(rng, C, hp.proj_in_channels) if proj else None,
            "proj_bias": bias(C) if proj else None,
            "mlp0_weight": xavier(rng, mlp, C), "mlp0_bias": bias(mlp),
            "mlp2_weight": xavier(rng, C, mlp), "mlp2_bias": bias(C),
        })
    if hp.io_resblocks:
        std = 1.0 / math.sqrt(27 * C)

        def res():
            return {"gn1_w": gamma(C), "gn1_b": bias(C),
                    "conv1_w": (rng.standard_normal((27, C, C)) * std).astype(np.float32), "conv1_b": bias(C),
                    "gn2_w": gamma(C), "gn2_b": bias(C),
                    "conv2_w": (rng.standard_normal((27, C, C)) * std).astype(np.float32), "conv2_b": bias(C)}

        w["io_in"] = [res() for _ in range(hp.io_resblocks)]
        w["io_out"] = [res() for _ in range(hp.io_resblocks)]
    return w
