"""Writer of small Pixal3D-style GGUF v3 packs for the loader tests (test
infrastructure).  Layout from the published GGUF specification: header
(magic, version 3, tensor count, metadata count), metadata key/value pairs,
tensor infos (name, dims innermost first, ggml type, offset), then the data
section aligned to general.alignment.  The metadata keys and tensor names
follow what the reference's loader reads (src/pack.cpp:127-260,
src/slat_flow.cpp:397-427 and :1347-1393): architecture "pixal3d",
tensor-name scheme "compact-v1", component hyperparameters under
"pixal3d.<component>.", tensors "<alias>.<module path>".
"""
from __future__ import annotations

import struct

import numpy as np

GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
_U32, _F32, _BOOL, _STRING = 4, 6, 7, 8
ALIGN = 32

ALIAS = {"shape_flow_512": "sh512", "shape_flow_1024": "sh1024", "texture_flow_1024": "tx1024"}


def _s(text: str) -> bytes:
    b = text.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, bool):
        return _s(key) + struct.pack("<IB", _BOOL, int(value))
    if isinstance(value, int):
        return _s(key) + struct.pack("<II", _U32, value)
    if isinstance(value, float):
        return _s(key) + struct.pack("<If", _F32, value)
    return _s(key) + struct.pack("<I", _STRING) + _s(value)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def stored(a: np.ndarray, ggml_type: int) -> np.ndarray:
    """The f32 values a tensor holds after storage in the given type."""
    a = np.asarray(a, np.float32)
    if ggml_type == GGML_F16:
        return a.astype(np.float16).astype(np.float32)
    if ggml_type == GGML_BF16:
        return (bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
    return a


def write_pack(path, metadata: dict, tensors: list) -> None:
    """tensors: (name, array in PyTorch layout, ggml type)."""
    infos, blobs, off = [], [], 0
    for name, a, t in tensors:
        a = np.ascontiguousarray(a, np.float32)
        if t == GGML_F32:
            raw = a.tobytes()
        elif t == GGML_F16:
            raw = a.astype(np.float16).tobytes()
        else:
            raw = bf16_bits(a).tobytes()
        dims = list(reversed(a.shape)) or [1]
        infos.append(_s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<IQ", t, off))
        pad = (-len(raw)) % ALIGN
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    meta = dict(metadata)
    meta.setdefault("general.alignment", ALIGN)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    body = head + b"".join(_kv(k, v) for k, v in meta.items()) + b"".join(infos)
    body += b"\0" * ((-len(body)) % ALIGN)
    with open(path, "wb") as f:
        f.write(body + b"".join(blobs))


BF16_KEYS = ("mlp0_weight", "mlp2_weight")


def flow_tensors(alias: str, w: dict, matrix_type: int = GGML_F16) -> list:
    """An oracle-keyed SLat-flow weight dict as (name, array, type) under the
    reference's module paths; MLP matrices in BF16, the other matrices in
    matrix_type, vectors in F32 (every type the loader converts)."""
    top = {"input_weight": "input_layer.weight", "input_bias": "input_layer.bias",
           "timestep_weight0": "t_embedder.mlp.0.weight", "timestep_bias0": "t_embedder.mlp.0.bias",
           "timestep_weight2": "t_embedder.mlp.2.weight", "timestep_bias2": "t_embedder.mlp.2.bias",
           "modulation_weight": "adaLN_modulation.1.weight", "modulation_bias": "adaLN_modulation.1.bias",
           "output_weight": "out_layer.weight", "output_bias": "out_layer.bias"}
    blk = {"modulation": "modulation", "self_to_qkv_weight": "self_attn.to_qkv.weight",
           "self_to_qkv_bias": "self_attn.to_qkv.bias", "self_q_gamma": "self_attn.q_rms_norm.gamma",
           "self_k_gamma": "self_attn.k_rms_norm.gamma", "self_to_out_weight": "self_attn.to_out.weight",
           "self_to_out_bias": "self_attn.to_out.bias", "norm2_weight": "norm2.weight", "norm2_bias": "norm2.bias",
           "cross_to_q_weight": "cross_attn.cross_attn_block.to_q.weight",
           "cross_to_q_bias": "cross_attn.cross_attn_block.to_q.bias",
           "cross_to_kv_weight": "cross_attn.cross_attn_block.to_kv.weight",
           "cross_to_kv_bias": "cross_attn.cross_attn_block.to_kv.bias",
           "cross_q_gamma": "cross_attn.cross_attn_block.q_rms_norm.gamma",
           "cross_k_gamma": "cross_attn.cross_attn_block.k_rms_norm.gamma",
           "cross_to_out_weight": "cross_attn.cross_attn_block.to_out.weight",
           "cross_to_out_bias": "cross_attn.cross_attn_block.to_out.bias",
           "proj_weight": "cross_attn.proj_linear.weight", "proj_bias": "cross_attn.proj_linear.bias",
           "mlp0_weight": "mlp.mlp.0.weight", "mlp0_bias": "mlp.mlp.0.bias",
           "mlp2_weight": "mlp.mlp.2.weight", "mlp2_bias": "mlp.mlp.2.bias"}
    out = []
    for k, name in top.items():
        a = np.asarray(w[k], np.float32)
        out.append((f"{alias}.{name}", a, matrix_type if a.ndim == 2 else GGML_F32))
    for i, b in enumerate(w["blocks"]):
        for k, name in blk.items():
            if b.get(k) is None:
                continue
            a = np.asarray(b[k], np.float32)
            t = (GGML_BF16 if k in BF16_KEYS else matrix_type) if a.ndim == 2 else GGML_F32
            out.append((f"{alias}.blocks.{i}.{name}", a, t))
    return out


def stored_flow_weights(w: dict, matrix_type: int = GGML_F16) -> dict:
    """The values flow_tensors' pack holds for w (after 16-bit storage)."""
    st = {k: (stored(v, matrix_type) if np.ndim(v) == 2 else v) for k, v in w.items() if k != "blocks"}
    st["blocks"] = [{k: (stored(v, GGML_BF16 if k in BF16_KEYS else matrix_type) if np.ndim(v) == 2 else v)
                     for k, v in b.items()} for b in w["blocks"]]
    return st


def flow_metadata(component: str, hp, resolution: int = 16) -> dict:
    k = f"pixal3d.{component}."
    return {"general.architecture": "pixal3d", "general.name": "test pack", "pixal3d.tensor_name_scheme": "compact-v1",
            "general.file_type": 1, "pixal3d.bundle_format": 1, "pixal3d.component.0": component,
            k + "model_class": "SLatFlowModel", k + "variant": "test", k + "resolution": resolution,
            k + "in_channels": hp.in_channels, k + "out_channels": hp.out_channels,
            k + "model_channels": hp.model_channels, k + "cond_channels": hp.cond_channels,
            k + "num_blocks": hp.num_blocks, k + "num_heads": hp.num_heads, k + "mlp_ratio": float(hp.mlp_ratio),
            k + "pe_mode": "rope", k + "share_mod": True, k + "qk_rms_norm": bool(hp.qk_rms_norm),
            k + "qk_rms_norm_cross": bool(hp.qk_rms_norm_cross), k + "rope_freq_min": float(hp.rope_freq_min),
            k + "rope_freq_base": float(hp.rope_freq_base), k + "image_attn_mode": hp.image_attn_mode,
            k + "proj_in_channels": int(hp.proj_in_channels)}
