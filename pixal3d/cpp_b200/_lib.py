"""ctypes binding of the C ABI in include/p3d.h (libp3dcuda.so).

The library is the product; there is no fallback.  Importing this module on
a machine without the built library raises immediately, and every call
checks its p3d_status and raises P3DError with the library's message.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libp3dcuda.so"

P3D_OK = 0
P3D_ERR_INVALID = 1
P3D_ERR_CUDA = 2
P3D_ERR_HASH_FULL = 3
P3D_ERR_TIMEOUT = 4
P3D_ERR_UNSUPPORTED = 5
P3D_ERR_NO_DEVICE = 6
P3D_ERR_DUPLICATE = 7
P3D_ERR_NONFINITE = 8

P3D_F32 = 0
P3D_BF16 = 1
P3D_F16 = 2

EPI_NONE = 0
EPI_GELU_TANH = 1
EPI_SILU = 2
EPI_RESIDUAL = 4

CONV_ORDER_CHUNK_ROWS = 4096  # P3D_CONV_ORDER_CHUNK_ROWS


class P3DError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"p3d status {status}: {message}")
        self.status = status


if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is not built; run `python -m pixal3d.cpp_b200.build` (no CPU fallback exists)")

lib = C.CDLL(str(LIB_PATH))

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
f32 = C.c_float
sz = C.c_size_t


class FlowHParams(C.Structure):
    """p3d_flow_hparams (include/p3d.h)."""
    _fields_ = [(n, i32) for n in (
        "in_channels", "out_channels", "model_channels", "cond_channels", "num_blocks", "num_heads",
        "mlp_hidden", "proj_in_channels", "proj_mode", "qk_rms_norm", "qk_rms_norm_cross", "pe_mode",
        "io_resblocks", "groups", "operand_dtype")] + [("norm_eps", f32), ("rope_freq_min", f32),
                                                        ("rope_freq_base", f32)]


BLOCK_WEIGHT_FIELDS = ["modulation", "qkv_w", "qkv_b", "q_gamma", "k_gamma", "out_w", "out_b", "norm2_w", "norm2_b",
                       "cq_w", "cq_b", "ckv_w", "ckv_b", "cq_gamma", "ck_gamma", "co_w", "co_b", "proj_w", "proj_b",
                       "mlp0_w", "mlp0_b", "mlp2_w", "mlp2_b"]
RESBLOCK_WEIGHT_FIELDS = ["gn1_w", "gn1_b", "conv1_w", "conv1_b", "gn2_w", "gn2_b", "conv2_w", "conv2_b"]
FLOW_TOP_FIELDS = ["input_w", "input_b", "t_w0", "t_b0", "t_w2", "t_b2", "mod_w", "mod_b", "output_w", "output_b"]


class BlockWeights(C.Structure):
    _fields_ = [(n, vp) for n in BLOCK_WEIGHT_FIELDS]


class ResBlockWeights(C.Structure):
    _fields_ = [(n, vp) for n in RESBLOCK_WEIGHT_FIELDS]


class FlowWeights(C.Structure):
    _fields_ = [(n, vp) for n in FLOW_TOP_FIELDS] + [
        ("blocks", C.POINTER(BlockWeights)), ("io_in", C.POINTER(ResBlockWeights)),
        ("io_out", C.POINTER(ResBlockWeights))]


class ProjectionView(C.Structure):
    """p3d_projection_view (include/p3d.h)."""
    _fields_ = [("feature_map", vp), ("height", i32), ("width", i32), ("channels", i32), ("image_resolution", i32),
                ("camera_angle_x", f32), ("distance", f32), ("mesh_scale", f32), ("has_transform", i32),
                ("transform_matrix", f32 * 16)]


class SamplerConfig(C.Structure):
    _fields_ = [("steps", i32), ("sigma_min", f32), ("rescale_t", f32), ("guidance_strength", f32),
                ("guidance_rescale", f32), ("guidance_interval_min", f32), ("guidance_interval_max", f32),
                ("use_graph", i32)]


def _sig(name, res, *args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_sig("p3d_version", i32)
_sig("p3d_ctx_create", i32, i32, vp, C.POINTER(vp))
_sig("p3d_ctx_destroy", i32, vp)
_sig("p3d_ctx_set_stream", i32, vp, vp)
_sig("p3d_ctx_stream", vp, vp)
_sig("p3d_last_error", C.c_char_p, vp)
_sig("p3d_ctx_check", i32, vp)
_sig("p3d_ctx_launch_count", i64, vp)
_sig("p3d_coord_hash_capacity", i64, i64)
_sig("p3d_coord_hash_build", i32, vp, vp, i64, vp, vp, i64)
_sig("p3d_neighbor_map27", i32, vp, vp, i64, vp, vp, i64, vp)
_sig("p3d_neighbor_map27_workspace", sz, i64)
_sig("p3d_neighbor_map27_ws", i32, vp, vp, i64, vp, sz, vp)
_sig("p3d_neighbor_map27_static", i32, vp, vp, i64, vp)
_sig("p3d_sparse_validate_workspace", sz, i64)
_sig("p3d_sparse_validate", i32, vp, vp, i64, vp, i32, i32, i32, i32, i32, vp, sz, vp)
_sig("p3d_device_alloc", i32, vp, sz, vp)
_sig("p3d_device_free", i32, vp, vp)
_sig("p3d_copy_to_device", i32, vp, vp, vp, sz)
_sig("p3d_copy_to_host", i32, vp, vp, vp, sz)
_sig("p3d_ctx_synchronize", i32, vp)
_sig("p3d_wait_selftest", i32, vp, i32, i64, vp)
_sig("p3d_conv_row_order_workspace", sz, i64, i32, i64)
_sig("p3d_conv_row_order", i32, vp, vp, vp, i64, i32, i64, vp, sz, vp)
_sig("p3d_downsample_grid_ints", i64, i32, i32, i32, i32, i32)
_sig("p3d_downsample_topology", i32, vp, vp, i64, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp)
_sig("p3d_downsample_mean", i32, vp, vp, i64, i32, i32, vp, i32, vp)
_sig("p3d_upsample_nearest", i32, vp, vp, i64, i32, vp, i32, vp)
_sig("p3d_c2s_topology", i32, vp, vp, i64, i32, vp, vp, vp, vp, vp, vp)
_sig("p3d_c2s_gather", i32, vp, vp, i64, vp, vp, i64, i32, i32, i32, vp)
_sig("p3d_linear", i32, vp, vp, i64, vp, i32, vp, i64, i64, i64, vp, i64, i32, i32, vp, i64, vp, i32)
_sig("p3d_subm_conv3d", i32, vp, vp, i64, i64, vp, vp, i32, vp, i64, vp, i64, i32, i32, vp, i64, vp, i32)
_sig("p3d_subm_conv3d_taps", i32, vp, vp, i64, i64, vp, vp, i32, vp, i64, vp, i64, i32, i32, vp, i64, vp, i32, vp)
_sig("p3d_conv_tile_taps", i32, vp, vp, i64, vp)
_sig("p3d_varlen_attention", i32, vp, vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, i32, i64, i64, i64, i32, i32, f32,
     i32)
_sig("p3d_ape_add", i32, vp, vp, i64, i32, vp)
_sig("p3d_project_features", i32, vp, C.POINTER(ProjectionView), i32, i32, vp, i64, vp, i64, i32, vp)
_sig("p3d_projection_relative_matrices", i32, vp, vp, vp, i32, vp)
_sig("p3d_slat_normalize", i32, vp, vp, i64, i32, vp, vp, i32, vp)
_sig("p3d_quantize_slat_coords_workspace", sz, i32)
_sig("p3d_quantize_slat_coords", i32, vp, vp, i64, i32, i32, i32, vp, vp, vp, sz)
_sig("p3d_batch_offsets", i32, vp, vp, i64, i32, vp)
_sig("p3d_window_count", i64, i32, i32, i32, i32, i32, i32)
_sig("p3d_window_partition_workspace", C.c_size_t, i64, i64)
_sig("p3d_window_partition", i32, vp, vp, i64, i32, i32, i32, i32, i32, i32, vp, vp, vp, C.c_size_t)
_sig("p3d_window_attention_scratch", C.c_size_t, i64, i32)
_sig("p3d_window_attention", i32, vp, vp, i64, vp, i64, vp, i64, vp, vp, i64, i32, i64, i32, i32, f32, i32, vp,
     C.c_size_t, vp, i64)
_sig("p3d_layernorm_modulate", i32, vp, vp, i64, i32, f32, vp, vp, vp, i64, vp, i32, vp, i32)
_sig("p3d_qk_rmsnorm_rope", i32, vp, vp, i64, i64, i32, i32, vp, vp, f32, f32, i32)
_sig("p3d_linear_headnorm", i32, vp, vp, i64, vp, i32, vp, i64, i64, i64, vp, i64, i32, i64, vp, i64, vp)
_sig("p3d_rope_table", i32, vp, vp, i64, i32, f32, f32, vp)
_sig("p3d_activation", i32, vp, vp, i64, i32, i32, vp)
_sig("p3d_repack_heads", i32, vp, vp, i64, i64, i32, i32, i32, vp, i64, i32)
_sig("p3d_timestep_mlp", i32, vp, vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp)
_sig("p3d_layernorm_act", i32, vp, vp, i64, i32, f32, vp, vp, i32, vp, i64, i32)
_sig("p3d_pack_operand", i32, vp, vp, i64, i32, vp, i64, i32)
_sig("p3d_group_norm_silu", i32, vp, vp, i64, i32, i32, f32, vp, vp, vp, i32, i32, vp, vp, i32)
_sig("p3d_euler_cfg_step", i32, vp, vp, vp, vp, i64, i32, vp, i32, f32, f32, f32, f32, f32, vp, vp)
_sig("p3d_convert", i32, vp, vp, i32, i64, vp, i32)

OPTIONAL = {}


def _optional(name, res, *args):
    try:
        OPTIONAL[name] = _sig(name, res, *args)
    except AttributeError:
        pass


_optional("p3d_flow_create", i32, vp, C.POINTER(FlowHParams), C.POINTER(FlowWeights), C.POINTER(vp))
_optional("p3d_flow_destroy", i32, vp)
_optional("p3d_flow_prepare", i32, vp, vp, i64, i32, i32, i32, i32, C.POINTER(i64))
_optional("p3d_flow_forward", i32, vp, vp, vp, vp, i32, vp, vp)
_optional("p3d_flow_sample", i32, vp, vp, vp, i32, vp, C.POINTER(SamplerConfig))
_optional("p3d_flow_sample_concat", i32, vp, vp, vp, i32, vp, vp, i32, C.POINTER(SamplerConfig))
_optional("p3d_flow_last_error", C.c_char_p, vp)
_optional("p3d_flow_launches_per_step", i64, vp)

DECODER_MAX_LEVELS = 8


class DecoderConfig(C.Structure):
    _fields_ = [("latent_channels", i32), ("out_channels", i32), ("levels", i32),
                ("model_channels", i32 * DECODER_MAX_LEVELS), ("num_blocks", i32 * DECODER_MAX_LEVELS),
                ("pred_subdiv", i32), ("norm_eps", f32), ("operand_dtype", i32)]


DECODER_BLOCK_FIELDS = ("norm_w", "norm_b", "norm1_w", "norm1_b", "conv1_w", "conv1_b", "conv2_w", "conv2_b",
                        "mlp0_w", "mlp0_b", "mlp2_w", "mlp2_b", "subdiv_w", "subdiv_b")


class DecoderBlock(C.Structure):
    _fields_ = [("kind", i32), ("channels", i32), ("out_channels", i32), ("mlp_hidden", i32)] + \
        [(n, vp) for n in DECODER_BLOCK_FIELDS]


class DecoderWeights(C.Structure):
    _fields_ = [("from_latent_w", vp), ("from_latent_b", vp), ("output_w", vp), ("output_b", vp),
                ("blocks", C.POINTER(DecoderBlock)), ("num_blocks", i32)]


_sig("p3d_decoder_create", i32, vp, C.POINTER(DecoderConfig), C.POINTER(DecoderWeights), C.POINTER(vp))
_sig("p3d_decoder_destroy", i32, vp)
_sig("p3d_decoder_run", i32, vp, vp, i64, i32, i32, i32, i32, vp, C.POINTER(vp), C.POINTER(i64), i32)
_sig("p3d_decoder_rows", i64, vp, i32)
_sig("p3d_decoder_coords", i32, vp, i32, vp)
_sig("p3d_decoder_output", i32, vp, vp)
_sig("p3d_decoder_subdivision", i32, vp, i32, vp)


def exported_symbols() -> list[str]:
    """Names the header declares; used by the CPU test that checks exports."""
    import re
    hdr = (Path(__file__).resolve().parent.parent.parent / "include" / "p3d.h").read_text()
    return sorted(set(re.findall(r"\b(p3d_[a-z0-9_]+)\s*\(", hdr)))
