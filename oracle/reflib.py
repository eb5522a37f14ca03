"""ctypes access to the compiled reference CPU path (oracle/_ref/libp3dref.so).

TEST INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke, bench.py's CPU
baseline).  The library is built by oracle/Makefile from the reference's own
sources plus oracle/ref_shim.cpp; every wrapper below names the reference
function it reaches.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_ref" / "libp3dref.so"
_lib = None

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} missing: run `make -C oracle` where the reference is mounted")
        _lib = C.CDLL(str(LIB_PATH))
    return _lib


class RefError(RuntimeError):
    pass


def _err():
    return C.create_string_buffer(512)


def _check(rc, err):
    if rc != 0:
        raise RefError(err.value.decode())


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int) -> None:
    """set_cpu_thread_override (include/pixal3d/cpu_threads.h:31)."""
    lib().p3dref_set_threads(int(n))


def _shape(coords, batch, shape):
    if batch is None:
        batch = int(coords[:, 0].max()) + 1 if coords.shape[0] else 1
    if shape is None:
        shape = tuple(int(v) + 1 for v in coords[:, 1:].max(axis=0)) if coords.shape[0] else (1, 1, 1)
    return batch, shape


def valid(coords, x, batch, shape) -> str | None:
    """SparseTensorF32::valid: None or the reference's error message."""
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    err = _err()
    rc = lib().p3dref_valid(coords.ctypes, C.c_int64(coords.shape[0]), x.ctypes, x.shape[1], batch, *shape, err,
                            len(err))
    return None if rc == 0 else err.value.decode()


def sparse_linear(coords, x, w, b, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    cout = w.shape[0]
    out = np.empty((x.shape[0], cout), np.float32)
    err = _err()
    _check(lib().p3dref_sparse_linear(coords.ctypes, C.c_int64(x.shape[0]), x.ctypes, x.shape[1], batch,
                                      *shape, _c(w, np.float32).ctypes, _c(b, np.float32).ctypes, cout,
                                      out.ctypes, err, 512), err)
    return out


def layer_norm(coords, x, eps, gamma=None, beta=None, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    out = np.empty_like(x)
    err = _err()
    g = _c(gamma, np.float32).ctypes if gamma is not None else None
    bb = _c(beta, np.float32).ctypes if beta is not None else None
    _check(lib().p3dref_layer_norm(coords.ctypes, C.c_int64(x.shape[0]), x.ctypes, x.shape[1], batch, *shape,
                                   C.c_float(eps), g, bb, out.ctypes, err, 512), err)
    return out


def subm_conv3d(coords, x, w, b, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    cout = w.shape[1]
    out = np.empty((x.shape[0], cout), np.float32)
    err = _err()
    _check(lib().p3dref_subm_conv3d(coords.ctypes, C.c_int64(x.shape[0]), x.ctypes, x.shape[1], batch, *shape,
                                    _c(w, np.float32).ctypes, _c(b, np.float32).ctypes, cout, out.ctypes,
                                    err, 512), err)
    return out


def neighbor_map27(coords, batch=None, shape=None):
    coords = _c(coords, np.int32)
    batch, shape = _shape(coords, batch, shape)
    n = coords.shape[0]
    out = np.empty((27, n), np.int32)
    err = _err()
    _check(lib().p3dref_neighbor_map27(coords.ctypes, C.c_int64(n), batch, *shape, out.ctypes, err, 512), err)
    return out


def coords_fingerprint(coords) -> int:
    coords = _c(coords, np.int32)
    f = lib().p3dref_coords_fingerprint
    f.restype = C.c_uint64
    return int(f(coords.ctypes, C.c_int64(coords.shape[0])))


def downsample_mean(coords, x, factor, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    n = x.shape[0]
    oc = np.empty((n, 4), np.int32)
    of = np.empty((n, x.shape[1]), np.float32)
    on = C.c_int64(0)
    osh = (C.c_int * 3)()
    err = _err()
    _check(lib().p3dref_downsample_mean(coords.ctypes, C.c_int64(n), x.ctypes, x.shape[1], batch, *shape, factor,
                                        oc.ctypes, of.ctypes, C.byref(on), osh, err, 512), err)
    m = on.value
    return oc[:m].copy(), of[:m].copy(), tuple(osh)


def channel_to_spatial(coords, x, factor, subdiv=None, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    n = x.shape[0]
    nc = factor ** 3
    oc = np.empty((n * nc, 4), np.int32)
    of = np.empty((n * nc, x.shape[1] // nc), np.float32)
    on = C.c_int64(0)
    err = _err()
    sd = _c(subdiv, np.float32).ctypes if subdiv is not None else None
    _check(lib().p3dref_channel_to_spatial(coords.ctypes, C.c_int64(n), x.ctypes, x.shape[1], batch, *shape,
                                           factor, sd, oc.ctypes, of.ctypes, C.byref(on), err, 512), err)
    m = on.value
    return oc[:m].copy(), of[:m].copy()


def sdpa(coords, q, k, v, heads, head_dim, scale, batch=None, shape=None):
    coords = _c(coords, np.int32)
    batch, shape = _shape(coords, batch, shape)
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty((q.shape[0], v.shape[1]), np.float32)
    err = _err()
    _check(lib().p3dref_sdpa(coords.ctypes, C.c_int64(q.shape[0]), batch, *shape, q.ctypes, k.ctypes, v.ctypes,
                             heads, head_dim, v.shape[1], C.c_float(scale), out.ctypes, err, 512), err)
    return out


def cross_attention(coords, q, offsets, k, v, heads, head_dim, scale, batch=None, shape=None):
    coords = _c(coords, np.int32)
    batch, shape = _shape(coords, batch, shape)
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    offsets = _c(offsets, np.int64)
    out = np.empty((q.shape[0], v.shape[1]), np.float32)
    err = _err()
    _check(lib().p3dref_cross_attention(coords.ctypes, C.c_int64(q.shape[0]), batch, *shape, q.ctypes,
                                        offsets.ctypes, k.ctypes, v.ctypes, heads, head_dim, v.shape[1],
                                        C.c_float(scale), out.ctypes, err, 512), err)
    return out


def rope(coords, x, heads, head_dim, fmin=1.0, fbase=10000.0, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    out = np.empty_like(x)
    err = _err()
    _check(lib().p3dref_rope(coords.ctypes, C.c_int64(x.shape[0]), batch, *shape, x.ctypes, heads, head_dim,
                             C.c_float(fmin), C.c_float(fbase), out.ctypes, err, 512), err)
    return out


def rms_norm(coords, x, heads, head_dim, gamma, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    out = np.empty_like(x)
    err = _err()
    _check(lib().p3dref_rms_norm(coords.ctypes, C.c_int64(x.shape[0]), batch, *shape, x.ctypes, heads, head_dim,
                                 _c(gamma, np.float32).ctypes, out.ctypes, err, 512), err)
    return out


def timestep_embed_mlp(t, hidden, w0, b0, w2, b2, freq=256):
    t = _c(t, np.float32)
    out = np.empty((t.shape[0], hidden), np.float32)
    err = _err()
    _check(lib().p3dref_timestep_embed_mlp(t.ctypes, C.c_int64(t.shape[0]), hidden, freq,
                                           _c(w0, np.float32).ctypes, _c(b0, np.float32).ctypes,
                                           _c(w2, np.float32).ctypes, _c(b2, np.float32).ctypes,
                                           out.ctypes, err, 512), err)
    return out


def _ptr_array(arrays):
    keep = [None if a is None else _c(a, np.float32) for a in arrays]
    arr = (C.c_void_p * len(keep))(*[None if a is None else a.ctypes.data for a in keep])
    return arr, keep


def transformer_block(coords, x, tmod, ctx_offsets, ctx, proj, cfg, w, batch=None, shape=None):
    """sparse_transformer_cross_block_f32; cfg is oracle.BlockConfig, w the
    dict keyed by oracle.BLOCK_FIELDS."""
    from oracle.oracle import BLOCK_FIELDS
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    cfg_i = (C.c_int * 9)(cfg.channels, cfg.num_heads, cfg.mlp_hidden, cfg.context_channels,
                          cfg.proj_in_channels, int(cfg.use_rope), int(cfg.qk_rms_norm),
                          int(cfg.qk_rms_norm_cross), int(cfg.use_projection))
    cfg_f = (C.c_float * 3)(cfg.norm_eps, cfg.rope_freq_min, cfg.rope_freq_base)
    wp, keep = _ptr_array([w.get(f) for f in BLOCK_FIELDS])
    out = np.empty_like(x)
    err = _err()
    tmod = _c(tmod, np.float32)
    ctx = _c(ctx, np.float32)
    offs = _c(ctx_offsets, np.int64)
    pj = _c(proj, np.float32).ctypes if proj is not None else None
    _check(lib().p3dref_transformer_block(coords.ctypes, C.c_int64(x.shape[0]), batch, *shape, x.ctypes,
                                          tmod.ctypes, offs.ctypes, ctx.ctypes, pj, cfg_i, cfg_f, wp,
                                          out.ctypes, err, 512), err)
    return out


def _flow_args(hp, w):
    from oracle.oracle import BLOCK_FIELDS, FLOW_TOP_FIELDS
    hp_i = (C.c_int * 11)(64, hp.in_channels, hp.out_channels, hp.model_channels, hp.cond_channels,
                          hp.num_blocks, hp.num_heads, hp.proj_in_channels,
                          int(hp.image_attn_mode == "proj"), int(hp.qk_rms_norm), int(hp.qk_rms_norm_cross))
    hp_f = (C.c_float * 4)(hp.mlp_ratio, hp.norm_eps, hp.rope_freq_min, hp.rope_freq_base)
    top, k1 = _ptr_array([w[f] for f in FLOW_TOP_FIELDS])
    blocks, k2 = _ptr_array([bw.get(f) for bw in w["blocks"] for f in BLOCK_FIELDS])
    return hp_i, hp_f, top, blocks, (k1, k2)


def slat_flow_forward(coords, x, timesteps, ctx_offsets, ctx, proj, hp, w, batch=None, shape=None):
    """slat_flow_forward_f32 (reference model only: pe_mode rope, no io stages)."""
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    hp_i, hp_f, top, blocks, keep = _flow_args(hp, w)
    out = np.empty((x.shape[0], hp.out_channels), np.float32)
    err = _err()
    ts = _c(timesteps, np.float32)
    pj = _c(proj, np.float32).ctypes if proj is not None else None
    _check(lib().p3dref_slat_flow_forward(coords.ctypes, C.c_int64(x.shape[0]), batch, *shape, x.ctypes,
                                          ts.ctypes, _c(ctx_offsets, np.int64).ctypes, _c(ctx, np.float32).ctypes,
                                          pj, hp_i, hp_f, top, blocks, out.ctypes, err, 512), err)
    return out


def slat_flow_sample(coords, noise, ctx_offsets, ctx, proj, hp, w, sc, record_x0=False, batch=None, shape=None):
    """flow_euler_sample_f32 driven by slat_flow_forward_f32 with the zeros
    negative condition of SLatFlowModel::sample."""
    coords, noise = _c(coords, np.int32), _c(noise, np.float32)
    batch, shape = _shape(coords, batch, shape)
    hp_i, hp_f, top, blocks, keep = _flow_args(hp, w)
    sc_f = (C.c_float * 6)(sc.sigma_min, sc.rescale_t, sc.guidance_strength, sc.guidance_rescale,
                           sc.guidance_interval_min, sc.guidance_interval_max)
    out = np.empty_like(noise)
    x0 = np.empty_like(noise) if record_x0 else None
    err = _err()
    pj = _c(proj, np.float32).ctypes if proj is not None else None
    _check(lib().p3dref_slat_flow_sample(coords.ctypes, C.c_int64(noise.shape[0]), batch, *shape, noise.ctypes,
                                         _c(ctx_offsets, np.int64).ctypes, _c(ctx, np.float32).ctypes, pj,
                                         hp_i, hp_f, top, blocks, sc.steps, sc_f, out.ctypes,
                                         x0.ctypes if x0 is not None else None, err, 512), err)
    return (out, x0) if record_x0 else out


VELOCITY_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_float), C.c_int64, C.c_int, C.c_float, C.c_int,
                          C.POINTER(C.c_float))


def flow_euler_sample(coords, noise, sc, model, batch=None, shape=None):
    """flow_euler_sample_f32 with a Python velocity model(state, t, cond)."""
    coords, noise = _c(coords, np.int32), _c(noise, np.float32)
    batch, shape = _shape(coords, batch, shape)
    n, ch = noise.shape

    def cb(user, state, n_, ch_, t, cond, vel):
        s = np.ctypeslib.as_array(state, shape=(n_, ch_)).copy()
        v = model(s, np.float32(t), bool(cond)).astype(np.float32)
        np.ctypeslib.as_array(vel, shape=(n_, ch_))[:] = v
        return 0

    fn = VELOCITY_FN(cb)
    sc_f = (C.c_float * 6)(sc.sigma_min, sc.rescale_t, sc.guidance_strength, sc.guidance_rescale,
                           sc.guidance_interval_min, sc.guidance_interval_max)
    out = np.empty_like(noise)
    err = _err()
    _check(lib().p3dref_flow_euler_sample(coords.ctypes, C.c_int64(n), batch, *shape, noise.ctypes, ch, sc.steps,
                                          sc_f, fn, None, out.ctypes, err, 512), err)
    return out


def convnext_block(coords, x, w, mlp_hidden, eps, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    wp, keep = _ptr_array([w[k] for k in ("norm_w", "norm_b", "conv_w", "conv_b",
                                           "mlp0_w", "mlp0_b", "mlp2_w", "mlp2_b")])
    out = np.empty_like(x)
    err = _err()
    _check(lib().p3dref_convnext_block(coords.ctypes, C.c_int64(x.shape[0]), batch, *shape, x.ctypes,
                                       x.shape[1], mlp_hidden, wp, C.c_float(eps), out.ctypes, err, 512), err)
    return out


def resblock_c2s(coords, x, w, eps, out_channels, pred_subdiv, subdiv=None, batch=None, shape=None):
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    n = x.shape[0]
    wp, keep = _ptr_array([w.get(k) for k in ("norm1_w", "norm1_b", "conv1_w", "conv1_b",
                                               "conv2_w", "conv2_b", "subdiv_w", "subdiv_b")])
    oc = np.empty((8 * n, 4), np.int32)
    of = np.empty((8 * n, out_channels), np.float32)
    on = C.c_int64(0)
    pred = np.empty((n, 8), np.float32) if pred_subdiv else None
    err = _err()
    sd = _c(subdiv, np.float32).ctypes if subdiv is not None else None
    _check(lib().p3dref_resblock_c2s(coords.ctypes, C.c_int64(n), batch, *shape, x.ctypes, x.shape[1],
                                     out_channels, wp, C.c_float(eps), int(pred_subdiv), sd, oc.ctypes,
                                     of.ctypes, C.byref(on), pred.ctypes if pred is not None else None,
                                     err, 512), err)
    m = on.value
    return oc[:m].copy(), of[:m].copy(), pred


def _m16(cam):
    return _c(cam.transform if cam.transform is not None else np.zeros(16, np.float32), np.float32).reshape(16)


def project_at_coords(fmap, grid_resolution, image_resolution, cam, coords):
    """project_grid_features_at_coords (src/projection.cpp:359-434); cam is an
    oracle.ProjCamera.  Returns (features [N, C], valid [N] uint8)."""
    fmap, coords = _c(fmap, np.float32), _c(coords, np.int32)
    h, w, c = fmap.shape
    n = coords.shape[0]
    m16 = _m16(cam)
    feats = np.empty((n, c), np.float32)
    valid = np.empty(n, np.uint8)
    err = _err()
    _check(lib().p3dref_project_at_coords(fmap.ctypes, h, w, c, grid_resolution, image_resolution,
                                          C.c_float(cam.camera_angle_x), C.c_float(cam.distance),
                                          C.c_float(cam.mesh_scale), int(cam.transform is not None), m16.ctypes,
                                          coords.ctypes, C.c_int64(n), feats.ctypes, valid.ctypes, err, 512), err)
    return feats, valid


def project_average(fmaps, grid_resolution, image_resolution, cams):
    """project_grid_features_average (src/projection.cpp:436-481) over views of
    one map shape: (features [r^3, C], valid [r^3] uint8)."""
    fmaps = [_c(f, np.float32) for f in fmaps]
    h, w, c = fmaps[0].shape
    ptrs = (C.c_void_p * len(fmaps))(*[f.ctypes.data for f in fmaps])
    camv = np.array([[k.camera_angle_x, k.distance, k.mesh_scale, float(k.transform is not None)] for k in cams],
                    np.float32)
    m16 = np.ascontiguousarray(np.stack([_m16(k) for k in cams]))
    pts = grid_resolution ** 3
    feats = np.empty((pts, c), np.float32)
    valid = np.empty(pts, np.uint8)
    err = _err()
    _check(lib().p3dref_project_average(ptrs, len(fmaps), h, w, c, grid_resolution, image_resolution, camv.ctypes,
                                        m16.ctypes, feats.ctypes, valid.ctypes, err, 512), err)
    return feats, valid


def relative_matrices(c2w, distances):
    """compute_relative_calc_matrices (src/projection.cpp:528-561): [n, 16]."""
    m = np.ascontiguousarray(np.asarray(c2w, np.float32).reshape(-1, 16))
    d = _c(distances, np.float32)
    out = np.empty_like(m)
    err = _err()
    _check(lib().p3dref_relative_matrices(m.ctypes, d.ctypes, m.shape[0], out.ctypes, err, 512), err)
    return out


def normalize_slat(coords, x, mean, std, batch=None, shape=None):
    """normalize_slat_f32 (src/pipeline.cpp:333-358)."""
    coords, x = _c(coords, np.int32), _c(x, np.float32)
    batch, shape = _shape(coords, batch, shape)
    out = np.empty_like(x)
    err = _err()
    _check(lib().p3dref_normalize_slat(coords.ctypes, C.c_int64(x.shape[0]), x.ctypes, x.shape[1], batch, *shape,
                                       _c(mean, np.float32).ctypes, _c(std, np.float32).ctypes, out.ctypes, err, 512),
           err)
    return out


def quantize_slat_coords(coords, low_resolution, requested_resolution=1024, max_tokens=0, batch=None, spatial=None):
    """quantize_slat_coords_f32 (src/pipeline.cpp:437-468): int32 [m, 4]."""
    coords = _c(coords, np.int32)
    n = coords.shape[0]
    batch = int(coords[:, 0].max()) + 1 if batch is None else batch
    spatial = low_resolution if spatial is None else spatial
    out = np.empty((max(n, 1), 4), np.int32)
    m = C.c_int64(0)
    err = _err()
    _check(lib().p3dref_quantize_slat_coords(coords.ctypes, C.c_int64(n), batch, spatial, low_resolution,
                                             requested_resolution, C.c_int64(max_tokens), out.ctypes, C.byref(m),
                                             err, 512), err)
    return out[:m.value].copy()
