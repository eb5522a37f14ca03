"""Torch-tensor front end of the C ABI (include/p3d.h).

PyTorch is plumbing here: it owns device memory and streams.  Every compute
call goes to libp3dcuda.so; each wrapper validates shapes/dtypes, passes raw
device pointers and the current torch stream, and raises P3DError on a
non-zero status.  Names follow the reference's operators
(src/sparse.cpp, src/sparse_transformer.cpp, src/flow_sampler.cpp).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from ._lib import P3DError

_CTX: dict[int, "Context"] = {}


class Context:
    """One p3d_ctx per device; its stream follows torch's current stream."""

    def __init__(self, device: int):
        h = C.c_void_p()
        rc = L.lib.p3d_ctx_create(device, None, C.byref(h))
        if rc != 0:
            raise P3DError(rc, f"p3d_ctx_create(device={device}) failed")
        self.h = h
        self.device = device

    def bind(self) -> "Context":
        s = torch.cuda.current_stream(self.device).cuda_stream
        L.lib.p3d_ctx_set_stream(self.h, C.c_void_p(s))
        return self

    def check(self, rc: int) -> None:
        if rc != 0:
            raise P3DError(rc, L.lib.p3d_last_error(self.h).decode())

    def sync_check(self) -> None:
        self.check(L.lib.p3d_ctx_check(self.h))

    @property
    def launches(self) -> int:
        return int(L.lib.p3d_ctx_launch_count(self.h))


def ctx(device: torch.device | int | None = None) -> Context:
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        idx = device.index if device.index is not None else torch.cuda.current_device()
    else:
        idx = int(device)
    if idx not in _CTX:
        _CTX[idx] = Context(idx)
    return _CTX[idx].bind()


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.P3D_F32
    if t.dtype == torch.bfloat16:
        return L.P3D_BF16
    if t.dtype == torch.float16:
        return L.P3D_F16
    raise TypeError(f"unsupported dtype {t.dtype}")


HALF = (torch.bfloat16, torch.float16)


def _rows(t: torch.Tensor) -> int:
    """Row pitch (elements) of a 2-D row-major view with unit column stride."""
    assert t.dim() == 2 and t.stride(1) == 1, "expected a 2-D row-major view"
    return t.stride(0)


# ---------------------------------------------------------------- topology

def neighbor_map27(coords: torch.Tensor) -> torch.Tensor:
    """[27, n] int32 neighbour map, sentinel n (build_neighbor_gather_map,
    src/slat_decoder.cpp:609-714)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    ws_bytes = int(L.lib.p3d_neighbor_map27_workspace(n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=coords.device)
    out = torch.empty((27, n), dtype=torch.int32, device=coords.device)
    c.check(L.lib.p3d_neighbor_map27_ws(c.h, _p(coords), n, _p(ws), ws_bytes, _p(out)))
    return out


def sparse_validate(coords: torch.Tensor, feats: torch.Tensor | None, batch: int, spatial) -> tuple[int, int] | None:
    """Device validity probe (SparseTensorF32::valid): None, or the first
    failing (row, check) with check 0 outside the shape, 1 duplicate, 2 batch
    order, 3 non-finite feature."""
    c = ctx(coords.device)
    n = coords.shape[0]
    ws_bytes = int(L.lib.p3d_sparse_validate_workspace(n))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=coords.device)
    first = torch.empty(1, dtype=torch.int64, device=coords.device)
    ch = feats.shape[1] if feats is not None else 1
    c.check(L.lib.p3d_sparse_validate(c.h, _p(coords), n, _p(feats), ch, batch, *spatial, _p(ws), ws_bytes,
                                      _p(first)))
    v = int(first.item())
    if v >= 0x7F7F7F7F7F7F7F7F:
        return None
    return v >> 2, v & 3


def downsample_topology(coords: torch.Tensor, batch: int, shape, factor: int = 2):
    """Parents of sparse_downsample_mean (src/sparse.cpp:536-602).
    Returns (out_coords [m,4], parent [n], child [m, f^3], m)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    gints = int(L.lib.p3d_downsample_grid_ints(batch, *shape, factor))
    grid = torch.empty(gints, dtype=torch.int32, device=coords.device)
    oc = torch.empty((max(n, 1), 4), dtype=torch.int32, device=coords.device)
    parent = torch.empty(max(n, 1), dtype=torch.int32, device=coords.device)
    child = torch.empty((max(n, 1), factor ** 3), dtype=torch.int32, device=coords.device)
    m = torch.zeros(1, dtype=torch.int64, device=coords.device)
    c.check(L.lib.p3d_downsample_topology(c.h, _p(coords), n, batch, *shape, factor, _p(grid), _p(oc), _p(parent),
                                          _p(child), _p(m)))
    mm = int(m.item())
    return oc[:mm], parent[:n], child[:mm], mm


def downsample_mean(x: torch.Tensor, child: torch.Tensor, factor: int = 2) -> torch.Tensor:
    c = ctx(x.device)
    m = child.shape[0]
    out = torch.empty((m, x.shape[1]), dtype=x.dtype, device=x.device)
    c.check(L.lib.p3d_downsample_mean(c.h, _p(x), m, x.shape[1], factor, _p(child), _dt(x), _p(out)))
    return out


def upsample_nearest(x: torch.Tensor, parent: torch.Tensor) -> torch.Tensor:
    c = ctx(x.device)
    n = parent.shape[0]
    out = torch.empty((n, x.shape[1]), dtype=x.dtype, device=x.device)
    c.check(L.lib.p3d_upsample_nearest(c.h, _p(x), n, x.shape[1], _p(parent), _dt(x), _p(out)))
    return out


def c2s_topology(coords: torch.Tensor, factor: int = 2, mask: torch.Tensor | None = None):
    """Subdivision topology (sparse_channel_to_spatial, src/sparse.cpp:604-702).
    Returns (out_coords [m,4], src_row [m], src_child [m], m)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    nc = factor ** 3
    scratch = torch.empty(n + 1, dtype=torch.int64, device=coords.device)
    oc = torch.empty((max(n * nc, 1), 4), dtype=torch.int32, device=coords.device)
    sr = torch.empty(max(n * nc, 1), dtype=torch.int32, device=coords.device)
    sc = torch.empty(max(n * nc, 1), dtype=torch.int8, device=coords.device)
    m = torch.zeros(1, dtype=torch.int64, device=coords.device)
    if mask is not None:
        assert mask.dtype == torch.float32 and mask.shape == (n, nc)
    c.check(L.lib.p3d_c2s_topology(c.h, _p(coords), n, factor, _p(mask), _p(scratch), _p(oc), _p(sr), _p(sc), _p(m)))
    mm = int(m.item())
    return oc[:mm], sr[:mm], sc[:mm], mm


def c2s_gather(x: torch.Tensor, src_row: torch.Tensor, src_child: torch.Tensor, cout: int,
               repeat: int = 1) -> torch.Tensor:
    c = ctx(x.device)
    m = src_row.shape[0]
    out = torch.empty((m, cout * repeat), dtype=x.dtype, device=x.device)
    c.check(L.lib.p3d_c2s_gather(c.h, _p(x), x.shape[1], _p(src_row), _p(src_child), m, cout, repeat, _dt(x),
                                 _p(out)))
    return out


# ------------------------------------------------------------ contractions

def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
           out_dtype: torch.dtype = torch.bfloat16, epilogue: int = L.EPI_NONE, gate: torch.Tensor | None = None,
           batch_offsets: torch.Tensor | None = None) -> torch.Tensor:
    """epilogue(x W^T + b) on tcgen05 (sparse_linear, src/sparse.cpp:337-451).
    x and w: the same 16-bit type (bf16 or f16)."""
    assert x.dtype in HALF and w.dtype == x.dtype
    c = ctx(x.device)
    m, k = x.shape
    n = w.shape[0]
    assert w.shape[1] == k and w.is_contiguous()
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    gate_ld = gate.stride(0) if gate is not None else 0
    nb = batch_offsets.shape[0] - 1 if batch_offsets is not None else 0
    c.check(L.lib.p3d_linear(c.h, _p(x), _rows(x), _p(w), _dt(x), _p(bias), m, n, k, _p(out), _rows(out), _dt(out), epilogue,
                             _p(gate), gate_ld, _p(batch_offsets), nb))
    return out


def linear_headnorm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, norm_cols: int,
                    gamma: torch.Tensor | None, rope_cols: int = 0, rope: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """x W^T + b with per-64-column-head RMS norm (columns < norm_cols, gamma
    per column) and interleaved RoPE (columns < rope_cols, rope from
    rope_table) applied to the f32 accumulators; 16-bit out of x's type."""
    assert x.dtype in HALF and w.dtype == x.dtype and w.is_contiguous()
    c = ctx(x.device)
    m, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    c.check(L.lib.p3d_linear_headnorm(c.h, _p(x), _rows(x), _p(w), _dt(x), _p(bias), m, n, k, _p(out), _rows(out),
                                      _dt(out), norm_cols, _p(gamma), rope_cols, _p(rope)))
    return out


def rope_table(coords: torch.Tensor, head_dim: int = 64, freq_min: float = 1.0,
               freq_base: float = 10000.0) -> torch.Tensor:
    """[head_dim/2, n, 2] f32 (cos, sin) per rotation pair and point
    (pair-major, the layout p3d_linear_headnorm reads)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    t = torch.empty((head_dim // 2, n, 2), dtype=torch.float32, device=coords.device)
    c.check(L.lib.p3d_rope_table(c.h, _p(coords), n, head_dim, freq_min, freq_base, _p(t)))
    return t


def subm_conv3d(x: torch.Tensor, nbr: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.float32,
                epilogue: int = L.EPI_NONE, gate: torch.Tensor | None = None,
                batch_offsets: torch.Tensor | None = None, tile_taps: torch.Tensor | None = None) -> torch.Tensor:
    """Gather-GEMM submanifold conv (sparse_submanifold_conv3d, src/sparse.cpp:999-1055).
    x [n, cin], w [27, cout, cin], both bf16 or both f16.  tile_taps
    (conv_tile_taps of nbr) lets the kernel skip taps no row of a 256-row
    tile uses; the result is the same."""
    assert x.dtype in HALF and w.dtype == x.dtype and x.is_contiguous() and w.is_contiguous()
    c = ctx(x.device)
    n, cin = x.shape
    cout = w.shape[1]
    if out is None:
        out = torch.empty((n, cout), dtype=out_dtype, device=x.device)
    gate_ld = gate.stride(0) if gate is not None else 0
    nb = batch_offsets.shape[0] - 1 if batch_offsets is not None else 0
    c.check(L.lib.p3d_subm_conv3d_taps(c.h, _p(x), n, cin, _p(nbr), _p(w), _dt(x), _p(bias), cout, _p(out), _rows(out),
                                       _dt(out), epilogue, _p(gate), gate_ld, _p(batch_offsets), nb, _p(tile_taps)))
    return out


def conv_row_order(coords: torch.Tensor, nbr: torch.Tensor, batch: int,
                   chunk_rows: int = L.CONV_ORDER_CHUNK_ROWS) -> torch.Tensor:
    """perm [n] int32: rows stably sorted by (batch, row // chunk_rows,
    neighbour pattern); the default chunk is the order in which the flow runs
    its fine-level convs (p3d_conv_row_order; chunk_rows <= 0: one chunk)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    ws_bytes = int(L.lib.p3d_conv_row_order_workspace(n, batch, chunk_rows))
    if ws_bytes == 0:
        raise ValueError("conv_row_order: chunk_rows too small for a 64-bit key")
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=coords.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    perm = torch.empty(n, dtype=torch.int32, device=coords.device)
    c.check(L.lib.p3d_conv_row_order(c.h, _p(coords), _p(nbr), n, batch, chunk_rows, C.c_void_p(base), ws_bytes,
                                     _p(perm)))
    return perm


def conv_tile_taps(nbr: torch.Tensor) -> torch.Tensor:
    """Per 256-row tile, the taps some row of the tile uses (p3d_conv_tile_taps)."""
    c = ctx(nbr.device)
    n = nbr.shape[1]
    taps = torch.empty(max((n + 255) // 256, 1), dtype=torch.int32, device=nbr.device)
    c.check(L.lib.p3d_conv_tile_taps(c.h, _p(nbr), n, _p(taps)))
    return taps


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_q: torch.Tensor, cu_k: torch.Tensor,
                     max_q: int, heads: int, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Flash attention over packed ragged sequences, head_dim 64
    (sparse_scaled_dot_product_attention / sparse_cross_attention)."""
    c = ctx(q.device)
    assert q.dtype in HALF and k.dtype == q.dtype and v.dtype == q.dtype
    if out is None:
        out = torch.empty((q.shape[0], heads * 64), dtype=q.dtype, device=q.device)
    c.check(L.lib.p3d_varlen_attention(c.h, _p(q), _rows(q), _p(k), _rows(k), _p(v), _rows(v), _p(out), _rows(out),
                                       _p(cu_q), _p(cu_k), cu_q.shape[0] - 1, max_q, q.shape[0], k.shape[0], heads,
                                       64, scale, _dt(q)))
    return out


def window_partition(coords: torch.Tensor, batch: int, window: int, shift: int, spatial) -> tuple:
    """Shifted-window partition (no reference; the config-3 decoder's 8^3
    windows): (perm, cu) with rows in window order and per-window offsets
    over all batch*nwx*nwy*nwz windows (empty ones included)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    sx, sy, sz = spatial
    m = int(L.lib.p3d_window_count(batch, window, shift, sx, sy, sz))
    assert m > 0, "bad window grid"
    perm = torch.empty(n, dtype=torch.int32, device=coords.device)
    cu = torch.empty(m + 1, dtype=torch.int32, device=coords.device)
    wsb = int(L.lib.p3d_window_partition_workspace(n, m))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=coords.device)
    c.check(L.lib.p3d_window_partition(c.h, _p(coords), n, batch, window, shift, sx, sy, sz, _p(perm), _p(cu), _p(ws),
                                       wsb))
    return perm, cu


def window_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, perm: torch.Tensor, cu: torch.Tensor,
                     window: int, heads: int, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Self-attention of each row to the rows of its window (p3d_window_attention)."""
    c = ctx(q.device)
    assert q.dtype in HALF and k.dtype == q.dtype and v.dtype == q.dtype
    n = q.shape[0]
    if out is None:
        out = torch.empty((n, heads * 64), dtype=q.dtype, device=q.device)
    sb = int(L.lib.p3d_window_attention_scratch(n, heads))
    scratch = torch.empty(max(sb, 16), dtype=torch.uint8, device=q.device)
    c.check(L.lib.p3d_window_attention(c.h, _p(q), _rows(q), _p(k), _rows(k), _p(v), _rows(v), _p(perm), _p(cu),
                                       cu.shape[0] - 1, window ** 3, n, heads, 64, scale, _dt(q), _p(scratch), sb,
                                       _p(out), _rows(out)))
    return out


# ------------------------------------------------------------ elementwise

def ape_add_(x: torch.Tensor, coords: torch.Tensor) -> torch.Tensor:
    """x += sinusoidal absolute 3D PE of coords (in place, f32)."""
    assert x.dtype == torch.float32 and x.is_contiguous()
    c = ctx(x.device)
    c.check(L.lib.p3d_ape_add(c.h, _p(coords), x.shape[0], x.shape[1], _p(x)))
    return x


def project_features(views, grid_resolution: int, coords: torch.Tensor | None = None, out_dtype=torch.float32,
                     out: torch.Tensor | None = None, valid: torch.Tensor | None = None):
    """Projected image features of grid points (p3d_project_features): views
    is a list of dicts with "feature_map" (f32 [H, W, C] on the device),
    "image_resolution", "camera_angle_x", "distance", "mesh_scale" and an
    optional row-major camera-to-world "transform" (16 floats).  coords None
    projects the whole grid in meshgrid "ij" order.  Returns (out, valid)."""
    fm0 = views[0]["feature_map"]
    dev = fm0.device
    c = ctx(dev)
    arr = (L.ProjectionView * len(views))()
    for i, v in enumerate(views):
        fm = v["feature_map"]
        assert fm.dtype == torch.float32 and fm.is_contiguous() and fm.dim() == 3
        pv = arr[i]
        pv.feature_map = fm.data_ptr()
        pv.height, pv.width, pv.channels = fm.shape
        pv.image_resolution = int(v["image_resolution"])
        pv.camera_angle_x = float(v["camera_angle_x"])
        pv.distance = float(v.get("distance", 2.0))
        pv.mesh_scale = float(v.get("mesh_scale", 1.0))
        t = v.get("transform")
        pv.has_transform = int(t is not None)
        if t is not None:
            for j, x in enumerate([float(a) for a in list(t)]):
                pv.transform_matrix[j] = x
    n = coords.shape[0] if coords is not None else grid_resolution ** 3
    ch = fm0.shape[2]
    if out is None:
        out = torch.empty((n, ch), dtype=out_dtype, device=dev)
    if valid is None:
        valid = torch.empty(n, dtype=torch.uint8, device=dev)
    c.check(L.lib.p3d_project_features(c.h, arr, len(views), grid_resolution, _p(coords), n, _p(out), out.stride(0),
                                       _dt(out), _p(valid)))
    return out, valid


def projection_relative_matrices(c2w, distances):
    """Host math (p3d_projection_relative_matrices, no device needed):
    [n, 16] float32 numpy."""
    import numpy as np
    m = np.ascontiguousarray(np.asarray(c2w, np.float32).reshape(-1, 16))
    d = np.ascontiguousarray(np.asarray(distances, np.float32))
    out = np.empty_like(m)
    rc = L.lib.p3d_projection_relative_matrices(None, m.ctypes.data, d.ctypes.data, m.shape[0], out.ctypes.data)
    if rc != 0:
        raise P3DError(rc, "p3d_projection_relative_matrices failed")
    return out


def slat_normalize(x: torch.Tensor, mean: torch.Tensor, std: torch.Tensor, denormalize: bool = False,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """(x - mean) / std, or x * std + mean (p3d_slat_normalize), f32 rows."""
    assert x.dtype == torch.float32 and x.is_contiguous()
    c = ctx(x.device)
    if out is None:
        out = torch.empty_like(x)
    c.check(L.lib.p3d_slat_normalize(c.h, _p(x), x.shape[0], x.shape[1], _p(mean.contiguous()),
                                     _p(std.contiguous()), int(denormalize), _p(out)))
    return out


def quantize_slat_coords(coords: torch.Tensor, batch: int, low_resolution: int, resolution: int = 1024) -> torch.Tensor:
    """Decoder coordinates -> unique sorted coordinates on the 1024 cascade
    grid (p3d_quantize_slat_coords); returns int32 [m, 4] (reads the count)."""
    c = ctx(coords.device)
    n = coords.shape[0]
    out = torch.empty((max(n, 1), 4), dtype=torch.int32, device=coords.device)
    count = torch.zeros(1, dtype=torch.int64, device=coords.device)
    wsb = int(L.lib.p3d_quantize_slat_coords_workspace(batch))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=coords.device)
    c.check(L.lib.p3d_quantize_slat_coords(c.h, _p(coords.contiguous()), n, batch, low_resolution, resolution,
                                           _p(out), _p(count), _p(ws), wsb))
    c.sync_check()
    return out[:int(count.item())]


def layernorm_modulate(x: torch.Tensor, eps: float, gamma=None, beta=None, mod: torch.Tensor | None = None,
                       batch_offsets: torch.Tensor | None = None, out_dtype=torch.bfloat16,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm (+affine) (+AdaLN: mod rows are [shift(C) | scale(C) | ...])."""
    assert x.dtype == torch.float32 and x.is_contiguous()
    c = ctx(x.device)
    n, ch = x.shape
    if out is None:
        out = torch.empty((n, ch), dtype=out_dtype, device=x.device)
    nb = batch_offsets.shape[0] - 1 if batch_offsets is not None else 0
    c.check(L.lib.p3d_layernorm_modulate(c.h, _p(x), n, ch, eps, _p(gamma), _p(beta), _p(mod),
                                         mod.stride(0) if mod is not None else 0, _p(batch_offsets), nb, _p(out),
                                         _dt(out)))
    return out


def qk_rmsnorm_rope(x: torch.Tensor, heads: int, head_dim: int, gamma: torch.Tensor | None = None,
                    coords: torch.Tensor | None = None, freq_min: float = 1.0, freq_base: float = 10000.0) -> None:
    """In place on 16-bit rows (view with row pitch)."""
    assert x.dtype in HALF
    c = ctx(x.device)
    c.check(L.lib.p3d_qk_rmsnorm_rope(c.h, _p(x), x.shape[0], _rows(x), heads, head_dim, _p(gamma), _p(coords),
                                      freq_min, freq_base, _dt(x)))


def activation(x: torch.Tensor, act: int) -> torch.Tensor:
    c = ctx(x.device)
    out = torch.empty_like(x)
    c.check(L.lib.p3d_activation(c.h, _p(x), x.numel(), act, _dt(x), _p(out)))
    return out


def group_norm_silu(x: torch.Tensor, groups: int, eps: float, gamma, beta, batch_offsets: torch.Tensor,
                    silu: bool = True, out_dtype=torch.bfloat16) -> torch.Tensor:
    c = ctx(x.device)
    n, ch = x.shape
    nb = batch_offsets.shape[0] - 1
    stats = torch.empty(3 * nb * groups, dtype=torch.float64, device=x.device)
    out = torch.empty((n, ch), dtype=out_dtype, device=x.device)
    c.check(L.lib.p3d_group_norm_silu(c.h, _p(x), n, ch, groups, eps, _p(gamma), _p(beta), _p(batch_offsets), nb,
                                      int(silu), _p(stats), _p(out), _dt(out)))
    return out


def euler_cfg_step(x: torch.Tensor, v_pos: torch.Tensor, v_neg: torch.Tensor | None, batch_offsets: torch.Tensor,
                   t: float, t_next: float, guidance: float, guidance_rescale: float, sigma_min: float,
                   x0_out: torch.Tensor | None = None) -> None:
    c = ctx(x.device)
    n, ch = x.shape
    nb = batch_offsets.shape[0] - 1
    stats = torch.empty(4 * nb, dtype=torch.float64, device=x.device)
    c.check(L.lib.p3d_euler_cfg_step(c.h, _p(x), _p(v_pos), _p(v_neg), n, ch, _p(batch_offsets), nb, t, t_next,
                                     guidance, guidance_rescale, sigma_min, _p(stats), _p(x0_out)))


def convert(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    c = ctx(x.device)
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    c.check(L.lib.p3d_convert(c.h, _p(x), _dt(x), x.numel(), _p(out), _dt(out)))
    return out


def batch_offsets(coords: torch.Tensor, batch: int) -> torch.Tensor:
    """int32 [batch+1] row offsets of a batch-contiguous coordinate list (p3d_batch_offsets)."""
    c = ctx(coords.device)
    off = torch.empty(batch + 1, dtype=torch.int32, device=coords.device)
    c.check(L.lib.p3d_batch_offsets(c.h, _p(coords), coords.shape[0], batch, _p(off)))
    return off


def pack_operand(x: torch.Tensor, ld: int, dtype: torch.dtype) -> torch.Tensor:
    """f32 [rows, cols] -> 16-bit [rows, ld] with zero columns cols..ld (p3d_pack_operand)."""
    assert x.dtype == torch.float32 and x.is_contiguous() and ld >= x.shape[1]
    c = ctx(x.device)
    out = torch.empty((x.shape[0], ld), dtype=dtype, device=x.device)
    c.check(L.lib.p3d_pack_operand(c.h, _p(x), x.shape[0], x.shape[1], _p(out), ld, _dt(out)))
    return out


def batch_offsets_of(coords: torch.Tensor, batch: int) -> torch.Tensor:
    """int32 [batch+1] row offsets of a batch-contiguous coordinate list."""
    b = coords[:, 0].to(torch.int64)
    counts = torch.bincount(b, minlength=batch)
    off = torch.zeros(batch + 1, dtype=torch.int32, device=coords.device)
    off[1:] = torch.cumsum(counts, 0).to(torch.int32)
    return off
