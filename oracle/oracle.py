"""CPU restatement (numpy, float32) of Pixal3D.cpp's sparse-voxel SLat hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA product in
``pixal3d/cpp_b200``; it is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline leg.  The product
never imports or calls it.

Parity status: PINNED.  ``tests/test_oracle_pin.py`` checks every function here
against (a) the reference's own deterministic fixtures, compiled from the
reference sources and run in this container (outputs committed under
``tests/golden/``), and (b) the compiled reference itself (``oracle/_ref``) on
seeded inputs, when that library is present.  Functions marked "no reference"
restate architecture pieces named by the benchmark configs that the reference
does not implement (GroupNorm32, SparseResBlock3d, nearest 2x upsample,
sinusoidal absolute PE, windowed attention); their parity is "vs own
restatement" only.

Conventions (match include/pixal3d/sparse.h:12-40 of the reference):
  coords  int32 [N, 4] rows of (batch, x, y, z), contiguous by batch
  feats   float32 [N, C] row-major
  linear weights [out, in]; conv weights [27, out, in] with
  kernel = kd*9 + kh*3 + kw, offsets (kd-1, kh-1, kw-1) applied to (x, y, z).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# Coordinates, hashing, neighbour maps
# --------------------------------------------------------------------------

def _fits16(c: np.ndarray, margin: int = 0) -> bool:
    return c.size == 0 or bool(c[:, 0].min() >= 0 and c[:, 0].max() < 2 ** 15 and
                               c[:, 1:].min() - margin >= -2 ** 15 and c[:, 1:].max() + margin < 2 ** 15)


def pack_keys(coords: np.ndarray, wide: bool | None = None) -> np.ndarray:
    """Keys whose order is the lexicographic order of the (b,x,y,z) rows and
    which are equal exactly when the rows are (the reference's CoordHash
    compares full int32 fields, src/sparse.cpp:34-42).  While every field
    fits 16 bits (b in [0, 2^15), x/y/z in [-2^15, 2^15)) the key is one int64;
    otherwise (or with wide=True) it is a 32-byte big-endian record of the
    four fields, slower but exact for any int64 values."""
    c = np.asarray(coords).astype(np.int64)
    if wide is None:
        wide = not _fits16(c)
    if not wide:
        return (c[:, 0] << 48) | ((c[:, 1] + 32768) << 32) | ((c[:, 2] + 32768) << 16) | (c[:, 3] + 32768)
    return np.ascontiguousarray((c + 2 ** 62).astype(">u8")).view("V32").ravel()


def neighbor_map27(coords: np.ndarray) -> np.ndarray:
    """27-offset gather map, layout [27][N], missing neighbour -> N.

    Follows build_reference_neighbor_gather_map (src/slat_decoder.cpp:670-714):
    for kernel index k = kd*9 + kh*3 + kw the neighbour of point p is the row
    holding (b, x+kd-1, y+kh-1, z+kw-1), else the sentinel N.
    """
    n = coords.shape[0]
    c = np.asarray(coords).astype(np.int64)
    wide = not _fits16(c, margin=1)  # one key form for the points and all probes
    keys = pack_keys(c, wide)
    order = np.argsort(keys, kind="stable")
    sk = keys[order]
    out = np.full((27, n), n, dtype=np.int32)
    for k in range(27):
        kd, kh, kw = k // 9, (k // 3) % 3, k % 3
        probe = c.copy()
        probe[:, 1] += kd - 1
        probe[:, 2] += kh - 1
        probe[:, 3] += kw - 1
        pk = pack_keys(probe, wide)
        pos = np.searchsorted(sk, pk)
        pos_c = np.minimum(pos, n - 1)
        hit = (pos < n) & (sk[pos_c] == pk)
        out[k, hit] = order[pos_c[hit]].astype(np.int32)
    return out


def coords_fingerprint(coords: np.ndarray) -> int:
    """FNV-1a over the coordinate bytes (src/slat_decoder.cpp:522-534)."""
    h = 1469598103934665603
    for byte in np.ascontiguousarray(coords, dtype=np.int32).tobytes():
        h ^= byte
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


VALID_ERRORS = ("sparse coordinate is outside its shape", "sparse coordinates contain a duplicate point",
                "sparse coordinates must be contiguous by batch", "sparse features contain a non-finite value")


def validate_first(coords, feats, batch, shape) -> tuple[int, int] | None:
    """First failing (row, check) of SparseTensorF32::valid's sequential scan
    (src/sparse.cpp:286-334): for each row in order, 0 = outside the shape,
    1 = same coordinate as an earlier row, 2 = batch index lower than the
    previous row's, 3 = a non-finite feature.  None when every row passes."""
    c = np.asarray(coords, np.int64).reshape(-1, 4)
    n = c.shape[0]
    code = np.full(n, 4, np.int64)
    if n:
        oob = (c[:, 0] < 0) | (c[:, 0] >= batch) | (c[:, 1] < 0) | (c[:, 1] >= shape[0]) | \
              (c[:, 2] < 0) | (c[:, 2] >= shape[1]) | (c[:, 3] < 0) | (c[:, 3] >= shape[2])
        _, first_idx, inv = np.unique(c, axis=0, return_index=True, return_inverse=True)
        dup = first_idx[inv.ravel()] != np.arange(n)
        dec = np.zeros(n, bool)
        dec[1:] = c[:-1, 0] > c[1:, 0]
        nonfinite = ~np.isfinite(np.asarray(feats, np.float32).reshape(n, -1)).all(axis=1) if feats is not None \
            else np.zeros(n, bool)
        for k, m in enumerate((oob, dup, dec, nonfinite)):
            code[(code == 4) & m] = k
    bad = np.nonzero(code < 4)[0]
    return None if bad.size == 0 else (int(bad[0]), int(code[bad[0]]))


def validate(coords, feats, batch, shape) -> str | None:
    """SparseTensorF32::valid (src/sparse.cpp:241-335): shape, then the
    sequential per-row scan of validate_first.  Returns None or the
    reference's error message."""
    if batch <= 0 or feats.shape[1] <= 0 or min(shape) <= 0:
        return "invalid sparse tensor shape"
    r = validate_first(coords, feats, batch, shape)
    return None if r is None else VALID_ERRORS[r[1]]


# --------------------------------------------------------------------------
# Dense-per-point ops
# --------------------------------------------------------------------------

def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """y = b + W x per row (sparse_linear, src/sparse.cpp:337-451;
    varlen_linear :453-488; row_linear src/slat_flow.cpp:85-111)."""
    return (x.astype(F32) @ w.astype(F32).T + b.astype(F32)).astype(F32)


def layer_norm(x: np.ndarray, eps: float, gamma=None, beta=None) -> np.ndarray:
    """Two-pass per-row LayerNorm (sparse_layer_norm, src/sparse.cpp:490-534)."""
    x = x.astype(F32)
    mean = x.mean(axis=1, keepdims=True, dtype=F32)
    d = x - mean
    var = (d * d).mean(axis=1, keepdims=True, dtype=F32)
    y = d * (F32(1.0) / np.sqrt(var + F32(eps)))
    if gamma is not None:
        y = y * gamma.astype(F32) + beta.astype(F32)
    return y.astype(F32)


def silu_stable(x: np.ndarray) -> np.ndarray:
    """SiLU as written in src/slat_flow.cpp:79-83 (sign-split form)."""
    x = x.astype(F32)
    with np.errstate(over="ignore"):
        pos = x / (F32(1) + np.exp(-x))
        e = np.exp(x)
        neg = x * e / (F32(1) + e)
    return np.where(x >= 0, pos, neg).astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    """SiLU x * 1/(1+exp(-x)) (src/slat_decoder.cpp:68-78, src/flow.cpp:83-88)."""
    x = x.astype(F32)
    with np.errstate(over="ignore"):
        return (x * (F32(1) / (F32(1) + np.exp(-x)))).astype(F32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """GELU, tanh approximation (src/sparse_transformer.cpp:123-134)."""
    x = x.astype(F32)
    return (F32(0.5) * x * (F32(1) + np.tanh(F32(0.7978845608028654) * (x + F32(0.044715) * x * x * x)))).astype(F32)


def affine_modulate(x, block_mod, tmod, batch_idx, channels, offset):
    """x*(1+scale)+shift with shift = mod[offset:offset+C], scale =
    mod[offset+C:offset+2C], mod = block.modulation + tmod[batch]
    (src/sparse_transformer.cpp:71-99)."""
    mod = block_mod[None, :] + tmod.reshape(-1, 6 * channels)[batch_idx]
    shift = mod[:, offset:offset + channels]
    scale = mod[:, offset + channels:offset + 2 * channels]
    return (x * (F32(1) + scale) + shift).astype(F32)


def gate(x, block_mod, tmod, batch_idx, channels, offset):
    """x * (mod[offset:offset+C]) (src/sparse_transformer.cpp:101-121)."""
    mod = block_mod[None, :] + tmod.reshape(-1, 6 * channels)[batch_idx]
    return (x * mod[:, offset:offset + channels]).astype(F32)


def rms_norm_heads(x, heads, head_dim, gamma):
    """x / max(||x||, 1e-12) * sqrt(hd) * gamma per head
    (sparse_multihead_rms_norm src/sparse.cpp:919-954; varlen :956-997)."""
    n = x.shape[0]
    xh = x.astype(F32).reshape(n, heads, head_dim)
    norm = np.sqrt((xh * xh).sum(axis=2, keepdims=True, dtype=F32))
    inv = F32(1) / np.maximum(norm, F32(1e-12))
    y = xh * inv * F32(math.sqrt(head_dim)) * gamma.astype(F32).reshape(1, heads, head_dim)
    return y.reshape(n, heads * head_dim).astype(F32)


def rope_tables(coords, head_dim, fmin=1.0, fbase=10000.0):
    """Per-point cos/sin of each rotation pair (src/sparse.cpp:881-906).
    pairs = hd/2, fd = pairs/3; pair p < 3*fd uses coordinate p//fd with
    frequency fmin / fbase^((p%fd)/fd); remaining pairs are unrotated."""
    pairs = head_dim // 2
    fd = pairs // 3
    freqs = np.array([F32(fmin) / np.power(F32(fbase), F32(i) / F32(fd)) for i in range(fd)], dtype=F32)
    n = coords.shape[0]
    phase = np.zeros((n, pairs), dtype=F32)
    for p in range(3 * fd):
        phase[:, p] = coords[:, 1 + p // fd].astype(F32) * freqs[p % fd]
    return np.cos(phase).astype(F32), np.sin(phase).astype(F32)


def rope(coords, x, heads, head_dim, fmin=1.0, fbase=10000.0):
    """Interleaved (even, odd) 3D RoPE (sparse_rotary_position_embedding,
    src/sparse.cpp:861-917)."""
    n = x.shape[0]
    cos, sin = rope_tables(coords, head_dim, fmin, fbase)
    xh = x.astype(F32).reshape(n, heads, head_dim // 2, 2)
    ev, od = xh[..., 0], xh[..., 1]
    c, s = cos[:, None, :], sin[:, None, :]
    out = np.stack([ev * c - od * s, ev * s + od * c], axis=-1)
    return out.reshape(n, heads * head_dim).astype(F32)


def _softmax_attend(q, k, v, scale, chunk=4096):
    # q [Lq, hd], k [Lk, hd], v [Lk, vd]: two-pass softmax as
    # src/sparse.cpp:754-778.  Rows are independent; long query sets run in
    # chunks of `chunk` rows so the score block stays small.
    if q.shape[0] > chunk:
        return np.concatenate([_softmax_attend(q[i:i + chunk], k, v, scale, chunk)
                               for i in range(0, q.shape[0], chunk)])
    s = (q @ k.T) * F32(scale)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=1, keepdims=True, dtype=F32)
    return (p @ v).astype(F32)


def sdpa(q_batch, q, k_batch, k, v, heads, head_dim, scale):
    """Batch-isolated attention (sparse_scaled_dot_product_attention,
    src/sparse.cpp:704-783).  *_batch are the per-row batch indices."""
    vc = v.shape[1]
    vd = vc // heads
    out = np.zeros((q.shape[0], vc), dtype=F32)
    for b in np.unique(q_batch):
        qi = np.nonzero(q_batch == b)[0]
        ki = np.nonzero(k_batch == b)[0]
        if ki.size == 0:
            raise ValueError("sparse attention has no keys or mismatched key/value rows")
        for h in range(heads):
            out[qi, h * vd:(h + 1) * vd] = _softmax_attend(
                q[qi, h * head_dim:(h + 1) * head_dim], k[ki, h * head_dim:(h + 1) * head_dim],
                v[ki, h * vd:(h + 1) * vd], scale)
    return out


def cross_attention(q_batch, q, offsets, k, v, heads, head_dim, scale):
    """Sparse queries x variable-length K/V (sparse_cross_attention,
    src/sparse.cpp:785-859)."""
    vc = v.shape[1]
    vd = vc // heads
    out = np.zeros((q.shape[0], vc), dtype=F32)
    for b in range(len(offsets) - 1):
        qi = np.nonzero(q_batch == b)[0]
        k0, k1 = int(offsets[b]), int(offsets[b + 1])
        if k1 == k0:
            raise ValueError("sparse cross-attention has an empty key sequence")
        if qi.size == 0:
            continue
        for h in range(heads):
            out[qi, h * vd:(h + 1) * vd] = _softmax_attend(
                q[qi, h * head_dim:(h + 1) * head_dim], k[k0:k1, h * head_dim:(h + 1) * head_dim],
                v[k0:k1, h * vd:(h + 1) * vd], scale)
    return out


# --------------------------------------------------------------------------
# Sparse convolution and topology ops
# --------------------------------------------------------------------------

def subm_conv3d(coords, x, w, b, nbr=None):
    """out[p] = b + sum_k W[k] x[nbr_k(p)] (sparse_submanifold_conv3d,
    src/sparse.cpp:999-1055); missing neighbours contribute zero."""
    n = coords.shape[0]
    if nbr is None:
        nbr = neighbor_map27(coords)
    xz = np.concatenate([x.astype(F32), np.zeros((1, x.shape[1]), F32)], axis=0)
    out = np.zeros((n, w.shape[1]), dtype=F32)
    for k in range(27):
        out += xz[nbr[k]] @ w[k].astype(F32).T
    return (out + b.astype(F32)).astype(F32)


def downsample_mean(coords, x, factor):
    """Mean-pool to coords // factor, output sorted lexicographically
    (sparse_downsample_mean, src/sparse.cpp:536-602).  Returns
    (coords_out, feats_out, parent) where parent[i] is the output row of
    input row i."""
    tc = coords.copy()
    tc[:, 1:] //= factor
    keys = pack_keys(tc)
    uk, parent = np.unique(keys, return_inverse=True)
    m = uk.size
    first = np.zeros(m, dtype=np.int64)
    first[parent[::-1]] = np.arange(coords.shape[0])[::-1]
    oc = tc[first].astype(np.int32)
    sums = np.zeros((m, x.shape[1]), dtype=F32)
    np.add.at(sums, parent, x.astype(F32))
    cnt = np.bincount(parent, minlength=m).astype(F32)
    return oc, (sums / cnt[:, None]).astype(F32), parent.astype(np.int64)


def channel_to_spatial(coords, x, factor, subdiv=None):
    """Subdivide: child c has offset (c%f, (c/f)%f, c/f^2) and features
    x[:, c*Cout:(c+1)*Cout]; with a mask only children with subdiv>0 are kept.
    Output is in parent order then child order
    (sparse_channel_to_spatial, src/sparse.cpp:604-702)."""
    n = coords.shape[0]
    nc = factor ** 3
    cout = x.shape[1] // nc
    child = np.arange(nc)
    off = np.stack([child % factor, (child // factor) % factor, child // (factor * factor)], axis=1)
    oc = np.empty((n, nc, 4), dtype=np.int32)
    oc[:, :, 0] = coords[:, None, 0]
    oc[:, :, 1:] = coords[:, None, 1:] * factor + off[None, :, :]
    of = x.reshape(n, nc, cout)
    if subdiv is None:
        keep = np.ones((n, nc), dtype=bool)
    else:
        keep = subdiv.reshape(n, nc) > 0
    return oc[keep].reshape(-1, 4), of[keep].reshape(-1, cout).astype(F32)


# --------------------------------------------------------------------------
# Transformer block, timestep embedding, flow model, sampler
# --------------------------------------------------------------------------

BLOCK_FIELDS = [
    "modulation", "self_to_qkv_weight", "self_to_qkv_bias", "self_q_gamma", "self_k_gamma",
    "self_to_out_weight", "self_to_out_bias", "norm2_weight", "norm2_bias",
    "cross_to_q_weight", "cross_to_q_bias", "cross_to_kv_weight", "cross_to_kv_bias",
    "cross_q_gamma", "cross_k_gamma", "cross_to_out_weight", "cross_to_out_bias",
    "proj_weight", "proj_bias", "mlp0_weight", "mlp0_bias", "mlp2_weight", "mlp2_bias",
]
"""Field order of SparseTransformerBlockWeightsF32
(include/pixal3d/sparse_transformer.h:30-54)."""


@dataclass
class BlockConfig:
    """SparseTransformerBlockConfig (include/pixal3d/sparse_transformer.h:13-27)."""
    channels: int
    num_heads: int
    mlp_hidden: int
    context_channels: int
    proj_in_channels: int = 0
    norm_eps: float = 1e-6
    rope_freq_min: float = 1.0
    rope_freq_base: float = 10000.0
    use_rope: bool = True
    qk_rms_norm: bool = True
    qk_rms_norm_cross: bool = True
    use_projection: bool = False


def transformer_block(coords, x, tmod, ctx_offsets, ctx, proj, cfg: BlockConfig, w: dict):
    """ModulatedSparseTransformerCrossBlock
    (sparse_transformer_cross_block_f32, src/sparse_transformer.cpp:138-292)."""
    C, H = cfg.channels, cfg.num_heads
    hd = C // H
    bidx = coords[:, 0].astype(np.int64)
    scale = F32(1.0) / F32(math.sqrt(hd))
    # self-attention branch (:194-235)
    h = affine_modulate(layer_norm(x, cfg.norm_eps), w["modulation"], tmod, bidx, C, 0)
    qkv = linear(h, w["self_to_qkv_weight"], w["self_to_qkv_bias"])
    q, k, v = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
    if cfg.qk_rms_norm:
        q = rms_norm_heads(q, H, hd, w["self_q_gamma"])
        k = rms_norm_heads(k, H, hd, w["self_k_gamma"])
    if cfg.use_rope:
        q = rope(coords, q, H, hd, cfg.rope_freq_min, cfg.rope_freq_base)
        k = rope(coords, k, H, hd, cfg.rope_freq_min, cfg.rope_freq_base)
    a = sdpa(bidx, q, bidx, k, v, H, hd, scale)
    o = gate(linear(a, w["self_to_out_weight"], w["self_to_out_bias"]), w["modulation"], tmod, bidx, C, 2 * C)
    out = (x + o).astype(F32)
    # cross-attention branch (:237-275)
    ci = layer_norm(out, cfg.norm_eps, w["norm2_weight"], w["norm2_bias"])
    cq = linear(ci, w["cross_to_q_weight"], w["cross_to_q_bias"])
    if cfg.qk_rms_norm_cross:
        cq = rms_norm_heads(cq, H, hd, w["cross_q_gamma"])
    kv = linear(ctx, w["cross_to_kv_weight"], w["cross_to_kv_bias"])
    ck, cv = kv[:, :C], kv[:, C:]
    if cfg.qk_rms_norm_cross:
        ck = rms_norm_heads(ck, H, hd, w["cross_k_gamma"])
    ca = cross_attention(bidx, cq, ctx_offsets, ck, cv, H, hd, scale)
    co = linear(ca, w["cross_to_out_weight"], w["cross_to_out_bias"])
    if cfg.use_projection:
        co = (co + linear(proj, w["proj_weight"], w["proj_bias"])).astype(F32)
    out = (out + co).astype(F32)
    # MLP branch (:277-290)
    m = affine_modulate(layer_norm(out, cfg.norm_eps), w["modulation"], tmod, bidx, C, 3 * C)
    m = gelu_tanh(linear(m, w["mlp0_weight"], w["mlp0_bias"]))
    m = gate(linear(m, w["mlp2_weight"], w["mlp2_bias"]), w["modulation"], tmod, bidx, C, 5 * C)
    return (out + m).astype(F32)


def timestep_embedding(t, dim=256, max_period=10000):
    """cos || sin sinusoidal embedding (src/flow.cpp:92-123)."""
    t = np.asarray(t, dtype=F32)
    half = dim // 2
    log_period = F32(math.log(float(max_period)))
    frac = np.arange(half, dtype=F32) / F32(half)
    freq = np.exp(-log_period * frac).astype(F32)
    arg = t[:, None] * freq[None, :]
    out = np.zeros((t.shape[0], dim), dtype=F32)
    out[:, :half] = np.cos(arg)
    out[:, half:2 * half] = np.sin(arg)
    return out


def timestep_embed_mlp(t, hidden, w0, b0, w2, b2, freq_dim=256):
    """Linear -> SiLU -> Linear (src/flow.cpp:125-180)."""
    e = timestep_embedding(t, freq_dim)
    return linear(silu(linear(e, w0, b0)), w2, b2)


FLOW_TOP_FIELDS = [
    "input_weight", "input_bias", "timestep_weight0", "timestep_bias0", "timestep_weight2",
    "timestep_bias2", "modulation_weight", "modulation_bias", "output_weight", "output_bias",
]
"""Field order of SLatFlowWeightsF32 (include/pixal3d/slat_flow.h:39-51)."""


@dataclass
class FlowHParams:
    """SLatFlowHParams subset (include/pixal3d/slat_flow.h:12-37), plus the
    benchmark-config extensions that have no reference: pe_mode 'ape'
    (sinusoidal absolute 3D PE) and io_resblocks > 0 (SparseResBlock3d input
    and output stages with a 2x downsample/upsample around the trunk)."""
    in_channels: int
    out_channels: int
    model_channels: int
    cond_channels: int
    num_blocks: int
    num_heads: int
    mlp_ratio: float = 4.0
    proj_in_channels: int = 0
    image_attn_mode: str = "cross"
    norm_eps: float = 1e-6
    rope_freq_min: float = 1.0
    rope_freq_base: float = 10000.0
    qk_rms_norm: bool = True
    qk_rms_norm_cross: bool = True
    pe_mode: str = "rope"
    io_resblocks: int = 0
    groups: int = 32

    def block_config(self) -> BlockConfig:
        return BlockConfig(
            channels=self.model_channels, num_heads=self.num_heads,
            mlp_hidden=int(self.model_channels * self.mlp_ratio),
            context_channels=self.cond_channels, proj_in_channels=self.proj_in_channels,
            norm_eps=self.norm_eps, rope_freq_min=self.rope_freq_min,
            rope_freq_base=self.rope_freq_base, use_rope=self.pe_mode == "rope",
            qk_rms_norm=self.qk_rms_norm, qk_rms_norm_cross=self.qk_rms_norm_cross,
            use_projection=self.image_attn_mode == "proj")


def slat_flow_forward(coords, x, timesteps, ctx_offsets, ctx, proj, hp: FlowHParams, w: dict):
    """SLat flow forward (slat_flow_forward_f32, src/slat_flow.cpp:161-249):
    input linear -> t-embedding MLP -> SiLU -> 6C modulation -> blocks ->
    LayerNorm(eps 1e-5) -> output linear.  With hp.io_resblocks the config-2
    input/output stages (no reference) wrap the trunk."""
    h = linear(x, w["input_weight"], w["input_bias"])
    temb = timestep_embed_mlp(timesteps, hp.model_channels, w["timestep_weight0"], w["timestep_bias0"],
                              w["timestep_weight2"], w["timestep_bias2"])
    tmod = linear(silu_stable(temb), w["modulation_weight"], w["modulation_bias"])
    cfg = hp.block_config()
    trunk_coords = coords
    if hp.io_resblocks:
        for i in range(hp.io_resblocks):
            h = resblock3d(coords, h, w["io_in"][i], hp.groups)
        trunk_coords, h, parent = downsample_mean(coords, h, 2)
    if hp.pe_mode == "ape":
        h = (h + absolute_pe(trunk_coords, hp.model_channels)).astype(F32)
    for bw in w["blocks"]:
        h = transformer_block(trunk_coords, h, tmod, ctx_offsets, ctx, proj, cfg, bw)
    if hp.io_resblocks:
        h = h[parent]
        for i in range(hp.io_resblocks):
            h = resblock3d(coords, h, w["io_out"][i], hp.groups)
    return linear(layer_norm(h, 1e-5), w["output_weight"], w["output_bias"])


@dataclass
class SamplerConfig:
    """FlowEulerSamplerConfig (include/pixal3d/flow_sampler.h:14-23)."""
    steps: int = 50
    sigma_min: float = 1e-5
    rescale_t: float = 1.0
    guidance_strength: float = 1.0
    guidance_rescale: float = 0.0
    guidance_interval_min: float = 0.0
    guidance_interval_max: float = 1.0


def sampler_schedule(cfg: SamplerConfig):
    """(t, t_next, guidance) per step (src/flow_sampler.cpp:268-286)."""
    out = []
    steps = F32(cfg.steps)
    r = F32(cfg.rescale_t)
    for i in range(cfg.steps):
        lin = F32(1) - F32(i) / steps
        t = r * lin / (F32(1) + (r - F32(1)) * lin)
        nl = F32(1) - F32(i + 1) / steps
        tn = r * nl / (F32(1) + (r - F32(1)) * nl)
        g = F32(cfg.guidance_strength) if (cfg.guidance_interval_min <= t <= cfg.guidance_interval_max) else F32(1)
        out.append((F32(t), F32(tn), g))
    return out


def batch_std(batch_idx, x, batch):
    """Population std of all values of each batch (sparse_batch_std,
    src/flow_sampler.cpp:164-198)."""
    out = np.zeros(batch, dtype=F32)
    for b in range(batch):
        v = x[batch_idx == b].astype(F32).ravel()
        m = v.sum(dtype=F32) / F32(v.size)
        m2 = (v * v).sum(dtype=F32) / F32(v.size)
        out[b] = np.sqrt(max(m2 - m * m, F32(0)))
    return out


def cfg_combine(state, t, pos, neg, g, cfg: SamplerConfig, batch_idx, batch):
    """CFG blend + optional guidance rescale (src/flow_sampler.cpp:200-241, :299-321)."""
    pred = (g * pos + (F32(1) - g) * neg).astype(F32)
    if cfg.guidance_rescale > 0:
        a = F32(1) - F32(cfg.sigma_min)
        bb = F32(cfg.sigma_min) + a * F32(t)
        x0p = a * state - bb * pos
        x0c = a * state - bb * pred
        sp = batch_std(batch_idx, x0p, batch)
        sc = batch_std(batch_idx, x0c, batch)
        ratio = np.where(sc != 0, sp / np.where(sc != 0, sc, 1), F32(1)).astype(F32)[batch_idx][:, None]
        gr = F32(cfg.guidance_rescale)
        x0c = gr * (x0c * ratio) + (F32(1) - gr) * x0c
        pred = ((a * state - x0c) / bb).astype(F32)
    return pred


def flow_euler_sample(state, cfg: SamplerConfig, model, batch_idx, batch, record_x0=False):
    """Flow-Euler integration t=1 -> 0 (flow_euler_sample_f32,
    src/flow_sampler.cpp:245-343).  model(state, 1000*t, conditional) -> v."""
    x = state.astype(F32).copy()
    x0_last = None
    a = F32(1) - F32(cfg.sigma_min)
    for t, tn, g in sampler_schedule(cfg):
        if g == 1:
            pred = model(x, F32(1000) * t, True)
        elif g == 0:
            pred = model(x, F32(1000) * t, False)
        else:
            pos = model(x, F32(1000) * t, True)
            neg = model(x, F32(1000) * t, False)
            pred = cfg_combine(x, t, pos, neg, g, cfg, batch_idx, batch)
        if record_x0:
            x0_last = (a * x - (F32(cfg.sigma_min) + a * t) * pred).astype(F32)
        x = (x - (t - tn) * pred).astype(F32)
    return (x, x0_last) if record_x0 else x


# --------------------------------------------------------------------------
# SLat decoder
# --------------------------------------------------------------------------

def convnext_block(coords, x, w, eps, nbr=None):
    """conv -> LN(affine) -> Linear -> SiLU -> Linear -> + x
    (sparse_convnext_block_f32, src/slat_decoder.cpp:185-222).
    w keys: norm_w, norm_b, conv_w, conv_b, mlp0_w, mlp0_b, mlp2_w, mlp2_b."""
    h = subm_conv3d(coords, x, w["conv_w"], w["conv_b"], nbr)
    h = layer_norm(h, eps, w["norm_w"], w["norm_b"])
    h = silu(linear(h, w["mlp0_w"], w["mlp0_b"]))
    return (linear(h, w["mlp2_w"], w["mlp2_b"]) + x).astype(F32)


def repeat_channels(x, out_channels):
    """dest[c*r + j] = src[c] (src/slat_decoder.cpp:80-109)."""
    return np.repeat(x, out_channels // x.shape[1], axis=1).astype(F32)


def resblock_c2s(coords, x, w, eps, out_channels, pred_subdiv, subdiv=None, nbr=None):
    """SparseResBlockC2S3d (sparse_resblock_c2s_f32, src/slat_decoder.cpp:224-288).
    w keys: norm1_w, norm1_b, conv1_w, conv1_b, conv2_w, conv2_b,
    subdiv_w, subdiv_b.  Returns (coords_out, feats_out, predicted_logits)."""
    pred = None
    if pred_subdiv:
        pred = linear(x, w["subdiv_w"], w["subdiv_b"])
        subdiv = pred
    h = silu(layer_norm(x, eps, w["norm1_w"], w["norm1_b"]))
    packed = subm_conv3d(coords, h, w["conv1_w"], w["conv1_b"], nbr)
    fc, hs = channel_to_spatial(coords, packed, 2, subdiv)
    _, skip = channel_to_spatial(coords, x, 2, subdiv)
    skip = repeat_channels(skip, out_channels)
    h = silu(layer_norm(hs, eps))
    h = subm_conv3d(fc, h, w["conv2_w"], w["conv2_b"])
    return fc, (h + skip).astype(F32), pred


def decoder_forward(coords, x, cfg: dict, w: dict, guides=None):
    """SLat decoder stack (slat_decoder_forward_f32, src/slat_decoder.cpp:290-376).
    cfg: model_channels, num_blocks, norm_eps, pred_subdiv, out_channels.
    w: from_latent_w/b, output_w/b, blocks (list of dicts, level order)."""
    h = linear(x, w["from_latent_w"], w["from_latent_b"])
    preds = []
    bi = 0
    levels = len(cfg["model_channels"])
    for level in range(levels):
        nbr = neighbor_map27(coords)
        for _ in range(cfg["num_blocks"][level]):
            h = convnext_block(coords, h, w["blocks"][bi], cfg["norm_eps"], nbr)
            bi += 1
        if level + 1 < levels:
            guide = guides[level] if guides is not None else None
            coords, h, p = resblock_c2s(coords, h, w["blocks"][bi], cfg["norm_eps"],
                                        cfg["model_channels"][level + 1], cfg["pred_subdiv"], guide, nbr)
            if p is not None:
                preds.append(p)
            bi += 1
    out = linear(layer_norm(h, 1e-5), w["output_w"], w["output_b"])
    return coords, out, preds


# --------------------------------------------------------------------------
# Benchmark-config pieces with NO reference implementation (own restatement)
# --------------------------------------------------------------------------

def group_norm(batch_idx, x, groups, eps=1e-5, gamma=None, beta=None, batch=None):
    """No reference.  GroupNorm over the points of each batch item: for batch b
    and group g, mean/var over all rows of b and the C/groups channels of g
    (population variance), then per-channel affine."""
    n, c = x.shape
    gs = c // groups
    out = np.empty_like(x, dtype=F32)
    nb = int(batch_idx.max()) + 1 if batch is None else batch
    for b in range(nb):
        rows = batch_idx == b
        xb = x[rows].astype(np.float64).reshape(-1, groups, gs)
        m = xb.mean(axis=(0, 2), keepdims=True)
        v = ((xb - m) ** 2).mean(axis=(0, 2), keepdims=True)
        y = ((xb - m) / np.sqrt(v + eps)).reshape(-1, c)
        if gamma is not None:
            y = y * gamma + beta
        out[rows] = y.astype(F32)
    return out


def resblock3d(coords, x, w, groups=32, eps=1e-5, nbr=None):
    """No reference.  SparseResBlock3d of the benchmark config:
    x + conv2(SiLU(GN(conv1(SiLU(GN(x)))))).  w keys: gn1_w, gn1_b, conv1_w,
    conv1_b, gn2_w, gn2_b, conv2_w, conv2_b."""
    if nbr is None:
        nbr = neighbor_map27(coords)
    bidx = coords[:, 0].astype(np.int64)
    h = silu(group_norm(bidx, x, groups, eps, w["gn1_w"], w["gn1_b"]))
    h = subm_conv3d(coords, h, w["conv1_w"], w["conv1_b"], nbr)
    h = silu(group_norm(bidx, h, groups, eps, w["gn2_w"], w["gn2_b"]))
    h = subm_conv3d(coords, h, w["conv2_w"], w["conv2_b"], nbr)
    return (x + h).astype(F32)


def absolute_pe(coords, channels):
    """No reference.  Sinusoidal absolute 3D PE: per axis a in (x,y,z), with
    fd = channels // 6 frequencies f_i = 1 / 10000^(i/fd), the block
    [sin(c_a f_i), cos(c_a f_i)]; the three blocks are concatenated and zero
    padded to `channels`."""
    fd = channels // 6
    f = (F32(1) / np.power(F32(10000), np.arange(fd, dtype=F32) / F32(fd))).astype(F32)
    parts = []
    for a in range(3):
        arg = coords[:, 1 + a].astype(F32)[:, None] * f[None, :]
        parts += [np.sin(arg), np.cos(arg)]
    pe = np.concatenate(parts, axis=1).astype(F32)
    if pe.shape[1] < channels:
        pe = np.concatenate([pe, np.zeros((pe.shape[0], channels - pe.shape[1]), F32)], axis=1)
    return pe


def window_partition(coords, window, shift):
    """No reference.  Shifted-window grouping for windowed attention: window id
    of a point = (b, (x+shift)//w, (y+shift)//w, (z+shift)//w).  Returns
    (order, cu_seqlens) where order lists rows grouped by window (windows in
    lexicographic order, rows in input order inside a window)."""
    wc = coords.astype(np.int64).copy()
    wc[:, 1:] = (wc[:, 1:] + shift) // window
    keys = pack_keys(wc)
    order = np.argsort(keys, kind="stable")
    _, counts = np.unique(keys[order], return_counts=True)
    cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return order, cu


def varlen_attention(q, k, v, cu_q, cu_k, heads, head_dim, scale):
    """Attention over packed sequences given cumulative offsets."""
    out = np.zeros((q.shape[0], v.shape[1]), dtype=F32)
    vd = v.shape[1] // heads
    for s in range(len(cu_q) - 1):
        q0, q1, k0, k1 = int(cu_q[s]), int(cu_q[s + 1]), int(cu_k[s]), int(cu_k[s + 1])
        if q1 == q0:
            continue
        for h in range(heads):
            out[q0:q1, h * vd:(h + 1) * vd] = _softmax_attend(
                q[q0:q1, h * head_dim:(h + 1) * head_dim], k[k0:k1, h * head_dim:(h + 1) * head_dim],
                v[k0:k1, h * vd:(h + 1) * vd], scale)
    return out


def window_partition_grid(coords, batch, window, shift, spatial):
    """No reference.  window_partition over the full window grid, the layout
    of p3d_window_partition: windows numbered w = ((b*nwx + wx)*nwy + wy)*nwz
    + wz with nw_d = ceil((s_d + shift) / window) (the same lexicographic
    window order), cu over every window, empty ones included (cu[-1] = N).
    perm lists rows by window, then by row index."""
    c = np.asarray(coords, dtype=np.int64)
    nw = [-(-(int(s) + shift) // window) for s in spatial]
    w = ((c[:, 0] * nw[0] + (c[:, 1] + shift) // window) * nw[1] + (c[:, 2] + shift) // window) * nw[2] + \
        (c[:, 3] + shift) // window
    m = batch * nw[0] * nw[1] * nw[2]
    perm = np.argsort(w, kind="stable").astype(np.int32)
    cu = np.zeros(m + 1, dtype=np.int32)
    cu[1:] = np.cumsum(np.bincount(w, minlength=m))
    return perm, cu


def window_attention(q, k, v, coords, window, shift, heads, head_dim, scale):
    """No reference.  Each row attends to the rows of its shifted window
    (window_partition), per head; output rows in the input order."""
    order, cu = window_partition(coords, window, shift)
    o = varlen_attention(q[order], k[order], v[order], cu, cu, heads, head_dim, scale)
    out = np.empty_like(o)
    out[order] = o
    return out


# --------------------------------------------------------------------------
# Config-3 decoder (shifted-window transformer + subdivide stages): NO
# reference implementation; restated from the benchmark configuration.
# --------------------------------------------------------------------------

def swin_block(coords, x, w, heads, window, shift, spatial, eps=1e-6):
    """No reference.  Pre-norm transformer block with shifted-window
    self-attention: x += Wo·attn_window(LN1(x)); x += W2·gelu_tanh(W1·LN2(x)).
    LayerNorms with affine (eps 1e-6), head_dim 64, scale 1/8, no q/k norm.
    w keys: norm1_w/b, qkv_w [3C, C], qkv_b, out_w [C, C], out_b, norm2_w/b,
    mlp0_w [rC, C], mlp0_b, mlp2_w [C, rC], mlp2_b."""
    c = x.shape[1]
    a = layer_norm(x, eps, w["norm1_w"], w["norm1_b"])
    qkv = linear(a, w["qkv_w"], w["qkv_b"])
    o = window_attention(qkv[:, :c], qkv[:, c:2 * c], qkv[:, 2 * c:], coords, window, shift, heads, 64,
                         1.0 / 8.0)
    x = (x + linear(o, w["out_w"], w["out_b"])).astype(F32)
    a = layer_norm(x, eps, w["norm2_w"], w["norm2_b"])
    h = gelu_tanh(linear(a, w["mlp0_w"], w["mlp0_b"]))
    return (x + linear(h, w["mlp2_w"], w["mlp2_b"])).astype(F32)


def subdivide(coords, x, mask):
    """No reference.  SparseSubdivide x2: every parent row spawns the children
    (2x+dx, 2y+dy, 2z+dz), child c = dx + 2 dy + 4 dz, kept where mask[:, c] > 0;
    each kept child copies its parent's features.  Output in parent order,
    then child order (the channel_to_spatial layout)."""
    return channel_to_spatial(coords, np.tile(x, (1, 8)), 2, mask)


def resblock3d_io(coords, x, w, groups=32, eps=1e-5, nbr=None):
    """No reference.  SparseResBlock3d with a channel change:
    conv2(SiLU(GN(conv1(SiLU(GN(x)))))) + skip(x), skip = linear C_in -> C_out.
    w keys: gn1_w/b, conv1_w [27, Co, Ci], conv1_b, gn2_w/b, conv2_w [27, Co, Co],
    conv2_b, skip_w [Co, Ci], skip_b."""
    if nbr is None:
        nbr = neighbor_map27(coords)
    bidx = coords[:, 0].astype(np.int64)
    h = silu(group_norm(bidx, x, groups, eps, w["gn1_w"], w["gn1_b"]))
    h = subm_conv3d(coords, h, w["conv1_w"], w["conv1_b"], nbr)
    h = silu(group_norm(bidx, h, groups, eps, w["gn2_w"], w["gn2_b"]))
    h = subm_conv3d(coords, h, w["conv2_w"], w["conv2_b"], nbr)
    return (h + linear(x, w["skip_w"], w["skip_b"])).astype(F32)


def swin_decoder_forward(coords, x, cfg: dict, w: dict, masks):
    """No reference.  Config-3 SLat decoder: latent -> linear to C0 + absolute
    3D PE -> num_blocks shifted-window blocks (shift 0 on even blocks,
    window/2 on odd) -> per stage s: subdivide with masks[s], then
    resblock3d_io to stage_channels[s] -> LayerNorm (eps 1e-5, no affine) ->
    linear to out_channels.  cfg: model_channels, num_heads, window, spatial
    (grid extent of the input level), groups.  w: from_latent_w/b, blocks,
    stages, output_w/b.  Returns (coords, out)."""
    c0 = cfg["model_channels"]
    h = (linear(x, w["from_latent_w"], w["from_latent_b"]) + absolute_pe(coords, c0)).astype(F32)
    sp = (cfg["spatial"],) * 3
    for i, bw in enumerate(w["blocks"]):
        shift = 0 if i % 2 == 0 else cfg["window"] // 2
        h = swin_block(coords, h, bw, cfg["num_heads"], cfg["window"], shift, sp)
    for s, sw in enumerate(w["stages"]):
        coords, h = subdivide(coords, h, masks[s])
        h = resblock3d_io(coords, h, sw, cfg.get("groups", 32))
    out = linear(layer_norm(h, 1e-5), w["output_w"], w["output_b"])
    return coords, out


# --------------------------------------------------------------------------
# Projection conditioning (image_attn_mode=proj producer)
# --------------------------------------------------------------------------

@dataclass
class ProjCamera:
    """ProjectionCamera (include/pixal3d/projection.h:13-27)."""
    camera_angle_x: float = 0.2
    distance: float = 2.0
    mesh_scale: float = 1.0
    transform: np.ndarray | None = None  # row-major [16] camera-to-world, or None (front view)


def front_matrix(distance: float) -> np.ndarray:
    """src/projection.cpp:21-29: canonical front-view camera-to-world."""
    d = F32(distance)
    return np.array([1, 0, 0, 0, 0, 0, -1, -d, 0, 1, 0, 0, 0, 0, 0, 1], F32)


def matmul4(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """multiply4x4 (src/projection.cpp:31-45): f32 sum over k in order."""
    a = np.asarray(a, F32).reshape(4, 4)
    b = np.asarray(b, F32).reshape(4, 4)
    out = np.zeros((4, 4), F32)
    for r in range(4):
        for c in range(4):
            v = F32(0)
            for k in range(4):
                v = F32(v + F32(a[r, k] * b[k, c]))
            out[r, c] = v
    return out.reshape(16)


def invert4(m: np.ndarray):
    """invert4x4 (src/projection.cpp:47-98): Gauss-Jordan on [M | I] with
    partial pivoting (first row of largest |pivot|), f32 arithmetic; None when
    the pivot is not > 1e-8 or not finite."""
    a = np.zeros((4, 8), F32)
    a[:, :4] = np.asarray(m, F32).reshape(4, 4)
    for r in range(4):
        a[r, r + 4] = 1
    for col in range(4):
        piv = col
        pabs = abs(a[piv, col])
        for row in range(col + 1, 4):
            if abs(a[row, col]) > pabs:
                piv, pabs = row, abs(a[row, col])
        if not (pabs > F32(1e-8)) or not np.isfinite(pabs):
            return None
        if piv != col:
            a[[piv, col]] = a[[col, piv]]
        s = a[col, col]
        a[col] = (a[col] / s).astype(F32)
        for row in range(4):
            if row == col:
                continue
            f = a[row, col]
            if f == 0:
                continue
            a[row] = (a[row] - (f * a[col]).astype(F32)).astype(F32)
    return np.ascontiguousarray(a[:, 4:]).reshape(16)


def projection_constants(cam: ProjCamera, image_resolution: int) -> dict:
    """prepare_projection_view (src/projection.cpp:233-259) and the option
    checks of validate_options (:205-231).  Raises ValueError with the
    reference's messages."""
    if image_resolution <= 0:
        raise ValueError("image_resolution must be positive")
    ang = F32(cam.camera_angle_x)
    if not (F32(0) < ang < F32(math.pi)) or not np.isfinite(ang):
        raise ValueError("camera_angle_x must be finite and in (0, pi)")
    if not (F32(cam.mesh_scale) > 0) or not np.isfinite(F32(cam.mesh_scale)):
        raise ValueError("mesh_scale must be finite and positive")
    if cam.transform is None and (not (F32(cam.distance) > 0) or not np.isfinite(F32(cam.distance))):
        raise ValueError("distance must be finite and positive")
    c2w = front_matrix(cam.distance) if cam.transform is None else np.asarray(cam.transform, F32).reshape(16)
    w2c = invert4(c2w)
    if w2c is None:
        raise ValueError("camera transform matrix is singular")
    focal = F32(F32(16.0) / F32(math.tan(float(F32(ang * F32(0.5))))))
    return {"w2c": w2c, "scale": F32(F32(1.0) / F32(F32(cam.mesh_scale) * F32(2.0))),
            "focal_px": F32(F32(focal * F32(image_resolution)) / F32(32.0)),
            "half": F32(F32(image_resolution) * F32(0.5))}


def grid_base(i: np.ndarray, r: int) -> np.ndarray:
    """-1 + 2 i / (r - 1) as in project_one (src/projection.cpp:276-291)."""
    if r == 1:
        return np.zeros(i.shape, F32)
    return (F32(-1.0) + ((F32(2.0) * i.astype(F32)) / F32(r - 1)).astype(F32)).astype(F32)


def project_points(ix, iy, iz, r: int, k: dict, image_resolution: int):
    """project_point (src/projection.cpp:116-146) of grid cells (ix, iy, iz)
    after the (x, y, z) -> (x, -z, y) * scale map (:293-298).  Returns
    x_pixel, y_pixel, valid (float32, float32, bool arrays)."""
    bx, by, bz = grid_base(ix, r), grid_base(iy, r), grid_base(iz, r)
    s = k["scale"]
    x = (bx * s).astype(F32)
    y = (-bz * s).astype(F32)
    z = (by * s).astype(F32)
    w = k["w2c"]

    def row(o):
        t = (F32(w[o]) * x).astype(F32) + (F32(w[o + 1]) * y).astype(F32)
        t = t.astype(F32) + (F32(w[o + 2]) * z).astype(F32)
        return (t.astype(F32) + F32(w[o + 3])).astype(F32)

    xc, yc, zc = row(0), row(4), row(8)
    depth = (-zc).astype(F32)
    den = ((-zc).astype(F32) + F32(1e-8)).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        xn = ((k["focal_px"] * xc).astype(F32) / den).astype(F32)
        yn = ((k["focal_px"] * yc).astype(F32) / den).astype(F32)
    xp = (xn + k["half"]).astype(F32)
    yp = ((-yn).astype(F32) + k["half"]).astype(F32)
    res = F32(image_resolution)
    valid = (xp >= 0) & (xp < res) & (yp >= 0) & (yp < res) & (depth > 0)
    return xp, yp, valid


def _clamp_ref(v, hi):
    """std::max(0, std::min(v, hi)) with the std:: comparison semantics
    (a NaN input ends at 0)."""
    t = np.where(F32(hi) < v, F32(hi), v)
    return np.where(F32(0) < t, t, F32(0)).astype(F32)


def bilinear_sample(fmap: np.ndarray, xp, yp, image_resolution: int) -> np.ndarray:
    """bilinear_weights + sample_bilinear_channel (src/projection.cpp:155-203):
    grid_sample bilinear, align_corners=False, padding border.  fmap f32
    [H, W, C]; returns [P, C]."""
    h, w, _ = fmap.shape
    res = F32(image_resolution)
    x = (((xp + F32(0.5)).astype(F32) * F32(w)).astype(F32) / res).astype(F32) - F32(0.5)
    y = (((yp + F32(0.5)).astype(F32) * F32(h)).astype(F32) / res).astype(F32) - F32(0.5)
    x = _clamp_ref(x.astype(F32), w - 1)
    y = _clamp_ref(y.astype(F32), h - 1)
    x0 = np.floor(x).astype(np.int64)
    y0 = np.floor(y).astype(np.int64)
    x1 = np.minimum(x0 + 1, w - 1)
    y1 = np.minimum(y0 + 1, h - 1)
    wx = (x - x0.astype(F32)).astype(F32)[:, None]
    wy = (y - y0.astype(F32)).astype(F32)[:, None]
    fm = np.asarray(fmap, F32)
    tl, tr = fm[y0, x0], fm[y0, x1]
    bl, br = fm[y1, x0], fm[y1, x1]
    omx = (F32(1) - wx).astype(F32)
    omy = (F32(1) - wy).astype(F32)
    top = ((tl * omx).astype(F32) + (tr * wx).astype(F32)).astype(F32)
    bot = ((bl * omx).astype(F32) + (br * wx).astype(F32)).astype(F32)
    return ((top * omy).astype(F32) + (bot * wy).astype(F32)).astype(F32)


def project_features_at_coords(fmap, grid_resolution: int, image_resolution: int, cam: ProjCamera, coords):
    """project_grid_features_at_coords (src/projection.cpp:359-434): features
    [N, C] and valid [N] (uint8) for sparse (0, x, y, z) rows of a
    grid_resolution^3 grid.  Raises ValueError like the reference."""
    if grid_resolution <= 0:
        raise ValueError("grid_resolution must be positive")
    k = projection_constants(cam, image_resolution)
    c = np.asarray(coords, np.int32).reshape(-1, 4)
    bad = (c[:, 0] != 0) | (c[:, 1:] < 0).any(1) | (c[:, 1:] >= grid_resolution).any(1)
    if bad.any():
        raise ValueError("sparse projection coordinate is outside the requested grid")
    xp, yp, valid = project_points(c[:, 1], c[:, 2], c[:, 3], grid_resolution, k, image_resolution)
    return bilinear_sample(np.asarray(fmap, F32), xp, yp, image_resolution), valid.astype(np.uint8)


def dense_grid_coords(r: int) -> np.ndarray:
    """All r^3 cells in torch.meshgrid(indexing="ij") order as (0, x, y, z)."""
    i = np.arange(r ** 3, dtype=np.int64)
    return np.stack([np.zeros_like(i), i // (r * r), (i // r) % r, i % r], 1).astype(np.int32)


def project_features_average(fmaps, grid_resolution: int, image_resolution: int, cams, coords=None):
    """project_grid_features_average (src/projection.cpp:436-481) when coords
    is None (dense grid), else the per-view sum of the multi-view condition
    projection (src/condition.cpp:878-940): f32 sum over views in order, then
    * (1 / views); valid = any view's valid."""
    if len(fmaps) == 0:
        raise ValueError("at least one projection view is required")
    if coords is None:
        coords = dense_grid_coords(grid_resolution)
    acc, val = None, None
    for fm, cam in zip(fmaps, cams):
        f, v = project_features_at_coords(fm, grid_resolution, image_resolution, cam, coords)
        acc = f if acc is None else (acc + f).astype(F32)
        val = v if val is None else (val | v)
    if len(fmaps) > 1:
        acc = (acc * F32(F32(1.0) / F32(len(fmaps)))).astype(F32)
    return acc, val


def relative_calc_matrices(c2w, distances):
    """compute_relative_calc_matrices (src/projection.cpp:528-561):
    relative[i] = F(distance[0]) * inverse(c2w[0]) * c2w[i]."""
    if len(c2w) == 0:
        raise ValueError("at least one camera transform is required")
    if len(c2w) != len(distances):
        raise ValueError("camera transform and distance counts must match")
    d0 = F32(distances[0])
    if not (d0 > 0) or not np.isfinite(d0):
        raise ValueError("main-view distance must be finite and positive")
    inv = invert4(c2w[0])
    if inv is None:
        raise ValueError("main-view camera transform matrix is singular")
    f = front_matrix(d0)
    return [matmul4(f, matmul4(inv, m)) for m in c2w]


# --------------------------------------------------------------------------
# SLat cascade glue (src/pipeline.cpp)
# --------------------------------------------------------------------------

def check_normalization(mean, std, channels):
    """valid_normalization (src/pipeline.cpp:268-285)."""
    mean, std = np.asarray(mean, F32), np.asarray(std, F32)
    if channels <= 0 or mean.shape != (channels,) or std.shape != (channels,):
        raise ValueError("SLat normalization channel count does not match model output")
    if not (np.isfinite(mean).all() and np.isfinite(std).all()) or (std == 0).any():
        raise ValueError("SLat normalization contains a non-finite or zero standard deviation")


def normalize_slat(x, mean, std):
    """normalize_slat_f32 (src/pipeline.cpp:333-358): (x - mean) / std in f32."""
    x = np.asarray(x, F32)
    check_normalization(mean, std, x.shape[1])
    with np.errstate(all="ignore"):
        y = ((x - np.asarray(mean, F32)).astype(F32) / np.asarray(std, F32)).astype(F32)
    if not np.isfinite(y).all():
        raise ValueError("SLat normalization produced a non-finite value")
    return y


def denormalize_slat(x, mean, std):
    """The latent denormalization of run_slat_stage_f32
    (src/pipeline.cpp:418-431): x * std + mean in f32 (two roundings)."""
    x = np.asarray(x, F32)
    check_normalization(mean, std, x.shape[1])
    with np.errstate(all="ignore"):
        y = ((x * np.asarray(std, F32)).astype(F32) + np.asarray(mean, F32)).astype(F32)
    if not np.isfinite(y).all():
        raise ValueError("SLat stage denormalization produced a non-finite value")
    return y


def quantize_slat_coords(coords, low_resolution, requested_resolution=1024, max_num_tokens=0):
    """quantize_slat_coords_f32 + quantize_at_resolution (src/pipeline.cpp:
    296-329, 437-468): each axis v -> llround((v + 0.5) / low * 63) in double
    (halves away from zero) on the 64^3 grid of resolution 1024, rows unique
    in lexicographic (b, x, y, z) order."""
    if requested_resolution != 1024:
        raise ValueError("SLat cascade resolution must be 1024")
    if low_resolution <= 0:
        raise ValueError("SLat cascade low resolution must be positive")
    c = np.asarray(coords, np.int64).reshape(-1, 4)
    grid = 1024 // 16
    mapped = (c[:, 1:].astype(np.float64) + 0.5) / float(low_resolution) * float(grid - 1)
    q = np.where(mapped >= 0, np.floor(mapped + 0.5), np.ceil(mapped - 0.5)).astype(np.int64)
    if ((q < 0) | (q >= grid)).any():
        raise ValueError("SLat decoder coordinate is outside cascade quantization range")
    rows = np.unique(np.concatenate([c[:, :1], q], 1), axis=0)
    if max_num_tokens and rows.shape[0] > max_num_tokens:
        raise ValueError("quantized SLat coordinate count exceeds max_num_tokens at resolution 1024")
    return rows.astype(np.int32)
