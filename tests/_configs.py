"""Seeded inputs of the BASELINE configurations at their full sizes, shared
by the golden generator (tests/golden/make_golden.py --only configs, which
runs the numpy oracle on the CPU) and the GPU parity tests that compare the
CUDA path with those goldens.

Every array comes from numpy's PCG64 generator with a fixed seed, so the
generator and the tests see identical bytes; each golden file also stores a
fingerprint of its inputs, checked before any comparison.

- config 1: one sparse transformer block on the 21,766-voxel shell, C=1024,
  16 heads x 64, qk RMS norm, sinusoidal absolute 3D PE, cross-attention to
  1,029 condition tokens, MLP x4 GELU-tanh, AdaLN from the timestep
  embedding at t = 0.5 (model time 500, as the sampler scales t by 1000).
  The block's input tokens are the N(0,1) features themselves: the model's
  input linear is the identity.  The model's final LayerNorm and a random
  1024 -> 8 output linear follow the block.
- config 2: one full SLat-flow forward as the benchmark runs it: CFG batch 2
  (the conditional image and its zeros-condition copy, same latent), input
  linear 8 -> 1024, two SparseResBlock3d at 64^3, 2x downsample, 24 blocks
  with 3D RoPE, 2x upsample, two SparseResBlock3d, output linear to 8.
- conv: the config-2 fine-level sparse conv C=1024 -> 1024 over the batch-2
  shell (43,532 rows), rows of each batch item stably sorted by neighbour
  pattern and tile taps skipped, as the flow runs it.
"""
from __future__ import annotations

import math

import numpy as np

from oracle import oracle as O
from pixal3d.cpp_b200.workloads import batched, shell_coords
from tests._models import random_flow_weights

C, HEADS, CTX = 1024, 16, 1029
RES = 64


def fingerprint(*arrays) -> np.ndarray:
    """Sum, sum of squares and a strided sample of each array (float64)."""
    out = []
    for a in arrays:
        f = np.asarray(a, np.float64).ravel()
        out += [f.sum(), (f * f).sum(), f[:: max(1, f.size // 97)][:97].sum()]
    return np.array(out, np.float64)


def weights_fingerprint(w: dict) -> np.ndarray:
    parts = [w[k] for k in sorted(k for k in w if isinstance(w[k], np.ndarray))]
    for bw in w["blocks"]:
        parts += [bw[k] for k in sorted(bw) if bw[k] is not None]
    for side in ("io_in", "io_out"):
        for rw in w.get(side, []):
            parts += [rw[k] for k in sorted(rw)]
    return fingerprint(np.concatenate([p.ravel()[:: max(1, p.size // 4096)] for p in parts]))


def cfg1():
    """Config-1 block: (coords, x, ts, ctx_offsets, ctx, hp, w)."""
    coords = shell_coords()
    n = coords.shape[0]
    hp = O.FlowHParams(in_channels=C, out_channels=8, model_channels=C, cond_channels=C, num_blocks=1,
                       num_heads=HEADS, mlp_ratio=4.0, pe_mode="ape")
    w = random_flow_weights(np.random.default_rng(101), hp)
    w["input_weight"] = np.eye(C, dtype=np.float32)
    w["input_bias"] = np.zeros(C, np.float32)
    rng = np.random.default_rng(102)
    x = rng.standard_normal((n, C)).astype(np.float32)
    ctx = rng.standard_normal((CTX, C)).astype(np.float32)
    ts = np.array([500.0], np.float32)
    offs = np.array([0, CTX], np.int64)
    return coords, x, ts, offs, ctx, hp, w


def cfg2():
    """Config-2 forward, CFG batch 2: (coords, x, ts, ctx_offsets, ctx, hp, w)."""
    img = shell_coords()
    coords = batched(img, 2)
    n = img.shape[0]
    hp = O.FlowHParams(in_channels=8, out_channels=8, model_channels=C, cond_channels=C, num_blocks=24,
                       num_heads=HEADS, mlp_ratio=4.0, io_resblocks=2, groups=32)
    w = random_flow_weights(np.random.default_rng(201), hp)
    rng = np.random.default_rng(202)
    xh = rng.standard_normal((n, 8)).astype(np.float32)
    x = np.ascontiguousarray(np.concatenate([xh, xh]))
    cond = rng.standard_normal((CTX, C)).astype(np.float32)
    ctx = np.ascontiguousarray(np.concatenate([cond, np.zeros_like(cond)]))
    ts = np.array([500.0, 500.0], np.float32)
    offs = np.array([0, CTX, 2 * CTX], np.int64)
    return coords, x, ts, offs, ctx, hp, w


CONV_ORDER_CHUNK_ROWS = 4096  # P3D_CONV_ORDER_CHUNK_ROWS (include/p3d.h)


def pattern_order(coords: np.ndarray, nbr: np.ndarray, chunk_rows: int = CONV_ORDER_CHUNK_ROWS) -> np.ndarray:
    """Row order of the flow's fine level: stable sort by (batch, row //
    chunk_rows, neighbour pattern), the pattern's bit t set when the row has a
    neighbour at tap t (chunk_rows <= 0: one chunk)."""
    n = coords.shape[0]
    pattern = ((nbr < n).astype(np.int64) << np.arange(27, dtype=np.int64)[:, None]).sum(0)
    chunk = np.arange(n, dtype=np.int64) // chunk_rows if chunk_rows > 0 else np.zeros(n, np.int64)
    key = (coords[:, 0].astype(np.int64) << 50) | (chunk << 27) | pattern
    return np.argsort(key, kind="stable")


def conv1024():
    """Fine-level conv of config 2 in the flow's row order:
    (coords_sorted, nbr_sorted, x16 f32 values of f16 operands [n][C],
    w16 f32 values of f16 weights [27][C][C], bias)."""
    coords = batched(shell_coords(), 2)
    order = pattern_order(coords, O.neighbor_map27(coords))
    cs = np.ascontiguousarray(coords[order])
    nbr = O.neighbor_map27(cs)
    rng = np.random.default_rng(301)
    x = rng.standard_normal((cs.shape[0], C)).astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((27, C, C)) / math.sqrt(27 * C)).astype(np.float16).astype(np.float32)
    b = (rng.standard_normal(C) * 0.02).astype(np.float32)
    return cs, nbr, x, w, b


def conv_rows(nbr: np.ndarray, x: np.ndarray, w: np.ndarray, b: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """The oracle conv (sparse_submanifold_conv3d, src/sparse.cpp:999-1055)
    restricted to the given output rows: f32 out[rows]."""
    n = x.shape[0]
    xz = np.concatenate([x, np.zeros((1, x.shape[1]), np.float32)])
    out = np.zeros((rows.size, w.shape[1]), np.float32)
    for k in range(27):
        out += xz[nbr[k, rows]] @ w[k].T
    return out + b


def sample_rows(n: int, count: int, seed: int) -> np.ndarray:
    """Sorted distinct rows, with the first and last rows included."""
    r = np.random.default_rng(seed).choice(n, size=count - 2, replace=False)
    return np.unique(np.concatenate([r, [0, n - 1]]))
