"""Seeded synthetic workloads for the benchmark configurations.

The reference publishes no dataset for this path; the benchmark configs are
defined on synthetic sphere-shell voxel sets with N(0,1) features and
random-init weights.  These generators are shared by the tests, the smoke
check and bench.py so that every consumer sees identical bytes.
"""
from __future__ import annotations

import math

import numpy as np


def shell_coords(res: int = 64, radius: float = 24.0, half_width: float = 1.5,
                 center: float | None = None, batch: int = 0) -> np.ndarray:
    """Integer voxels (b,x,y,z) of a res^3 grid with | |p-c| - radius | <= half_width,
    sorted lexicographically.  res=64, radius=24, half_width=1.5 gives the
    config-0 shell (21,766 voxels)."""
    c = res / 2.0 if center is None else center
    g = np.arange(res, dtype=np.float64)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    d = np.sqrt((x - c) ** 2 + (y - c) ** 2 + (z - c) ** 2)
    m = np.abs(d - radius) <= half_width
    xyz = np.stack([x[m], y[m], z[m]], axis=1).astype(np.int32)
    b = np.full((xyz.shape[0], 1), batch, np.int32)
    return np.ascontiguousarray(np.concatenate([b, xyz], axis=1))


def batched(coords: np.ndarray, batch: int) -> np.ndarray:
    """Repeat one coordinate set for batch items 0..batch-1 (CFG pairs)."""
    parts = []
    for b in range(batch):
        c = coords.copy()
        c[:, 0] = b
        parts.append(c)
    return np.ascontiguousarray(np.concatenate(parts, axis=0))


def image_shells(num_images: int, seed: int = 0, res: int = 64):
    """Per-image ragged shells for the multi-image config: radius ~ U(12,30),
    half-width ~ U(1,2.5), seeded."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(num_images):
        r = float(rng.uniform(12.0, 30.0))
        hw = float(rng.uniform(1.0, 2.5))
        out.append(shell_coords(res, r, hw))
    return out


def normal(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (rng.standard_normal(shape) * std).astype(np.float32)


def xavier(rng: np.random.Generator, out_f: int, in_f: int) -> np.ndarray:
    bound = math.sqrt(6.0 / (in_f + out_f))
    return rng.uniform(-bound, bound, size=(out_f, in_f)).astype(np.float32)
