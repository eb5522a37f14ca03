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


def pack_cfg(images: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """Varlen CFG batch of several images for one sampler run: image i's
    coordinates become batch item i (conditional) and item I + i (its
    unconditional copy), rows contiguous per item.  Returns (coords [2 sum
    N_i, 4], offsets [I + 1] of the conditional rows of each image)."""
    parts = []
    for half in range(2):
        for i, c in enumerate(images):
            cc = np.array(c, np.int32, copy=True)
            cc[:, 0] = half * len(images) + i
            parts.append(cc)
    offs = np.zeros(len(images) + 1, np.int64)
    offs[1:] = np.cumsum([c.shape[0] for c in images])
    return np.ascontiguousarray(np.concatenate(parts)), offs


def split_packs(order: list[int], sizes: list[int], max_voxels: int) -> list[list[int]]:
    """Consecutive groups of `order` whose voxel total stays <= max_voxels
    (an image larger than the limit gets a group of its own)."""
    packs: list[list[int]] = []
    cur: list[int] = []
    tot = 0
    for i in order:
        if cur and tot + sizes[i] > max_voxels:
            packs.append(cur)
            cur, tot = [], 0
        cur.append(i)
        tot += sizes[i]
    if cur:
        packs.append(cur)
    return packs


# Cascade-scale SLat decoder (the reference's real shape decode grows
# 9,857 -> 46,537 -> 206,980 -> 909,164 -> 4,005,638 points over four 2x
# subdivisions).  Five levels of representative widths; the level-0 input is
# the r = 16, half-width 1.5 shell of the 64^3 grid (9,682 voxels), and the
# guided subdivision keeps each child with probability 0.565, which grows it
# to about 4M points.
CASCADE_CHANNELS = (512, 256, 128, 64, 32)
CASCADE_BLOCKS = (1, 1, 1, 1, 1)
CASCADE_LATENT, CASCADE_OUT = 32, 8
CASCADE_KEEP = 0.565


def cascade_input() -> np.ndarray:
    return shell_coords(64, 16.0, 1.5)


def cascade_guides(n0: int, levels: int, p_keep: float = CASCADE_KEEP, seed: int = 0) -> list[np.ndarray]:
    """Subdivision logits for a guided decode: level l gets [n_l, 8] values,
    +1 (child kept) with probability p_keep, else -1; n_{l+1} is the number of
    kept children, so the row counts follow from the masks alone."""
    rng = np.random.default_rng(seed)
    out = []
    n = n0
    for _ in range(levels - 1):
        keep = rng.random((n, 8)) < p_keep
        out.append(np.where(keep, 1.0, -1.0).astype(np.float32))
        n = int(keep.sum())
    return out


def random_decoder_weights(rng: np.random.Generator, chans, num_blocks, latent: int, out: int, mlp_ratio: int = 4):
    """Random-init SLat decoder weights in the level order the decoder takes
    (num_blocks[l] ConvNeXt blocks, then a channel-to-spatial block between
    levels): linears xavier-uniform, convs N(0, 1/sqrt(27 cin)), norms
    1 + N(0, .05), biases N(0, .05), subdivision bias N(0, .5)."""
    def xav(o, i):
        a = math.sqrt(6.0 / (o + i))
        return rng.uniform(-a, a, (o, i)).astype(np.float32)

    def conv(o, i):
        return (rng.standard_normal((27, o, i)) / math.sqrt(27 * i)).astype(np.float32)

    def vec(n, s=0.05, m=0.0):
        return (m + rng.standard_normal(n) * s).astype(np.float32)

    blocks = []
    for level, c in enumerate(chans):
        for _ in range(num_blocks[level]):
            blocks.append({"norm_w": vec(c, 0.05, 1.0), "norm_b": vec(c), "conv_w": conv(c, c), "conv_b": vec(c),
                           "mlp0_w": xav(mlp_ratio * c, c), "mlp0_b": vec(mlp_ratio * c),
                           "mlp2_w": xav(c, mlp_ratio * c), "mlp2_b": vec(c)})
        if level + 1 < len(chans):
            o = chans[level + 1]
            blocks.append({"norm1_w": vec(c, 0.05, 1.0), "norm1_b": vec(c), "conv1_w": conv(8 * o, c),
                           "conv1_b": vec(8 * o), "conv2_w": conv(o, o), "conv2_b": vec(o),
                           "subdiv_w": xav(8, c), "subdiv_b": vec(8, 0.5)})
    return {"from_latent_w": xav(chans[0], latent), "from_latent_b": vec(chans[0]), "output_w": xav(out, chans[-1]),
            "output_b": vec(out), "blocks": blocks}


def random_swin_weights(rng: np.random.Generator, c0: int = 128, stages=(64, 32), latent: int = 8, out: int = 16,
                        blocks: int = 2, mlp_ratio: int = 4) -> dict:
    """Random-init weights of the config-3 shifted-window decoder (keys as
    SwinDecoder takes them): linears xavier-uniform, convs N(0, 1/sqrt(27
    cin)), norms 1 + N(0, .05), biases N(0, .05)."""
    def xav(o, i):
        a = math.sqrt(6.0 / (o + i))
        return rng.uniform(-a, a, (o, i)).astype(np.float32)

    def vec(n, s=0.05, m=0.0):
        return (m + rng.standard_normal(n) * s).astype(np.float32)

    def conv(o, i):
        return (rng.standard_normal((27, o, i)) / math.sqrt(27 * i)).astype(np.float32)

    w = {"from_latent_w": xav(c0, latent), "from_latent_b": vec(c0), "blocks": [], "stages": []}
    for _ in range(blocks):
        w["blocks"].append({"norm1_w": vec(c0, 0.05, 1.0), "norm1_b": vec(c0), "qkv_w": xav(3 * c0, c0),
                            "qkv_b": vec(3 * c0), "out_w": xav(c0, c0), "out_b": vec(c0),
                            "norm2_w": vec(c0, 0.05, 1.0), "norm2_b": vec(c0), "mlp0_w": xav(mlp_ratio * c0, c0),
                            "mlp0_b": vec(mlp_ratio * c0), "mlp2_w": xav(c0, mlp_ratio * c0), "mlp2_b": vec(c0)})
    ci = c0
    for co in stages:
        w["stages"].append({"gn1_w": vec(ci, 0.05, 1.0), "gn1_b": vec(ci), "conv1_w": conv(co, ci), "conv1_b": vec(co),
                            "gn2_w": vec(co, 0.05, 1.0), "gn2_b": vec(co), "conv2_w": conv(co, co),
                            "conv2_b": vec(co), "skip_w": xav(co, ci), "skip_b": vec(co)})
        ci = co
    w["output_w"] = xav(out, ci)
    w["output_b"] = vec(out)
    return w
