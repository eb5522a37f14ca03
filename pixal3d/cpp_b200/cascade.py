"""Device-resident SLat part of the Pixal3D cascade.

Mirrors the SLat stages of the reference's run_pixal3d_cascade_f32
(src/pipeline.cpp:731-820) with every tensor kept on the device between
stages:

  shape LR   sample at the sparse-structure coordinates, latent * std + mean
  hand-off   shape decoder upsample_coords (`upsample_times` C2S levels),
             then quantize_slat_coords_f32 to the 64^3 grid of resolution 1024
  shape HR   sample at the quantized coordinates, denormalize
  texture    concat condition = (shape HR latent - mean) / std, fresh noise
             of texture_in - shape_latent channels, sample, denormalize

Noise and conditions come from caller callbacks, as in the reference
(Pixal3DNoiseBuilderF32 / Pixal3DConditionBuilderF32 in
include/pixal3d/pipeline.h): noise(stage, coords, channels, grid) -> f32
[n, channels]; condition(stage, coords, grid) -> (tokens f32 [T, cond],
token offsets per image, projected rows f32 [n, proj_in] or None).  Stage
names: "shape_slat_low", "shape_slat_high", "texture_slat".

Each sampling run batches the conditional and the unconditional (zero
condition) copies of every image as 2 x images items, as the device sampler
(p3d_flow_sample) expects.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .decoder import Decoder
from .flow import FlowModel


@dataclass
class SamplerSettings:
    """FlowEulerSamplerConfig fields used by the device sampler."""
    steps: int = 25
    guidance_strength: float = 3.0
    guidance_rescale: float = 0.0
    sigma_min: float = 1e-5
    rescale_t: float = 3.0
    guidance_interval: tuple = (0.0, 1.0)


@dataclass
class Normalization:
    """SLatNormalizationF32: latent = normalized * std + mean (device f32)."""
    mean: torch.Tensor
    std: torch.Tensor


def _images(coords: torch.Tensor) -> int:
    return int(coords[:, 0].max().item()) + 1 if coords.shape[0] else 1


def sample_stage(model: FlowModel, coords: torch.Tensor, grid: int, noise: torch.Tensor, tokens: torch.Tensor,
                 token_offsets, sampler: SamplerSettings, norm: Normalization, proj: torch.Tensor | None = None,
                 concat: torch.Tensor | None = None) -> torch.Tensor:
    """run_slat_stage_f32 (src/pipeline.cpp:360-435) on the device: CFG/Euler
    sampling of `noise` at `coords` (batch-contiguous images), then the
    latent denormalization.  Returns the denormalized latent [n, out]."""
    images = _images(coords)
    both = torch.cat([coords, coords + torch.tensor([images, 0, 0, 0], dtype=coords.dtype, device=coords.device)])
    offs = [int(v) for v in token_offsets]
    offs2 = offs + [offs[-1] + v for v in offs[1:]]
    model.prepare(both.contiguous(), 2 * images, (grid, grid, grid), offs2)
    x = noise.clone().contiguous()
    model.sample(x, torch.cat([tokens, tokens]).contiguous(), steps=sampler.steps,
                 guidance_strength=sampler.guidance_strength, guidance_rescale=sampler.guidance_rescale,
                 sigma_min=sampler.sigma_min, rescale_t=sampler.rescale_t,
                 guidance_interval=sampler.guidance_interval, proj=proj, concat=concat)
    return ops.slat_normalize(x, norm.mean, norm.std, denormalize=True, out=x)


class SLatCascade:
    """The three SLat flows and the shape decoder, resident on one device."""

    def __init__(self, shape_low: FlowModel, shape_high: FlowModel, texture: FlowModel, shape_decoder: Decoder,
                 shape_norm: Normalization, texture_norm: Normalization, low_resolution: int = 64,
                 upsample_times: int = 4, max_num_tokens: int = 49152):
        self.shape_low, self.shape_high, self.texture = shape_low, shape_high, texture
        self.decoder = shape_decoder
        self.shape_norm, self.texture_norm = shape_norm, texture_norm
        self.low_resolution = low_resolution
        self.upsample_times = upsample_times
        self.max_num_tokens = max_num_tokens

    def run(self, structure_coords: torch.Tensor, noise_fn, condition_fn, shape_sampler: SamplerSettings,
            texture_sampler: SamplerSettings) -> dict:
        out = {}
        low_grid = self.low_resolution
        c = structure_coords.contiguous()
        # shape LR
        hp = self.shape_low.hp
        tokens, toffs, proj = condition_fn("shape_slat_low", c, low_grid)
        noise = noise_fn("shape_slat_low", c, hp.in_channels, low_grid)
        out["shape_slat_low"] = lat = sample_stage(self.shape_low, c, low_grid, noise, tokens, toffs, shape_sampler,
                                                   self.shape_norm, proj)
        # hand-off: decoder coordinate upsampling, quantization to the 1024 grid
        up, _, _ = self.decoder.run(c, lat, _images(c), (low_grid, low_grid, low_grid),
                                    stop_level=self.upsample_times)
        out["shape_upsampled_coords"] = up
        up_res = low_grid << self.upsample_times
        high = ops.quantize_slat_coords(up, _images(up), up_res, 1024)
        if self.max_num_tokens and high.shape[0] > self.max_num_tokens:
            raise ValueError("quantized SLat coordinate count exceeds max_num_tokens at resolution 1024")
        if high.shape[0] == 0:
            raise ValueError("shape decoder upsample produced no high-resolution coordinates")
        out["high_coords"] = high
        grid = 1024 // 16
        # shape HR
        hp = self.shape_high.hp
        tokens, toffs, proj = condition_fn("shape_slat_high", high, grid)
        noise = noise_fn("shape_slat_high", high, hp.in_channels, grid)
        out["shape_slat_high"] = shape = sample_stage(self.shape_high, high, grid, noise, tokens, toffs, shape_sampler,
                                                      self.shape_norm, proj)
        # texture: the normalized shape latent as concat condition
        hp = self.texture.hp
        fresh = hp.in_channels - shape.shape[1]
        if fresh <= 0:
            raise ValueError("texture flow input has no channels left for fresh noise")
        tokens, toffs, proj = condition_fn("texture_slat", high, grid)
        noise = noise_fn("texture_slat", high, fresh, grid)
        concat = ops.slat_normalize(shape, self.shape_norm.mean, self.shape_norm.std)
        out["texture_slat"] = sample_stage(self.texture, high, grid, noise, tokens, toffs, texture_sampler,
                                           self.texture_norm, proj, concat)
        ops.ctx(c.device).sync_check()
        return out


def seeded_noise(seed: int):
    """A noise builder: N(0, 1) rows from a per-stage torch generator."""
    def fn(stage, coords, channels, grid):
        g = torch.Generator(device=coords.device)
        g.manual_seed(seed * 1000 + ["shape_slat_low", "shape_slat_high", "texture_slat"].index(stage))
        return torch.randn((coords.shape[0], channels), device=coords.device, generator=g)
    return fn


__all__ = ["SLatCascade", "SamplerSettings", "Normalization", "sample_stage", "seeded_noise"]
