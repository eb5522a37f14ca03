"""Device-resident SLat flow model and sampler (p3d_flow_* in include/p3d.h).

Mirrors the reference's SLatFlowModel (include/pixal3d/slat_flow.h:72-115):
`forward` is slat_flow_forward_f32 (src/slat_flow.cpp:161-249) and `sample`
is SLatFlowModel::sample + flow_euler_sample_f32 (src/slat_flow.cpp:1401-1447,
src/flow_sampler.cpp:245-343), with CFG batched as 2x images and the whole
loop on the device.  Weights are given as f32 CUDA tensors keyed by the
reference's field names (SLatFlowWeightsF32 / SparseTransformerBlockWeightsF32).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from .ops import ctx as _ctx

# reference field name -> p3d struct field
TOP_MAP = {"input_weight": "input_w", "input_bias": "input_b", "timestep_weight0": "t_w0", "timestep_bias0": "t_b0",
           "timestep_weight2": "t_w2", "timestep_bias2": "t_b2", "modulation_weight": "mod_w",
           "modulation_bias": "mod_b", "output_weight": "output_w", "output_bias": "output_b"}
BLOCK_MAP = {"modulation": "modulation", "self_to_qkv_weight": "qkv_w", "self_to_qkv_bias": "qkv_b",
             "self_q_gamma": "q_gamma", "self_k_gamma": "k_gamma", "self_to_out_weight": "out_w",
             "self_to_out_bias": "out_b", "norm2_weight": "norm2_w", "norm2_bias": "norm2_b",
             "cross_to_q_weight": "cq_w", "cross_to_q_bias": "cq_b", "cross_to_kv_weight": "ckv_w",
             "cross_to_kv_bias": "ckv_b", "cross_q_gamma": "cq_gamma", "cross_k_gamma": "ck_gamma",
             "cross_to_out_weight": "co_w", "cross_to_out_bias": "co_b", "proj_weight": "proj_w",
             "proj_bias": "proj_b", "mlp0_weight": "mlp0_w", "mlp0_bias": "mlp0_b", "mlp2_weight": "mlp2_w",
             "mlp2_bias": "mlp2_b"}


@dataclass
class HParams:
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
    operand_dtype: str = "f16"

    def to_c(self) -> L.FlowHParams:
        return L.FlowHParams(
            in_channels=self.in_channels, out_channels=self.out_channels, model_channels=self.model_channels,
            cond_channels=self.cond_channels, num_blocks=self.num_blocks, num_heads=self.num_heads,
            mlp_hidden=int(self.model_channels * self.mlp_ratio), proj_in_channels=self.proj_in_channels,
            proj_mode=int(self.image_attn_mode == "proj"), qk_rms_norm=int(self.qk_rms_norm),
            qk_rms_norm_cross=int(self.qk_rms_norm_cross), pe_mode=1 if self.pe_mode == "ape" else 0,
            io_resblocks=self.io_resblocks, groups=self.groups,
            operand_dtype=L.P3D_BF16 if self.operand_dtype == "bf16" else L.P3D_F16, norm_eps=self.norm_eps,
            rope_freq_min=self.rope_freq_min, rope_freq_base=self.rope_freq_base)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class FlowModel:
    """Weights resident on one device; prepare() binds a coordinate set."""

    def __init__(self, hp: HParams, weights: dict, device: int | None = None):
        self.hp = hp
        self.device = torch.cuda.current_device() if device is None else int(device)
        device = self.device
        self._keep = []
        dev = torch.device("cuda", device)

        def t(a):
            if a is None:
                return None
            if not isinstance(a, torch.Tensor):
                a = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            a = a.to(dev, torch.float32).contiguous()
            self._keep.append(a)
            return a

        fw = L.FlowWeights()
        for ref_name, c_name in TOP_MAP.items():
            setattr(fw, c_name, _ptr(t(weights[ref_name])))
        blocks = (L.BlockWeights * hp.num_blocks)()
        for i, bw in enumerate(weights["blocks"]):
            for ref_name, c_name in BLOCK_MAP.items():
                setattr(blocks[i], c_name, _ptr(t(bw.get(ref_name))))
        fw.blocks = C.cast(blocks, C.POINTER(L.BlockWeights))
        io_arrays = []
        for side in ("io_in", "io_out"):
            if hp.io_resblocks:
                arr = (L.ResBlockWeights * hp.io_resblocks)()
                for i, rw in enumerate(weights[side]):
                    for f in L.RESBLOCK_WEIGHT_FIELDS:
                        setattr(arr[i], f, _ptr(t(rw[f])))
                setattr(fw, side, C.cast(arr, C.POINTER(L.ResBlockWeights)))
                io_arrays.append(arr)
        self.ctx = _ctx(device)
        h = C.c_void_p()
        hpc = hp.to_c()
        self.ctx.check(L.OPTIONAL["p3d_flow_create"](self.ctx.h, C.byref(hpc), C.byref(fw), C.byref(h)))
        self.h = h
        self._keep = []  # device copies now live inside the flow object
        self.prepared = False

    def prepare(self, coords: torch.Tensor, batch: int, shape, ctx_offsets) -> None:
        offs = (C.c_int64 * (batch + 1))(*[int(v) for v in ctx_offsets])
        self.coords = coords
        self.batch = batch
        self.n = coords.shape[0]
        self.ctx = _ctx(self.device)
        self.ctx.check(L.OPTIONAL["p3d_flow_prepare"](self.h, _ptr(coords), self.n, batch, *shape, offs))
        self.prepared = True

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, ctx_feats: torch.Tensor,
                proj: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        c = _ctx(self.device)
        if out is None:
            out = torch.empty((self.n, self.hp.out_channels), dtype=torch.float32, device=x.device)
        dt = {torch.bfloat16: L.P3D_BF16, torch.float16: L.P3D_F16}.get(ctx_feats.dtype, L.P3D_F32)
        c.check(L.OPTIONAL["p3d_flow_forward"](self.h, _ptr(x.contiguous()), _ptr(timesteps), _ptr(ctx_feats), dt,
                                               _ptr(proj), _ptr(out)))
        return out

    def sample(self, x: torch.Tensor, ctx_feats: torch.Tensor, steps: int, guidance_strength: float = 1.0,
               guidance_rescale: float = 0.0, sigma_min: float = 1e-5, rescale_t: float = 1.0,
               guidance_interval=(0.0, 1.0), proj: torch.Tensor | None = None, use_graph: bool = True,
               concat: torch.Tensor | None = None) -> torch.Tensor:
        """In-place Euler/CFG integration of x (f32 [n/2, out_channels], the
        conditional rows).  concat (f32 [n/2, in - out]): the fixed concat
        condition appended to the state in every forward."""
        c = _ctx(self.device)
        cfg = L.SamplerConfig(steps=steps, sigma_min=sigma_min, rescale_t=rescale_t,
                              guidance_strength=guidance_strength, guidance_rescale=guidance_rescale,
                              guidance_interval_min=guidance_interval[0], guidance_interval_max=guidance_interval[1],
                              use_graph=int(use_graph))
        dt = {torch.bfloat16: L.P3D_BF16, torch.float16: L.P3D_F16}.get(ctx_feats.dtype, L.P3D_F32)
        if concat is None:
            c.check(L.OPTIONAL["p3d_flow_sample"](self.h, _ptr(x), _ptr(ctx_feats), dt, _ptr(proj), C.byref(cfg)))
        else:
            concat = concat.contiguous()
            c.check(L.OPTIONAL["p3d_flow_sample_concat"](self.h, _ptr(x), _ptr(ctx_feats), dt, _ptr(proj),
                                                         _ptr(concat), concat.shape[1], C.byref(cfg)))
        return x

    @property
    def launches_per_step(self) -> int:
        return int(L.OPTIONAL["p3d_flow_launches_per_step"](self.h))

    def close(self) -> None:
        if getattr(self, "h", None):
            L.OPTIONAL["p3d_flow_destroy"](self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
