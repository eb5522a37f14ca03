"""Device-resident SLat decoder (p3d_decoder_* in include/p3d.h).

Mirrors the reference's slat_decoder_forward_f32 / SLatDecoderModel::decode
(src/slat_decoder.cpp:290-376) and slat_decoder_upsample_coords_f32
(:378-455).  Weights are given as f32 CUDA tensors keyed like the oracle's
decoder dicts: from_latent_w/b, output_w/b, blocks = list (level order) of
ConvNeXt blocks {norm_w, norm_b, conv_w [27, C, C], conv_b, mlp0_w, mlp0_b,
mlp2_w, mlp2_b} and channel-to-spatial blocks {norm1_w, norm1_b, conv1_w
[27, 8*O, C], conv1_b, conv2_w [27, O, O], conv2_b, subdiv_w [8, C], subdiv_b}.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .ops import ctx as _ctx

_CONVNEXT = {"norm_w": "norm_w", "norm_b": "norm_b", "conv_w": "conv1_w", "conv_b": "conv1_b", "mlp0_w": "mlp0_w",
             "mlp0_b": "mlp0_b", "mlp2_w": "mlp2_w", "mlp2_b": "mlp2_b"}
_C2S = {"norm1_w": "norm1_w", "norm1_b": "norm1_b", "conv1_w": "conv1_w", "conv1_b": "conv1_b", "conv2_w": "conv2_w",
        "conv2_b": "conv2_b", "subdiv_w": "subdiv_w", "subdiv_b": "subdiv_b"}


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


class Decoder:
    def __init__(self, model_channels, num_blocks, latent_channels: int, out_channels: int, weights: dict,
                 pred_subdiv: bool = True, norm_eps: float = 1e-6, device: int | None = None,
                 operand_dtype: str = "f16"):
        self.device = torch.cuda.current_device() if device is None else int(device)
        dev = torch.device("cuda", self.device)
        self.levels = len(model_channels)
        self.model_channels = list(model_channels)
        self.out_channels = out_channels
        self.pred_subdiv = pred_subdiv
        cfg = L.DecoderConfig(latent_channels=latent_channels, out_channels=out_channels, levels=self.levels,
                              pred_subdiv=int(pred_subdiv), norm_eps=norm_eps,
                              operand_dtype=L.P3D_BF16 if operand_dtype == "bf16" else L.P3D_F16)
        for i, (c, b) in enumerate(zip(model_channels, num_blocks)):
            cfg.model_channels[i] = c
            cfg.num_blocks[i] = b
        keep = []

        def t(v):
            x = torch.as_tensor(v, dtype=torch.float32).to(dev).contiguous()
            keep.append(x)
            return C.c_void_p(x.data_ptr())

        blocks = (L.DecoderBlock * len(weights["blocks"]))()
        bi = 0
        for level in range(self.levels):
            for k in range(num_blocks[level] + (1 if level + 1 < self.levels else 0)):
                src = weights["blocks"][bi]
                blk = blocks[bi]
                ch = model_channels[level]
                if k < num_blocks[level]:
                    blk.kind, blk.channels, blk.out_channels = 0, ch, ch
                    blk.mlp_hidden = int(src["mlp0_w"].shape[0])
                    for a, f in _CONVNEXT.items():
                        setattr(blk, f, t(src[a]))
                else:
                    blk.kind, blk.channels, blk.out_channels = 1, ch, model_channels[level + 1]
                    for a, f in _C2S.items():
                        if a in src and src[a] is not None:
                            setattr(blk, f, t(src[a]))
                bi += 1
        w = L.DecoderWeights(from_latent_w=t(weights["from_latent_w"]), from_latent_b=t(weights["from_latent_b"]),
                             output_w=t(weights["output_w"]), output_b=t(weights["output_b"]),
                             blocks=C.cast(blocks, C.POINTER(L.DecoderBlock)), num_blocks=len(weights["blocks"]))
        self.ctx = _ctx(self.device)
        h = C.c_void_p()
        self.ctx.check(L.lib.p3d_decoder_create(self.ctx.h, C.byref(cfg), C.byref(w), C.byref(h)))
        self.h = h
        del keep  # the decoder holds its own 16-bit copies

    def run(self, coords: torch.Tensor, latent: torch.Tensor, batch: int, spatial, guides=None,
            stop_level: int | None = None):
        """Decode; returns (coords, feats, predicted subdivisions per level)
        or, with stop_level, the hidden (coords, feats) at that level."""
        c = _ctx(self.device)
        stop = self.levels if stop_level is None else int(stop_level)
        gp = grows = None
        if guides is not None:
            gp = (C.c_void_p * (self.levels - 1))(*[C.c_void_p(g.data_ptr()) for g in guides])
            grows = (C.c_int64 * (self.levels - 1))(*[g.shape[0] for g in guides])
        coords = coords.contiguous()
        latent = latent.contiguous()
        c.check(L.lib.p3d_decoder_run(self.h, _ptr(coords), coords.shape[0], batch, *spatial, _ptr(latent), gp, grows,
                                      stop))
        last = min(stop, self.levels - 1)
        rows = int(L.lib.p3d_decoder_rows(self.h, last))
        out_coords = torch.empty((rows, 4), dtype=torch.int32, device=coords.device)
        c.check(L.lib.p3d_decoder_coords(self.h, last, _ptr(out_coords)))
        cols = self.out_channels if stop == self.levels else self.model_channels[stop]
        feats = torch.empty((rows, cols), dtype=torch.float32, device=coords.device)
        c.check(L.lib.p3d_decoder_output(self.h, _ptr(feats)))
        preds = []
        if self.pred_subdiv and stop == self.levels:
            for level in range(self.levels - 1):
                r = int(L.lib.p3d_decoder_rows(self.h, level))
                p = torch.empty((r, 8), dtype=torch.float32, device=coords.device)
                c.check(L.lib.p3d_decoder_subdivision(self.h, level, _ptr(p)))
                preds.append(p)
        return out_coords, feats, preds

    def close(self):
        if getattr(self, "h", None):
            L.lib.p3d_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
