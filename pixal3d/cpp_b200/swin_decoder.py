"""Config-3 SLat decoder on the device (no reference implementation; the
benchmark configuration's shifted-window decoder, restated in
oracle.swin_decoder_forward).

    latent [N, 8] -> linear to C0 (+ sinusoidal absolute 3D PE)
    -> num_blocks pre-norm blocks: x += Wo . window_attention(LN1(x)),
       x += W2 . gelu_tanh(W1 . LN2(x)); windows of window^3 voxels, shifted
       by window/2 on odd blocks
    -> per stage: subdivide x2 with a keep mask (children copy the parent
       row), SparseResBlock3d with a channel change:
       conv2(SiLU(GN(conv1(SiLU(GN(x)))))) + skip(x)
    -> LayerNorm (eps 1e-5, no affine) -> linear to out_channels.

Every step is a C-ABI kernel of libp3dcuda.so (tcgen05 GEMMs and gather
convs, the windowed tcgen05 attention, the subdivision topology and the
fused elementwise kernels); torch only owns the device buffers.  Operands are
16-bit (f16 by default), accumulation and the residual stream f32.  Conv
inputs narrower than a multiple of 64 channels are zero-padded.

Weights (f32 arrays or tensors, keyed like the oracle): from_latent_w/b,
blocks[i] = {norm1_w/b, qkv_w [3C, C], qkv_b, out_w, out_b, norm2_w/b, mlp0_w
[rC, C], mlp0_b, mlp2_w [C, rC], mlp2_b}, stages[s] = {gn1_w/b, conv1_w
[27, Co, Ci], conv1_b, gn2_w/b, conv2_w [27, Co, Co], conv2_b, skip_w
[Co, Ci], skip_b}, output_w/b.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import ops


def _pad64(c: int) -> int:
    return (c + 63) // 64 * 64


class SwinDecoder:
    def __init__(self, cfg: dict, weights: dict, device: int | None = None, operand_dtype: str = "f16"):
        self.cfg = dict(cfg)
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else int(device))
        self.dt = torch.bfloat16 if operand_dtype == "bf16" else torch.float16
        self.c0 = int(cfg["model_channels"])
        self.heads = int(cfg["num_heads"])
        assert self.c0 == self.heads * 64, "head_dim 64"
        self.window = int(cfg["window"])
        self.groups = int(cfg.get("groups", 32))

        def f32(a):
            return torch.as_tensor(a, dtype=torch.float32).to(self.device).contiguous()

        def op(a):
            return f32(a).to(self.dt).contiguous()

        def conv(a, cin_pad):
            w = f32(a)  # [27, Co, Ci]
            if w.shape[2] < cin_pad:
                w = torch.nn.functional.pad(w, (0, cin_pad - w.shape[2]))
            return w.to(self.dt).contiguous()

        w = weights
        self.w_in, self.b_in = op(w["from_latent_w"]), f32(w["from_latent_b"])
        assert self.w_in.shape[1] % 8 == 0, "latent channels must be a multiple of 8"
        self.blocks = []
        for b in w["blocks"]:
            self.blocks.append({k: (op(v) if k.endswith("_w") and not k.startswith("norm") else f32(v))
                                for k, v in b.items()})
        self.stages = []
        for s in w["stages"]:
            co, ci = s["skip_w"].shape[0], s["skip_w"].shape[1]
            self.stages.append({
                "ci": ci, "co": co, "ci_pad": _pad64(ci), "co_pad": _pad64(co),
                "gn1_w": f32(s["gn1_w"]), "gn1_b": f32(s["gn1_b"]), "gn2_w": f32(s["gn2_w"]), "gn2_b": f32(s["gn2_b"]),
                "conv1_w": conv(s["conv1_w"], _pad64(ci)), "conv1_b": f32(s["conv1_b"]),
                "conv2_w": conv(s["conv2_w"], _pad64(co)), "conv2_b": f32(s["conv2_b"]),
                "skip_w": op(s["skip_w"]), "skip_b": f32(s["skip_b"])})
        self.w_out, self.b_out = op(w["output_w"]), f32(w["output_b"])

    def _gn_silu_operand(self, x: torch.Tensor, gamma, beta, offs, batch: int, width: int) -> torch.Tensor:
        """SiLU(GroupNorm(x)) as a 16-bit conv operand of `width` columns."""
        if width == x.shape[1]:
            return ops.group_norm_silu(x, self.groups, 1e-5, gamma, beta, offs, True, self.dt)
        y = ops.group_norm_silu(x, self.groups, 1e-5, gamma, beta, offs, True, torch.float32)
        return ops.pack_operand(y, width, self.dt)

    def run(self, coords: torch.Tensor, latent: torch.Tensor, masks, batch: int = 1):
        """coords int32 [N, 4] (batch-contiguous, grid cfg['spatial']^3),
        latent f32 [N, latent_channels], masks: per stage an f32 [rows, 8]
        keep mask (> 0 keeps the child).  Returns (coords, out f32)."""
        C, W = self.c0, self.window
        sp = (int(self.cfg["spatial"]),) * 3
        h = ops.linear(ops.convert(latent.contiguous(), self.dt), self.w_in, self.b_in, out_dtype=torch.float32)
        ops.ape_add_(h, coords)
        parts = [ops.window_partition(coords, batch, W, 0, sp), ops.window_partition(coords, batch, W, W // 2, sp)]
        for i, b in enumerate(self.blocks):
            a = ops.layernorm_modulate(h, 1e-6, gamma=b["norm1_w"], beta=b["norm1_b"], out_dtype=self.dt)
            qkv = ops.linear(a, b["qkv_w"], b["qkv_b"], out_dtype=self.dt)
            perm, cu = parts[i % 2]
            o = ops.window_attention(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], perm, cu, W, self.heads, 0.125)
            ops.linear(o, b["out_w"], b["out_b"], out=h, epilogue=L.EPI_RESIDUAL)
            a = ops.layernorm_modulate(h, 1e-6, gamma=b["norm2_w"], beta=b["norm2_b"], out_dtype=self.dt)
            m = ops.linear(a, b["mlp0_w"], b["mlp0_b"], out_dtype=self.dt, epilogue=L.EPI_GELU_TANH)
            ops.linear(m, b["mlp2_w"], b["mlp2_b"], out=h, epilogue=L.EPI_RESIDUAL)
        for s, st in enumerate(self.stages):
            mask = torch.as_tensor(masks[s], dtype=torch.float32).to(self.device).contiguous()
            oc, sr, _, mm = ops.c2s_topology(coords, 2, mask)
            hc = ops.c2s_gather(h, sr, torch.zeros(mm, dtype=torch.int8, device=self.device), st["ci"])
            coords = oc.contiguous()
            nbr = ops.neighbor_map27(coords)
            offs = ops.batch_offsets(coords, batch)
            g = self._gn_silu_operand(hc, st["gn1_w"], st["gn1_b"], offs, batch, st["ci_pad"])
            t = ops.subm_conv3d(g, nbr, st["conv1_w"], st["conv1_b"])
            g2 = self._gn_silu_operand(t, st["gn2_w"], st["gn2_b"], offs, batch, st["co_pad"])
            h = ops.linear(ops.convert(hc, self.dt), st["skip_w"], st["skip_b"], out_dtype=torch.float32)
            ops.subm_conv3d(g2, nbr, st["conv2_w"], st["conv2_b"], out=h, epilogue=L.EPI_RESIDUAL)
        a = ops.layernorm_modulate(h, 1e-5, out_dtype=self.dt)
        return coords, ops.linear(a, self.w_out, self.b_out, out_dtype=torch.float32)
