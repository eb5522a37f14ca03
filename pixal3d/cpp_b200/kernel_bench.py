"""Micro-benchmarks of single kernels of the SLat path (device time: CUDA
events around a CUDA-graph replay of --reps calls).

    python -m pixal3d.cpp_b200.kernel_bench --kernel conv1024 [--reps 10]

Kernels (config-2 shapes unless noted):
  conv1024   gather-GEMM sparse conv 1024->1024 on the 64^3 shell, batch 2
  conv1024t  the same with rows in neighbour-pattern order and tile tap skipping
  conv64     config-0 conv 64->64 on the shell (21,766 voxels)
  qkv        trunk qkv linear, 8,184 x 1024 -> 3072
  mlp0       trunk MLP up-projection with GELU, 8,184 x 1024 -> 4096
  qkvn       qkv linear with the fused q/k head RMS norm + RoPE epilogue
  out        attention output projection into the f32 residual, gated
  mlp2       MLP down-projection (K = 4096) into the f32 residual, gated
  proj       fine-level input projection, 43,532 x 64 -> 1024, f32 out
  gn         GroupNorm(32) + SiLU, 43,532 x 1024 f32 -> f16 (stats + apply)
  ln         trunk LayerNorm + AdaLN modulation, 8,184 x 1024 f32 -> f16
  attn       trunk self-attention, 2 sequences x 4,092, 16 heads x 64
  cross      trunk cross-attention, 2 x 4,092 queries x 1,029 keys
Each run is small enough for an ncu capture (a few hundred MB on the
device) while its inputs exceed the 126 MB L2.  Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import ops
from . import _lib as L
from .workloads import shell_coords, batched

C = 1024


def _time(fn, reps):
    """Device time per call: `reps` calls captured in one CUDA graph and
    replayed between two events (no host launch cost in the interval);
    eager launches when the call cannot be captured."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
    except RuntimeError:
        graph = None
        torch.cuda.synchronize()
    e0.record()
    if graph is not None:
        graph.replay()
    else:
        for _ in range(reps):
            fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def run(kernel: str, reps: int) -> dict:
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    h = torch.float16
    if kernel in ("conv1024", "conv1024t", "conv64"):
        cc = shell_coords()
        ch = 64 if kernel == "conv64" else 1024
        coords = torch.from_numpy(batched(cc, 2) if ch == 1024 else cc).to(dev)
        n = coords.shape[0]
        nbr = ops.neighbor_map27(coords)
        taps = None
        if kernel == "conv1024t":
            # as the flow's fine level runs: rows in neighbour-pattern order, tile taps
            order = ops.conv_row_order(coords, nbr, 2).long()
            nbr = ops.neighbor_map27(coords[order].contiguous())
            taps = ops.conv_tile_taps(nbr)
        pairs = int((nbr < n).sum().item())
        x = torch.randn((n, ch), device=dev, generator=g).to(h)
        w = (torch.randn((27, ch, ch), device=dev, generator=g) / math.sqrt(27 * ch)).to(h)
        b = torch.zeros(ch, device=dev)
        out = torch.empty((n, ch), device=dev)
        ms = _time(lambda: ops.subm_conv3d(x, nbr, w, b, out=out, tile_taps=taps), reps)
        flops = 2.0 * pairs * ch * ch
        bytes_ = n * ch * 2 + 27 * ch * ch * 2 + 27 * n * 4 + n * ch * 4
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "gbs": bytes_ / ms / 1e6,
                "flops": flops, "bytes": bytes_, "rows": n, "pairs": pairs}
    if kernel in ("qkv", "mlp0"):
        m = 2 * 4092
        nout = 3 * C if kernel == "qkv" else 4 * C
        x = torch.randn((m, C), device=dev, generator=g).to(h)
        w = (torch.randn((nout, C), device=dev, generator=g) / 32).to(h)
        b = torch.zeros(nout, device=dev)
        out = torch.empty((m, nout), device=dev, dtype=h)
        epi = L.EPI_GELU_TANH if kernel == "mlp0" else L.EPI_NONE
        ms = _time(lambda: ops.linear(x, w, b, out=out, epilogue=epi), reps)
        flops = 2.0 * m * C * nout
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "flops": flops, "m": m, "n": nout, "k": C}
    if kernel in ("out", "mlp2", "proj"):
        # gated residual linears of the trunk (f32 residual stream), and the
        # fine-level input projection (f32 output, K = 64)
        m = 2 * 4092 if kernel != "proj" else 2 * 21766
        k = {"out": C, "mlp2": 4 * C, "proj": 64}[kernel]
        x = torch.randn((m, k), device=dev, generator=g).to(h)
        w = (torch.randn((C, k), device=dev, generator=g) / math.sqrt(k)).to(h)
        b = torch.zeros(C, device=dev)
        out = torch.zeros((m, C), device=dev)
        if kernel == "proj":
            ms = _time(lambda: ops.linear(x, w, b, out=out), reps)
        else:
            gate = torch.randn((2, C), device=dev, generator=g)
            offs = torch.tensor([0, m // 2, m], dtype=torch.int32, device=dev)
            ms = _time(lambda: ops.linear(x, w, b, out=out, epilogue=L.EPI_RESIDUAL, gate=gate,
                                          batch_offsets=offs), reps)
        flops = 2.0 * m * C * k
        bytes_ = m * k * 2 + C * k * 2 + m * C * 4 * (1 if kernel == "proj" else 2)
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "gbs": bytes_ / ms / 1e6, "flops": flops,
                "m": m, "n": C, "k": k}
    if kernel == "gn":
        # io-resblock GroupNorm(32) + SiLU on the fine level, f32 -> f16
        cc = batched(shell_coords(), 2)
        n = cc.shape[0]
        x = torch.randn((n, C), device=dev, generator=g)
        gam = torch.ones(C, device=dev)
        bet = torch.zeros(C, device=dev)
        offs = torch.tensor([0, n // 2, n], dtype=torch.int32, device=dev)
        ms = _time(lambda: ops.group_norm_silu(x, 32, 1e-5, gam, bet, offs, True, h), reps)
        bytes_ = 2 * n * C * 4 + n * C * 2  # stats read + apply read + f16 write
        return {"kernel": kernel, "ms": ms, "gbs": bytes_ / ms / 1e6, "bytes": bytes_, "rows": n}
    if kernel == "qkvn":
        m = 2 * 4092
        coords = torch.from_numpy(batched(shell_coords(), 2)[:m]).to(dev)
        x = torch.randn((m, C), device=dev, generator=g).to(h)
        w = (torch.randn((3 * C, C), device=dev, generator=g) / 32).to(h)
        b = torch.zeros(3 * C, device=dev)
        gam = torch.ones(2 * C, device=dev)
        table = ops.rope_table(coords, 64)
        out = torch.empty((m, 3 * C), device=dev, dtype=h)
        ms = _time(lambda: ops.linear_headnorm(x, w, b, 2 * C, gam, 2 * C, table, out=out), reps)
        flops = 2.0 * m * C * 3 * C
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "flops": flops, "m": m, "n": 3 * C, "k": C}
    if kernel == "ln":
        m = 2 * 4092
        x = torch.randn((m, C), device=dev, generator=g)
        mod = torch.randn((2, 6 * C), device=dev, generator=g)
        offs = torch.tensor([0, 4092, m], dtype=torch.int32, device=dev)
        out = torch.empty((m, C), device=dev, dtype=h)
        ms = _time(lambda: ops.layernorm_modulate(x, 1e-6, mod=mod, batch_offsets=offs, out=out), reps)
        bytes_ = m * C * 4 + m * C * 2
        return {"kernel": kernel, "ms": ms, "gbs": bytes_ / ms / 1e6, "bytes": bytes_}
    if kernel in ("attn", "cross"):
        nq = 4092
        nk = nq if kernel == "attn" else 1029
        q = torch.randn((2 * nq, C), device=dev, generator=g).to(h)
        k = torch.randn((2 * nk, C), device=dev, generator=g).to(h)
        v = torch.randn((2 * nk, C), device=dev, generator=g).to(h)
        cq = torch.tensor([0, nq, 2 * nq], dtype=torch.int32, device=dev)
        ck = torch.tensor([0, nk, 2 * nk], dtype=torch.int32, device=dev)
        out = torch.empty((2 * nq, C), device=dev, dtype=h)
        ms = _time(lambda: ops.varlen_attention(q, k, v, cq, ck, nq, 16, 0.125, out=out), reps)
        flops = 2 * 4.0 * nq * nk * C
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "flops": flops}
    if kernel in ("project", "project3"):
        # projection conditioning: the 64^3 shell sampled from 37 x 37 x 1024
        # DINO-sized maps (1 or 3 views), f16 rows for the proj_linear GEMM
        nv = 1 if kernel == "project" else 3
        coords = torch.from_numpy(shell_coords()).to(dev)
        coords[:, 0] = 0
        n = coords.shape[0]
        maps = [torch.randn((37, 37, C), device=dev, generator=g) for _ in range(nv)]
        views = [{"feature_map": m, "image_resolution": 518, "camera_angle_x": 0.6, "distance": 2.0,
                  "mesh_scale": 1.0} for m in maps]
        out = torch.empty((n, C), device=dev, dtype=torch.float16)
        valid = torch.empty(n, device=dev, dtype=torch.uint8)
        ms = _time(lambda: ops.project_features(views, 64, coords, out=out, valid=valid), reps)
        write = n * C * 2 + n * 17
        corner = 4 * n * C * 4 * nv
        return {"kernel": kernel, "ms": ms, "points": n, "views": nv, "write_bytes": write, "corner_bytes": corner,
                "write_gbs": write / ms / 1e6, "corner_gbs": corner / ms / 1e6}
    raise SystemExit(f"unknown kernel {kernel}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True)
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args()
    print(json.dumps(run(a.kernel, a.reps)))


if __name__ == "__main__":
    main()
