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
  nbr        coordinate hash build + 27-neighbour map, batch-2 shell (43,532)
  rowsort    conv row order (device radix sort by batch and neighbour pattern)
  down       2x downsample topology + mean of 1024 f32 channels (43,532 -> 8,184)
  c2s        channel-to-spatial topology + gather, 21,766 -> ~87k rows x 768
  window     8^3 window partition + windowed attention, 21,766 x 12 heads (config 3)
  dconv      config-3 stage-2 conv, ~347k rows, 64 (32 padded) -> 32 channels
  euler      Euler/CFG update with guidance rescale, 21,766 x 8
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


def run(kernel: str, reps: int, chunk: int | None = None) -> dict:
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
            # as the flow's fine level runs: rows in neighbour-pattern order
            # inside chunks of caller rows, tile taps
            order = ops.conv_row_order(coords, nbr, 2, *(() if chunk is None else (chunk,))).long()
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
    if kernel in ("nbr", "rowsort", "down"):
        coords = torch.from_numpy(batched(shell_coords(), 2)).to(dev)
        n = coords.shape[0]
        if kernel == "nbr":
            ms = _time(lambda: ops.neighbor_map27(coords), reps)
            bytes_ = n * 16 + 27 * n * 4
            return {"kernel": kernel, "ms": ms, "gbs": bytes_ / ms / 1e6, "bytes": bytes_, "rows": n}
        if kernel == "rowsort":
            nbr = ops.neighbor_map27(coords)
            ms = _time(lambda: ops.conv_row_order(coords, nbr, 2), reps)
            bytes_ = 27 * n * 4 + n * 16 + n * 4
            return {"kernel": kernel, "ms": ms, "gbs": bytes_ / ms / 1e6, "bytes": bytes_, "rows": n}
        x = torch.randn((n, C), device=dev, generator=g)
        _, _, child, m = ops.downsample_topology(coords, 2, (64, 64, 64), 2)
        t_topo = _time(lambda: ops.downsample_topology(coords, 2, (64, 64, 64), 2), reps)
        ms = _time(lambda: ops.downsample_mean(x, child, 2), reps)
        bytes_ = n * C * 4 + m * C * 4 + m * 8 * 4
        return {"kernel": kernel, "ms_mean": ms, "ms_topology": t_topo, "gbs_mean": bytes_ / ms / 1e6,
                "rows_in": n, "rows_out": m}
    if kernel == "c2s":
        cc = torch.from_numpy(shell_coords()).to(dev)
        n = cc.shape[0]
        mask = (torch.rand((n, 8), device=dev, generator=g) < 0.5).float()
        x = torch.randn((n, 8 * 96), device=dev, generator=g)
        oc, sr, sc, m = ops.c2s_topology(cc, 2, mask)
        t_topo = _time(lambda: ops.c2s_topology(cc, 2, mask), reps)
        zero = torch.zeros(m, dtype=torch.int8, device=dev)
        xs = torch.randn((n, 768), device=dev, generator=g)
        ms = _time(lambda: ops.c2s_gather(xs, sr, zero, 768), reps)
        bytes_ = 2 * m * 768 * 4
        return {"kernel": kernel, "ms_gather": ms, "ms_topology": t_topo, "gbs_gather": bytes_ / ms / 1e6,
                "rows_in": n, "rows_out": m}
    if kernel == "window":
        cc = torch.from_numpy(shell_coords()).to(dev)
        n, Cw, H = cc.shape[0], 768, 12
        qkv = torch.randn((n, 3 * Cw), device=dev, generator=g).to(h)
        perm, cu = ops.window_partition(cc, 1, 8, 4, (64, 64, 64))
        t_part = _time(lambda: ops.window_partition(cc, 1, 8, 4, (64, 64, 64)), reps)
        ms = _time(lambda: ops.window_attention(qkv[:, :Cw], qkv[:, Cw:2 * Cw], qkv[:, 2 * Cw:], perm, cu, 8, H, 0.125),
                   reps)
        key = (((cc[:, 1] + 4) // 8) * 64 + (cc[:, 2] + 4) // 8) * 64 + (cc[:, 3] + 4) // 8
        cnt = torch.bincount(key.long()).double()
        flops = 4.0 * float((cnt * cnt).sum()) * Cw
        return {"kernel": kernel, "ms_attention": ms, "ms_partition": t_part, "tflops": flops / ms / 1e9,
                "flops": flops, "rows": n}
    if kernel == "dconv":
        cc = shell_coords()
        # two masked subdivisions (keep 0.5) of the config-0 shell: ~347k rows at 256^3
        import numpy as np
        rng = np.random.default_rng(0)
        c = torch.from_numpy(cc).to(dev)
        for _ in range(2):
            m = torch.from_numpy((rng.random((c.shape[0], 8)) < 0.5).astype(np.float32)).to(dev)
            c, _, _, _ = ops.c2s_topology(c, 2, m)
            c = c.contiguous()
        n = c.shape[0]
        nbr = ops.neighbor_map27(c)
        pairs = int((nbr < n).sum().item())
        x = torch.randn((n, 64), device=dev, generator=g).to(h)
        w = (torch.randn((27, 32, 64), device=dev, generator=g) / math.sqrt(27 * 32)).to(h)
        b = torch.zeros(32, device=dev)
        out = torch.empty((n, 32), device=dev)
        ms = _time(lambda: ops.subm_conv3d(x, nbr, w, b, out=out), reps)
        flops = 2.0 * pairs * 64 * 32
        bytes_ = n * 64 * 2 + 27 * n * 4 + n * 32 * 4
        return {"kernel": kernel, "ms": ms, "tflops": flops / ms / 1e9, "gbs": bytes_ / ms / 1e6, "rows": n,
                "pairs": pairs}
    if kernel == "euler":
        n = 21766
        x = torch.randn((n, 8), device=dev, generator=g)
        vp = torch.randn((n, 8), device=dev, generator=g)
        vn = torch.randn((n, 8), device=dev, generator=g)
        offs = torch.tensor([0, n], dtype=torch.int32, device=dev)
        ms = _time(lambda: ops.euler_cfg_step(x, vp, vn, offs, 0.5, 0.46, 3.0, 0.7, 1e-5), reps)
        bytes_ = 4 * n * 8 * 4
        return {"kernel": kernel, "ms": ms, "gbs": bytes_ / ms / 1e6, "bytes": bytes_}
    raise SystemExit(f"unknown kernel {kernel}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--chunk", type=int, default=None,
                    help="conv1024t: chunk_rows of the row order (default: the flow's; 0: one chunk)")
    a = ap.parse_args()
    r = run(a.kernel, a.reps, a.chunk)
    if a.chunk is not None:
        r["chunk_rows"] = a.chunk
    print(json.dumps(r))


if __name__ == "__main__":
    main()
