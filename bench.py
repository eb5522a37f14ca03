#!/usr/bin/env python
"""Benchmark: SLat flow sampler steps/s at N=21,766 active voxels on B200.

Workload ("Full SLat-flow sampler"): the config-0
64^3 sphere shell (21,766 voxels), input linear 8->1024, two SparseResBlock3d
(3x3x3 sparse conv C=1024, GroupNorm32, SiLU) at 64^3, 2x downsample to 32^3
(4,092 voxels), 24 transformer blocks (16 heads x 64, MLP x4, qk RMS norm,
3D RoPE, AdaLN, cross-attention to 1029 x 1024 condition tokens), nearest 2x
upsample, two SparseResBlock3d, output linear to 8.  One step = one CFG-2
forward (conditional + zeros condition, batched) + the Euler/CFG update.
Weights random-init (seeded), condition tokens and noise N(0,1) (seeded).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --workload cfg4 [--gpus N] [--steps 25]

N > 1: launched by torchrun, one rank per GPU; every rank samples its own
image (weak scaling); NCCL broadcasts the condition tokens before timing and
gathers the results after it.  Rank 0 prints ONE JSON line.

--workload cfg4: 64 independent images with ragged
shells (radius ~ U(12, 30), half-width ~ U(1, 2.5); 4,256 to 55,719 voxels),
each with its own 1,029 x 1,024 condition, assigned to ranks by greedy LPT on
voxel count and packed per rank into varlen CFG batches; every image runs
the full config-2 sampler (--steps Euler steps, default 25).  Reports
images/s end to end (host inputs copied in, latents copied out), the
per-step latency and the measured load imbalance.
"""
from __future__ import annotations

import argparse
import re
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# ncu summary of the roofline kernel on this exact workload (one launch);
# its "traffic_bytes_per_launch = N" line is dram read + write bytes.
TRAFFIC_FILE = REPO / "profiles" / "gemm2_conv1024_fine_batch2.md"
METRIC = "SLat flow steps/s @N=20k voxels (CFG batch 2, 24 blocks, C=1024)"

# config-2 shapes
RES, RADIUS, HALF_WIDTH = 64, 24.0, 1.5
C, HEADS, BLOCKS, CTX_TOKENS, CH = 1024, 16, 24, 1029, 8


class _stdout_to_stderr:
    """Within the block, writes to file descriptor 1 (C and Python) land on
    stderr; C stdio buffers are flushed before descriptor 1 is restored."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        try:
            import ctypes
            ctypes.CDLL(None).fflush(None)
        except OSError:
            pass
        os.dup2(self.saved, 1)
        os.close(self.saved)
        return False


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", choices=["cfg2", "cfg1", "cfg3", "cascade", "cfg4"], default="cfg2")
    ap.add_argument("--steps", type=int, default=None, help="timed steps (cfg4: sampler steps per image)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--blocks", type=int, default=BLOCKS, help=argparse.SUPPRESS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


def load_peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- our arm

def make_weights(torch, dev, seed: int):
    """Random-init config-2 weights on the device (f32, seeded).
    Linears xavier-uniform; convs N(0, 1/sqrt(27 C)); biases N(0, .02);
    norms 1 + N(0, .05); block modulation N(0, .1)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def xav(o, i):
        b = math.sqrt(6.0 / (o + i))
        return torch.empty((o, i), device=dev).uniform_(-b, b, generator=g)

    def nrm(*shape, std=1.0, mean=0.0):
        return torch.randn(*shape, device=dev, generator=g) * std + mean

    mlp = 4 * C
    w = {"input_weight": xav(C, CH), "input_bias": nrm(C, std=0.02),
         "timestep_weight0": xav(C, 256), "timestep_bias0": nrm(C, std=0.02),
         "timestep_weight2": xav(C, C), "timestep_bias2": nrm(C, std=0.02),
         "modulation_weight": xav(6 * C, C), "modulation_bias": nrm(6 * C, std=0.02),
         "output_weight": xav(CH, C), "output_bias": nrm(CH, std=0.02), "blocks": []}
    for _ in range(BLOCKS_RUN):
        w["blocks"].append({
            "modulation": nrm(6 * C, std=0.1), "self_to_qkv_weight": xav(3 * C, C),
            "self_to_qkv_bias": nrm(3 * C, std=0.02), "self_q_gamma": nrm(C, std=0.05, mean=1.0),
            "self_k_gamma": nrm(C, std=0.05, mean=1.0), "self_to_out_weight": xav(C, C),
            "self_to_out_bias": nrm(C, std=0.02), "norm2_weight": nrm(C, std=0.05, mean=1.0),
            "norm2_bias": nrm(C, std=0.02), "cross_to_q_weight": xav(C, C), "cross_to_q_bias": nrm(C, std=0.02),
            "cross_to_kv_weight": xav(2 * C, C), "cross_to_kv_bias": nrm(2 * C, std=0.02),
            "cross_q_gamma": nrm(C, std=0.05, mean=1.0), "cross_k_gamma": nrm(C, std=0.05, mean=1.0),
            "cross_to_out_weight": xav(C, C), "cross_to_out_bias": nrm(C, std=0.02),
            "mlp0_weight": xav(mlp, C), "mlp0_bias": nrm(mlp, std=0.02),
            "mlp2_weight": xav(C, mlp), "mlp2_bias": nrm(C, std=0.02)})
    std = 1.0 / math.sqrt(27 * C)

    def res():
        return {"gn1_w": nrm(C, std=0.05, mean=1.0), "gn1_b": nrm(C, std=0.02), "conv1_w": nrm(27, C, C, std=std),
                "conv1_b": nrm(C, std=0.02), "gn2_w": nrm(C, std=0.05, mean=1.0), "gn2_b": nrm(C, std=0.02),
                "conv2_w": nrm(27, C, C, std=std), "conv2_b": nrm(C, std=0.02)}

    w["io_in"] = [res(), res()]
    w["io_out"] = [res(), res()]
    return w


BLOCKS_RUN = BLOCKS


def algorithmic_flops(n_img: int, n_trunk_img: int, pairs_img: int) -> dict:
    """Useful FLOPs of one CFG-2 step (2 x one image's forward)."""
    mlp = 4 * C
    lin_trunk = 2 * n_trunk_img * C * (3 * C + C + C + C + mlp + mlp)  # qkv, out, cross q, cross out, mlp0, mlp2
    kv = 2 * CTX_TOKENS * C * 2 * C
    attn_self = 4 * n_trunk_img * n_trunk_img * C
    attn_cross = 4 * n_trunk_img * CTX_TOKENS * C
    convs = 8 * 2 * pairs_img * C * C
    io_lin = 2 * n_img * (CH * C + C * CH)
    per_img = BLOCKS_RUN * (lin_trunk + kv + attn_self + attn_cross) + convs + io_lin
    return {"total": 2 * per_img, "conv": 2 * convs, "trunk_linear": 2 * BLOCKS_RUN * (lin_trunk + kv),
            "attention": 2 * BLOCKS_RUN * (attn_self + attn_cross)}


def time_conv_kernel(torch, ops, coords_dev, reps=10):
    """Average device time of the dominant kernel (gather-GEMM sparse conv,
    C=1024, the config-2 fine level, batch 2) measured with CUDA events on
    the launching stream, as the flow runs it: rows of each batch item in
    neighbour-pattern order, taps no row of a 256-row tile uses skipped."""
    n = coords_dev.shape[0]
    order = ops.conv_row_order(coords_dev, ops.neighbor_map27(coords_dev), 2).long()
    nbr = ops.neighbor_map27(coords_dev[order].contiguous())
    taps = ops.conv_tile_taps(nbr)
    pairs = int((nbr < n).sum().item())
    x = torch.randn((n, C), device="cuda").to(torch.float16)
    w = (torch.randn((27, C, C), device="cuda") / math.sqrt(27 * C)).to(torch.float16)
    b = torch.zeros(C, device="cuda")
    out = torch.empty((n, C), device="cuda")
    for _ in range(2):
        ops.subm_conv3d(x, nbr, w, b, out=out, tile_taps=taps)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(reps):
        ops.subm_conv3d(x, nbr, w, b, out=out, tile_taps=taps)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * pairs * C * C
    del x, w, out
    return ms, flops, pairs


def time_conv_cfg0(torch, ops, reps=50):
    """Config 0: one 64->64 submanifold conv on the 21,766-voxel shell.
    Algorithmic bytes = read x (N*64*2) + weights (27*64*64*2) + neighbour map
    (27*N*4) + write out f32 (N*64*4)."""
    from pixal3d.cpp_b200.workloads import shell_coords
    c = torch.from_numpy(shell_coords()).cuda()
    n = c.shape[0]
    nbr = ops.neighbor_map27(c)
    pairs = int((nbr < n).sum().item())
    x = torch.randn((n, 64), device="cuda").to(torch.float16)
    w = (torch.randn((27, 64, 64), device="cuda") / math.sqrt(27 * 64)).to(torch.float16)
    b = torch.zeros(64, device="cuda")
    out = torch.empty((n, 64), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    times = []
    for i in range(reps + 3):
        flush.zero_()  # evict L2 (> 126 MB) between launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.subm_conv3d(x, nbr, w, b, out=out)
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    # Back-to-back launches replayed from one CUDA graph (one ~11 MB conv is
    # dominated by launch and fill latency when timed alone).  The launches
    # rotate over 16 copies of (x, neighbour map, weights, out), 176 MB in
    # all, more than the 126 MB L2, so each launch reads its inputs from HBM.
    copies = 16
    sets = [(x.clone(), nbr.clone(), w.clone(), torch.empty_like(out)) for _ in range(copies)]
    graph_reps = 3 * copies
    for xs, ns, ws, os_ in sets:
        ops.subm_conv3d(xs, ns, ws, b, out=os_)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(graph_reps):
            xs, ns, ws, os_ = sets[i % copies]
            ops.subm_conv3d(xs, ns, ws, b, out=os_)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms_graph = e0.elapsed_time(e1) / graph_reps
    del g, sets
    bytes_ = n * 64 * 2 + 27 * 64 * 64 * 2 + 27 * n * 4 + n * 64 * 4
    return ms, bytes_, 2.0 * pairs * 64 * 64, ms_graph


def cpu_conv_cfg0(reps: int = 5):
    """The reference's sparse_submanifold_conv3d (oracle/_ref, compiled from
    the reference sources) on the config-0 shell, 64 -> 64, all host threads:
    median seconds of `reps` runs, and the thread count."""
    import numpy as np
    from oracle import reflib
    from pixal3d.cpp_b200.workloads import shell_coords
    threads = os.cpu_count() or 1
    reflib.set_threads(threads)
    c = shell_coords()
    rng = np.random.default_rng(0)
    x = rng.standard_normal((c.shape[0], 64)).astype(np.float32)
    w = (rng.standard_normal((27, 64, 64)) / math.sqrt(27 * 64)).astype(np.float32)
    b = np.zeros(64, np.float32)
    times = []
    for _ in range(reps + 1):
        t0 = time.perf_counter()
        reflib.subm_conv3d(c, x, w, b, 1, (RES, RES, RES))
        times.append(time.perf_counter() - t0)
    return statistics.median(times[1:]), threads


def cpu_baseline_sample(target_seconds: float = 20.0):
    """The reference's own CPU path (oracle/_ref, compiled from the reference
    sources) on this host's cores, on a bounded sample of the config-2 step:
      - sparse_transformer_cross_block_f32 at 256 voxels per item (batch 2,
        C=1024, 1029 condition tokens): its non-attention part scales
        linearly to the trunk size N=4,092;
      - the reference's (serial) sparse_scaled_dot_product_attention timed
        alone at 512 voxels per item, scaled by N^2 to N=4,092;
      - sparse_submanifold_conv3d 1024->1024 on a sub-slab of the shell,
        scaled by neighbour pairs to the full shell (8 convs x batch 2).
    Returns (extrapolated seconds per step, details)."""
    import numpy as np
    from oracle import reflib, oracle as O
    from pixal3d.cpp_b200.workloads import shell_coords, batched
    threads = os.cpu_count() or 1
    reflib.set_threads(threads)
    rng = np.random.default_rng(0)
    cfg = O.BlockConfig(channels=C, num_heads=HEADS, mlp_hidden=4 * C, context_channels=C)
    sc = 0.02
    w = {"modulation": rng.standard_normal(6 * C).astype(np.float32) * 0.1}
    for f, shp in [("self_to_qkv_weight", (3 * C, C)), ("self_to_out_weight", (C, C)), ("cross_to_q_weight", (C, C)),
                   ("cross_to_kv_weight", (2 * C, C)), ("cross_to_out_weight", (C, C)), ("mlp0_weight", (4 * C, C)),
                   ("mlp2_weight", (C, 4 * C))]:
        w[f] = (rng.standard_normal(shp) * sc).astype(np.float32)
        w[f.replace("weight", "bias")] = np.zeros(shp[0], np.float32)
    for f in ("self_q_gamma", "self_k_gamma", "norm2_weight", "cross_q_gamma", "cross_k_gamma"):
        w[f] = np.ones(C, np.float32)
    w["norm2_bias"] = np.zeros(C, np.float32)
    ctx = rng.standard_normal((2 * CTX_TOKENS, C)).astype(np.float32)
    offs = np.array([0, CTX_TOKENS, 2 * CTX_TOKENS], np.int64)
    tmod = (rng.standard_normal((2, 6 * C)) * 0.1).astype(np.float32)
    full = shell_coords()
    # block at ns voxels per item: its non-attention part scales with N
    ns, na = 256, 512
    cc = batched(full[:ns], 2)
    x = rng.standard_normal((cc.shape[0], C)).astype(np.float32)
    t0 = time.perf_counter()
    reflib.transformer_block(cc, x, tmod, offs, ctx, None, cfg, w, 2, (RES, RES, RES))
    t_b = time.perf_counter() - t0
    q = rng.standard_normal((cc.shape[0], C)).astype(np.float32)
    t0 = time.perf_counter()
    reflib.sdpa(cc, q, q, q, HEADS, C // HEADS, 0.125, 2, (RES, RES, RES))
    t_a = time.perf_counter() - t0
    # the reference's serial attention, timed alone at na voxels per item, scales with N^2
    ca = batched(full[:na], 2)
    qa = rng.standard_normal((ca.shape[0], C)).astype(np.float32)
    t0 = time.perf_counter()
    reflib.sdpa(ca, qa, qa, qa, HEADS, C // HEADS, 0.125, 2, (RES, RES, RES))
    t_a_big = time.perf_counter() - t0
    nt = 4092
    t_block = (t_b - t_a) * nt / ns + t_a_big * (nt / na) ** 2
    times = [t_b, t_a, t_a_big]
    # conv: a slab of the shell (x < 22) at C=1024, scaled by pairs
    slab = full[full[:, 1] < 14]
    xs = rng.standard_normal((slab.shape[0], C)).astype(np.float32)
    wc = (rng.standard_normal((27, C, C)) / math.sqrt(27 * C)).astype(np.float32)
    t0 = time.perf_counter()
    reflib.subm_conv3d(slab, xs, wc, np.zeros(C, np.float32), 1, (RES, RES, RES))
    t_slab = time.perf_counter() - t0
    pairs_slab = int((O.neighbor_map27(slab) < slab.shape[0]).sum())
    pairs_full = int((O.neighbor_map27(full) < full.shape[0]).sum())
    t_conv = t_slab * pairs_full / pairs_slab
    step = BLOCKS_RUN * t_block + 8 * 2 * t_conv
    return step, {"threads": threads, "block_at_256x2_s": round(t_b, 3), "sdpa_at_256x2_s": round(t_a, 3),
                  "sdpa_at_512x2_s": round(t_a_big, 3),
                  "t_block_N4092_s": round(t_block, 2), "t_conv_c1024_s": round(t_conv, 2),
                  "sample_seconds": round(sum(times) + t_slab, 1)}


def init_ranks(torch, dist):
    """(world, rank, local rank); one process per GPU, NCCL when world > 1."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        # NCCL prints its version line ("NCCL version ...") to the process's
        # stdout at communicator creation under NCCL_DEBUG=VERSION/WARN, where
        # NCCL_DEBUG_FILE is not used.  Point file descriptor 1 at stderr while
        # the communicator is created (eagerly here, plus a barrier), so rank
        # 0's stdout carries only the JSON result line.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        with _stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
    return world, rank, local


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    world, rank, local = init_ranks(torch, dist)
    from pixal3d.cpp_b200 import dist as D
    from pixal3d.cpp_b200 import ops
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    from pixal3d.cpp_b200.workloads import shell_coords, batched

    global BLOCKS_RUN
    BLOCKS_RUN = args.blocks
    dev = torch.device("cuda", local)
    peaks, peak_kind = load_peaks()
    img = shell_coords(RES, RADIUS, HALF_WIDTH)
    n_img = img.shape[0]
    coords = torch.from_numpy(batched(img, 2)).to(dev)

    # condition tokens: rank 0 draws them, NCCL broadcasts to every rank
    g = torch.Generator(device=dev)
    g.manual_seed(2024)
    cond = torch.randn((CTX_TOKENS, C), device=dev, generator=g)
    D.broadcast_(cond, src=0)
    ctx2 = torch.cat([cond, torch.zeros_like(cond)]).to(torch.float16)

    hp = HParams(in_channels=CH, out_channels=CH, model_channels=C, cond_channels=C, num_blocks=BLOCKS_RUN,
                 num_heads=HEADS, mlp_ratio=4.0, io_resblocks=2, groups=32, operand_dtype="f16")
    w = make_weights(torch, dev, seed=1234)
    model = FlowModel(hp, w, device=local)
    del w
    torch.cuda.empty_cache()
    model.prepare(coords, 2, (RES, RES, RES), [0, CTX_TOKENS, 2 * CTX_TOKENS])
    gn = torch.Generator(device=dev)
    gn.manual_seed(7 + rank)
    x = torch.randn((n_img, CH), device=dev, generator=gn)

    # warm-up (also captures the per-step CUDA graph)
    model.sample(x, ctx2, steps=max(args.warmup, 1), guidance_strength=3.0)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.ctx(local).launches
    e0.record(s)
    model.sample(x, ctx2, steps=args.steps, guidance_strength=3.0)
    e1.record(s)
    torch.cuda.synchronize()
    launches = ops.ctx(local).launches - launches0
    ms_local = e0.elapsed_time(e1)
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms_max = D.max_over_ranks(ms_local, dev)
    # NCCL gather of the sampled latents to rank 0 (outside the timed region)
    D.gather_rows(x, dst=0)

    value = world * args.steps / (ms_max / 1000.0)
    ms_per_step = ms_max / args.steps

    result = None
    if rank == 0:
        nbr_pairs = int((ops.neighbor_map27(torch.from_numpy(img).to(dev)) < n_img).sum().item())
        fl = algorithmic_flops(n_img, 4092, nbr_pairs)
        conv_ms, conv_flops, _ = time_conv_kernel(torch, ops, coords)
        conv_tflops = conv_flops / (conv_ms / 1000.0) / 1e12
        peak_t = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        traffic = None
        if TRAFFIC_FILE.exists():
            mt = re.search(r"traffic_bytes_per_launch\s*=\s*(\d+)", TRAFFIC_FILE.read_text())
            traffic = int(mt.group(1)) if mt else None
        c0_ms, c0_bytes, c0_flops, c0_graph_ms = time_conv_cfg0(torch, ops)
        hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 operands, f32 accumulate/residual",
            "data": "synthetic: seeded sphere shell, N(0,1) noise and condition tokens, random-init weights",
            "config": {"workload": "config2: full SLat-flow sampler step, CFG batch 2",
                       "voxels_per_image": n_img, "trunk_voxels_per_image": 4092, "model_channels": C,
                       "blocks": BLOCKS_RUN, "heads": HEADS, "condition_tokens": CTX_TOKENS,
                       "io_resblocks": 2, "images_per_gpu": 1, "parallelism": f"dp{world} (images)",
                       "l2": "per-step working set (1.26 GB of weights streamed per step) exceeds the 126 MB L2",
                       "cuda_graph": "one captured step replayed per step"},
            "step_tflop": round(fl["total"] / 1e12, 3),
            "achieved_tflops": round(fl["total"] / (ms_per_step / 1000.0) / 1e12, 1),
            "gpu_launches": int(launches),
            "clocks": clk,
            "roofline": {"kernel": "gather-GEMM sparse conv 1024->1024 (tcgen05), fine level batch 2",
                         "bound": "tensor", "achieved": round(conv_tflops, 1), "peak": peak_t,
                         "peak_kind": f"{peak_kind} bf16 burst (f16 dense rate is identical)",
                         "unit": "TFLOP/s", "frac": round(conv_tflops / peak_t, 4), "traffic": traffic,
                         "avg_launch_ms": round(conv_ms, 4), "flops_per_launch": conv_flops},
            "sparse_conv_cfg0": {"ms_graph": round(c0_graph_ms, 4), "algorithmic_bytes": c0_bytes,
                                 "achieved_gbs": round(c0_bytes / (c0_graph_ms / 1000.0) / 1e9, 1), "peak_gbs": hbm,
                                 "frac_hbm": round(c0_bytes / (c0_graph_ms / 1000.0) / 1e9 / hbm, 4),
                                 "tflops": round(c0_flops / (c0_graph_ms / 1000.0) / 1e12, 2),
                                 "timing": "ms_graph: 48 back-to-back launches replayed from one CUDA graph, "
                                           "rotating over 16 input/output copies (176 MB > L2, so inputs come "
                                           "from HBM); ms_single_flushed: one launch after a 256 MB L2-flush "
                                           "write, median of 50",
                                 "ms_single_flushed": round(c0_ms, 4),
                                 "frac_hbm_single_flushed": round(c0_bytes / (c0_ms / 1000.0) / 1e9 / hbm, 4)},
        }
    # e2e: the public sampler call with HOST buffers (pinned), copies inside
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(torch, model, img, cond, args, dev, world, rank)
    if rank == 0:
        result["e2e"] = e2e
        if world == 1 and not args.no_cpu_baseline:
            try:
                cs, thr = cpu_conv_cfg0()
                result["sparse_conv_cfg0"]["cpu_reference"] = {
                    "ms": round(cs * 1000.0, 2), "cores": thr, "kind": "reference",
                    "sample": "sparse_submanifold_conv3d 64->64 on the full config-0 shell, measured (median of 5)"}
            except Exception as ex:  # reported, not fatal
                result["sparse_conv_cfg0"]["cpu_reference"] = {"error": str(ex)[:200]}
            try:
                step_s, det = cpu_baseline_sample()
                result["cpu_baseline"] = {"value": round(1.0 / step_s, 8), "unit": "steps/s",
                                          "cores": det["threads"], "kind": "reference",
                                          "sample": ("reference sparse_transformer_cross_block_f32 at 256 voxels "
                                                     "x batch 2 (non-attention part scaled by N) + reference "
                                                     "attention at 512 x 2 (scaled by N^2) to N=4092 + "
                                                     "sparse_submanifold_conv3d 1024->1024 on a shell slab scaled "
                                                     "by neighbour pairs; extrapolated to one step"),
                                          "details": det}
            except Exception as ex:  # reported, not fatal
                result["cpu_baseline"] = {"value": None, "unit": "steps/s", "error": str(ex)[:200]}
        print(json.dumps(result), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(torch, model, img, cond, args, dev, world, rank):
    """End to end through the public API: per call, H2D of coords, noise and
    condition from pinned host memory, prepare (topology), sample K steps,
    D2H of the result; device-timed, max over ranks."""
    import torch.distributed as dist
    n_img = img.shape[0]
    from pixal3d.cpp_b200.workloads import batched
    h_coords = torch.from_numpy(batched(img, 2)).pin_memory()
    h_noise = torch.randn((n_img, CH)).pin_memory()
    h_cond = torch.cat([cond.cpu(), torch.zeros_like(cond.cpu())]).pin_memory()
    h_out = torch.empty((n_img, CH)).pin_memory()
    steps = args.steps
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(s)
    d_coords = h_coords.to(dev, non_blocking=True)
    d_x = h_noise.to(dev, non_blocking=True)
    d_ctx = h_cond.to(dev, non_blocking=True)
    model.prepare(d_coords, 2, (RES, RES, RES), [0, CTX_TOKENS, 2 * CTX_TOKENS])
    model.sample(d_x, d_ctx, steps=steps, guidance_strength=3.0)
    h_out.copy_(d_x, non_blocking=True)
    e1.record(s)
    torch.cuda.synchronize()
    from pixal3d.cpp_b200 import dist as D
    ms = D.max_over_ranks(e0.elapsed_time(e1), dev)
    h2d = h_coords.numel() * 4 + h_noise.numel() * 4 + h_cond.numel() * 4
    return {"value": round(world * steps / (ms / 1000.0), 3), "unit": "steps/s",
            "h2d_bytes_per_step": int(h2d / steps), "d2h_bytes_per_step": int(h_out.numel() * 4 / steps),
            "ms_per_call": round(ms, 2), "steps_per_call": steps,
            "includes": "H2D coords/noise/condition, topology prepare (neighbour map, downsample, RoPE table; "
                        "workspaces and the step graph reused when the topology's shape is unchanged), "
                        "K sampler steps, D2H latents"}


# ------------------------------------------------------- config 1 (one block)

def cfg1_flops(n: int) -> dict:
    """Algorithmic FLOPs of one config-1 block at n tokens (batch 1)."""
    lin = 2 * n * C * C * (3 + 1 + 1 + 1 + 4 + 4)
    kv = 2 * CTX_TOKENS * C * 2 * C
    self_attn = 4 * n * n * C
    cross = 4 * n * CTX_TOKENS * C
    return {"block": lin + kv + self_attn + cross, "linear": lin + kv, "self_attention": self_attn,
            "cross_attention": cross}


def run_cfg1(args):
    """One config-1 sparse transformer block (N = 21,766 tokens of 1,024
    channels, 16 heads, sinusoidal absolute PE, 1,029 condition tokens,
    t = 0.5) through the flow forward (identity input linear, final LayerNorm
    and a 1024 -> 8 output linear around the block): ms per forward."""
    import torch
    import torch.distributed as dist
    world, rank, local = init_ranks(torch, dist)
    from pixal3d.cpp_b200 import dist as D
    from pixal3d.cpp_b200 import ops
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    from pixal3d.cpp_b200.workloads import shell_coords
    global BLOCKS_RUN
    BLOCKS_RUN = 1
    dev = torch.device("cuda", local)
    coords = torch.from_numpy(shell_coords()).to(dev)
    n = coords.shape[0]
    w = make_weights(torch, dev, seed=1234)
    w["input_weight"] = torch.eye(C, device=dev)
    w["input_bias"] = torch.zeros(C, device=dev)
    hp = HParams(in_channels=C, out_channels=CH, model_channels=C, cond_channels=C, num_blocks=1, num_heads=HEADS,
                 mlp_ratio=4.0, pe_mode="ape", operand_dtype="f16")
    model = FlowModel(hp, w, device=local)
    del w
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    x = torch.randn((n, C), device=dev, generator=g)
    cond = torch.randn((CTX_TOKENS, C), device=dev, generator=g).to(torch.float16)
    ts = torch.full((1,), 500.0, device=dev)
    model.prepare(coords, 1, (RES, RES, RES), [0, CTX_TOKENS])
    out = torch.empty((n, CH), device=dev)
    for _ in range(max(args.warmup, 1)):
        model.forward(x, ts, cond, out=out)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.ctx(local).launches
    e0.record()
    for _ in range(args.steps):
        model.forward(x, ts, cond, out=out)
    e1.record()
    torch.cuda.synchronize()
    launches = ops.ctx(local).launches - launches0
    ms = D.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    fl = cfg1_flops(n)
    peaks, kind = load_peaks()
    if rank == 0:
        tf = fl["block"] / (ms / 1000.0) / 1e12
        print(json.dumps({
            "metric": "config-1 sparse transformer block forward (N=21,766, C=1024)", "value": round(ms, 3),
            "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "weak", "dtype": "f16 operands, f32 accumulate/residual",
            "data": "synthetic: config-0 shell coords, N(0,1) tokens and condition, random-init weights",
            "config": {"workload": "config1: one block, batch 1, N=21,766, 16 heads x 64, APE, 1,029 condition "
                                   "tokens; identity input linear, final LayerNorm and 1024->8 output linear",
                       "parallelism": f"replicas x{world}"},
            "block_tflop": round(fl["block"] / 1e12, 4), "achieved_tflops": round(tf, 1),
            "frac_of_bf16_burst": round(tf / peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]), 4),
            "gpu_launches": int(launches), "flops_split_tflop": {k: round(v / 1e12, 4) for k, v in fl.items()}}),
            flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_cfg1(args):
    """The reference's sparse_transformer_cross_block_f32 (oracle/_ref,
    compiled from the reference sources) once at the config-1 shape on all
    host threads.  Its self-attention is a serial loop, so one run takes on
    the order of 15-20 minutes."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import numpy as np
    from oracle import reflib, oracle as O
    from pixal3d.cpp_b200.workloads import shell_coords
    if not reflib.available():
        print(json.dumps({"impl": "reference", "workload": "cfg1", "unavailable": "oracle/_ref not built"}))
        return
    threads = os.cpu_count() or 1
    reflib.set_threads(threads)
    rng = np.random.default_rng(0)
    coords = shell_coords()
    n = coords.shape[0]
    cfg = O.BlockConfig(channels=C, num_heads=HEADS, mlp_hidden=4 * C, context_channels=C)
    w = {"modulation": (rng.standard_normal(6 * C) * 0.1).astype(np.float32)}
    for f, shp in [("self_to_qkv_weight", (3 * C, C)), ("self_to_out_weight", (C, C)), ("cross_to_q_weight", (C, C)),
                   ("cross_to_kv_weight", (2 * C, C)), ("cross_to_out_weight", (C, C)), ("mlp0_weight", (4 * C, C)),
                   ("mlp2_weight", (C, 4 * C))]:
        w[f] = (rng.standard_normal(shp) * 0.02).astype(np.float32)
        w[f.replace("weight", "bias")] = np.zeros(shp[0], np.float32)
    for f in ("self_q_gamma", "self_k_gamma", "norm2_weight", "cross_q_gamma", "cross_k_gamma"):
        w[f] = np.ones(C, np.float32)
    w["norm2_bias"] = np.zeros(C, np.float32)
    x = rng.standard_normal((n, C)).astype(np.float32)
    ctx = rng.standard_normal((CTX_TOKENS, C)).astype(np.float32)
    tmod = (rng.standard_normal((1, 6 * C)) * 0.1).astype(np.float32)
    t0 = time.perf_counter()
    out = reflib.transformer_block(coords, x, tmod, np.array([0, CTX_TOKENS], np.int64), ctx, None, cfg, w, 1,
                                   (RES, RES, RES))
    sec = time.perf_counter() - t0
    fl = cfg1_flops(n)
    print(json.dumps({"impl": "reference", "metric": "config-1 sparse transformer block forward (N=21,766, C=1024)",
                      "value": round(sec * 1000.0, 1), "unit": "ms", "higher_is_better": False, "dtype": "f32",
                      "cpu_baseline": {"value": round(sec * 1000.0, 1), "unit": "ms", "cores": threads,
                                       "kind": "reference", "sample": "one full config-1 block, measured once"},
                      "achieved_gflops": round(fl["block"] / sec / 1e9, 2), "finite": bool(np.isfinite(out).all()),
                      "e2e": {"value": round(sec * 1000.0, 1), "unit": "ms", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


# ------------------------------------------------------- decoders

def run_cfg3(args):
    """the shifted-window SLat decoder (no reference
    implementation) from the 21,766-voxel 64^3 shell: input linear to 768 +
    APE, 12 window blocks (8^3 windows, 12 heads x 64, MLP x4), subdivide to
    128^3 with a seeded Bernoulli(0.5) mask + SparseResBlock3d to C=128,
    subdivide to 256^3 + SparseResBlock3d to C=32, linear head to 32.  ms per
    decode; the CPU baseline is this repo's numpy restatement (no reference
    code exists) run once on the same inputs."""
    import numpy as np
    import torch
    import torch.distributed as dist
    world, rank, local = init_ranks(torch, dist)
    from pixal3d.cpp_b200 import dist as D
    from pixal3d.cpp_b200 import ops
    from pixal3d.cpp_b200.swin_decoder import SwinDecoder
    from pixal3d.cpp_b200.workloads import random_swin_weights, shell_coords
    dev = torch.device("cuda", local)
    cfg = {"model_channels": 768, "num_heads": 12, "window": 8, "spatial": RES, "groups": 32}
    rng = np.random.default_rng(41)
    w = random_swin_weights(rng, c0=768, stages=(128, 32), latent=8, out=32, blocks=12)
    coords = shell_coords()
    n = coords.shape[0]
    x = rng.standard_normal((n, 8)).astype(np.float32)
    m1 = (rng.random((n, 8)) < 0.5).astype(np.float32)
    m2 = (rng.random((int(m1.sum()), 8)) < 0.5).astype(np.float32)
    d = SwinDecoder(cfg, w, device=local)
    cd, xd = torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev)
    masks = [torch.from_numpy(m1).to(dev), torch.from_numpy(m2).to(dev)]
    for _ in range(max(args.warmup, 1)):
        oc, out = d.run(cd, xd, masks)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.ctx(local).launches
    e0.record()
    for _ in range(args.steps):
        oc, out = d.run(cd, xd, masks)
    e1.record()
    torch.cuda.synchronize()
    launches = ops.ctx(local).launches - launches0
    ms = D.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    if rank == 0:
        # algorithmic flops: block linears + window attention + stage convs/skips
        C0, blocks = 768, 12
        fl = blocks * 2 * n * C0 * C0 * (3 + 1 + 4 + 4)
        for shift in (0, 4):
            key = ((coords[:, 1] + shift) // 8 * 64 + (coords[:, 2] + shift) // 8) * 64 + (coords[:, 3] + shift) // 8
            cnt = np.bincount(key).astype(np.float64)
            fl += (blocks // 2) * 4 * float((cnt * cnt).sum()) * C0
        rows = [n]
        cur = cd
        ci = C0
        for mask, co in zip(masks, (128, 32)):
            oc_s, _, _, mm = ops.c2s_topology(cur, 2, mask)
            cur = oc_s.contiguous()
            pairs = int((ops.neighbor_map27(cur) < mm).sum().item())
            fl += 2 * pairs * ci * co + 2 * pairs * co * co + 2 * mm * ci * co
            rows.append(int(mm))
            ci = co
        fl += 2 * rows[-1] * 32 * 32
        peaks, kind = load_peaks()
        tf = fl / (ms / 1000.0) / 1e12
        result = {"metric": "config-3 shifted-window SLat decode (21,766 -> 256^3)", "value": round(ms, 3),
                  "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                  "higher_is_better": False, "scaling": "weak", "dtype": "f16 operands, f32 accumulate/residual",
                  "data": "synthetic: config-0 shell, N(0,1) latent, seeded Bernoulli(0.5) masks, random-init weights",
                  "config": {"workload": "config3: 12 window blocks C=768, stages to C=128 (128^3) and C=32 (256^3)",
                             "rows_per_level": rows, "parallelism": f"replicas x{world}"},
                  "tflop": round(fl / 1e12, 4), "achieved_tflops": round(tf, 1),
                  "frac_of_bf16_burst": round(tf / peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]), 4),
                  "gpu_launches": int(launches), "out_finite": bool(torch.isfinite(out).all())}
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as O
            t0 = time.perf_counter()
            O.swin_decoder_forward(coords, x, cfg, w, [m1, m2])
            sec = time.perf_counter() - t0
            result["cpu_baseline"] = {"value": round(sec * 1000.0, 1), "unit": "ms", "cores": os.cpu_count(),
                                      "kind": "port", "sample": "the numpy restatement of the whole decode, once "
                                                                "(the config has no reference implementation)"}
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_cascade(args):
    """The device SLat decoder at cascade scale: five levels (512 -> 256 ->
    128 -> 64 -> 32 channels) from the 9,682-voxel 64^3 shell to about 4.04M
    points, guided subdivision with seeded masks (keep 0.565), as the
    reference's real shape decode grows 9,857 -> 4,005,638 points.  Times the
    whole decode and each level (ConvNeXt blocks + the channel-to-spatial
    block into the next level), plus the predicted-subdivision decode."""
    import numpy as np
    import torch
    import torch.distributed as dist
    world, rank, local = init_ranks(torch, dist)
    from pixal3d.cpp_b200 import dist as D
    from pixal3d.cpp_b200 import workloads as WL
    from pixal3d.cpp_b200.decoder import Decoder
    dev = torch.device("cuda", local)
    w = WL.random_decoder_weights(np.random.default_rng(31), WL.CASCADE_CHANNELS, WL.CASCADE_BLOCKS,
                                  WL.CASCADE_LATENT, WL.CASCADE_OUT)
    coords = WL.cascade_input()
    x = np.random.default_rng(32).standard_normal((coords.shape[0], WL.CASCADE_LATENT)).astype(np.float32)
    guides = [torch.from_numpy(g).to(dev) for g in WL.cascade_guides(coords.shape[0], len(WL.CASCADE_CHANNELS), seed=33)]
    cd, xd = torch.from_numpy(coords).to(dev), torch.from_numpy(x).to(dev)
    levels = len(WL.CASCADE_CHANNELS)
    dg = Decoder(list(WL.CASCADE_CHANNELS), list(WL.CASCADE_BLOCKS), WL.CASCADE_LATENT, WL.CASCADE_OUT, w,
                 pred_subdiv=False, device=local)
    dp = Decoder(list(WL.CASCADE_CHANNELS), list(WL.CASCADE_BLOCKS), WL.CASCADE_LATENT, WL.CASCADE_OUT, w,
                 pred_subdiv=True, device=local)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            r = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, r

    reps = max(1, min(args.steps, 5))
    if world > 1:
        dist.barrier()
    ms_full, (oc, out, _) = timed(lambda: dg.run(cd, xd, 1, (RES, RES, RES), guides=guides), reps)
    cum = [0.0]
    for stop in range(1, levels):
        t, _ = timed(lambda: dg.run(cd, xd, 1, (RES, RES, RES), guides=guides, stop_level=stop), reps)
        cum.append(t)
    cum.append(ms_full)
    ms_pred, (ocp, _, _) = timed(lambda: dp.run(cd, xd, 1, (RES, RES, RES)), reps)
    ms_full = D.max_over_ranks(ms_full, dev)
    if rank == 0:
        rows = [coords.shape[0]]
        n = coords.shape[0]
        for g in guides:
            n = int((g > 0).sum().item())
            rows.append(n)
        print(json.dumps({
            "metric": "SLat decoder at cascade scale (9,682 -> 4.04M points)", "value": round(ms_full, 2),
            "unit": "ms", "n_gpus": world, "steps": reps, "higher_is_better": False, "scaling": "weak",
            "dtype": "f16 operands, f32 accumulate/residual",
            "data": "synthetic: r=16 shell at 64^3, N(0,1) 32-channel latent, seeded keep masks p=0.565, "
                    "random-init weights",
            "config": {"workload": "five-level decoder 512/256/128/64/32, one ConvNeXt block per level, guided "
                                   "subdivision", "parallelism": f"replicas x{world}"},
            "rows_per_level": rows, "out_rows": int(oc.shape[0]),
            "level_ms": [round(cum[i + 1] - cum[i], 2) for i in range(levels)],
            "points_per_s": round(oc.shape[0] / (ms_full / 1000.0), 1),
            "predicted_subdivision": {"ms": round(ms_pred, 2), "out_rows": int(ocp.shape[0])},
            "out_finite": bool(torch.isfinite(out).all()),
            "reference_published": "shape decoder 43.0-45.2 s GPU-first, 596.9 s hybrid, 1,822.6 s forced CPU "
                                   "(RTX 4090 D host, troubleshooting_history.md:387-390)"}), flush=True)
    dg.close()
    dp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------- config 4 (images/s)

CFG4_IMAGES = 64
CFG4_PACK_VOXELS = 400_000  # voxels of one varlen CFG batch (x2 rows with the unconditional copies)


def cfg4_cost(voxels: int) -> float:
    """Relative sampling cost of one image for the LPT plan: linear in the
    voxel count (convs, linears, norms, cross-attention) plus the trunk
    self-attention, quadratic in it: 24 x 210 us of a 32 ms config-2 step at
    21,766 voxels, about 16 % of the step's time."""
    return voxels * (1.0 + 0.16 * voxels / 21766.0)


def run_cfg4(args):
    """BASELINE config 4 on this rank's LPT share of the 64 images."""
    import numpy as np
    import torch
    import torch.distributed as dist

    world, rank, local = init_ranks(torch, dist)
    from pixal3d.cpp_b200 import dist as D
    from pixal3d.cpp_b200 import ops
    from pixal3d.cpp_b200.flow import FlowModel, HParams
    from pixal3d.cpp_b200.workloads import image_shells, pack_cfg, split_packs

    dev = torch.device("cuda", local)
    shells = image_shells(CFG4_IMAGES, seed=0)
    sizes = [int(c.shape[0]) for c in shells]
    plan = D.lpt_assign([cfg4_cost(v) for v in sizes], world)
    packs = split_packs(plan[rank], sizes, CFG4_PACK_VOXELS)
    hp = HParams(in_channels=CH, out_channels=CH, model_channels=C, cond_channels=C, num_blocks=BLOCKS,
                 num_heads=HEADS, mlp_ratio=4.0, io_resblocks=2, groups=32, operand_dtype="f16")
    w = make_weights(torch, dev, seed=1234)  # same seed on every rank: one model
    model = FlowModel(hp, w, device=local)
    del w
    torch.cuda.empty_cache()

    # Host inputs of this rank's images, pinned: each image's own condition
    # tokens and initial noise, generated from the image index (no broadcast).
    host = []
    for pk in packs:
        coords, offs = pack_cfg([shells[i] for i in pk])
        conds = [np.random.default_rng(10_000 + i).standard_normal((CTX_TOKENS, C)).astype(np.float16) for i in pk]
        noise = [np.random.default_rng(20_000 + i).standard_normal((sizes[i], CH)).astype(np.float32) for i in pk]
        ctx = np.concatenate(conds + [np.zeros((CTX_TOKENS * len(pk), C), np.float16)])
        host.append({
            "coords": torch.from_numpy(coords).pin_memory(),
            "x": torch.from_numpy(np.concatenate(noise)).pin_memory(),
            "ctx": torch.from_numpy(ctx.view(np.int16)).pin_memory(),
            "ctx_offsets": [CTX_TOKENS * j for j in range(2 * len(pk) + 1)],
            "out": torch.empty((int(offs[-1]), CH)).pin_memory(),
            "images": len(pk),
        })

    def run_pack(h, steps):
        d_coords = h["coords"].to(dev, non_blocking=True)
        d_x = h["x"].to(dev, non_blocking=True)
        d_ctx = h["ctx"].to(dev, non_blocking=True).view(torch.float16)
        model.prepare(d_coords, 2 * h["images"], (RES, RES, RES), h["ctx_offsets"])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        model.sample(d_x, d_ctx, steps=steps, guidance_strength=3.0)
        e1.record()
        h["out"].copy_(d_x, non_blocking=True)
        return e0, e1

    # warm-up: the first pack, one step (kernel loading, graph capture)
    if host:
        run_pack(host[0], max(1, min(args.warmup, 2)))
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.ctx(local).launches
    t0.record()
    sample_events = [run_pack(h, args.steps) for h in host]
    t1.record()
    torch.cuda.synchronize()
    launches = ops.ctx(local).launches - launches0
    clk = clocks.stop()
    ms_rank = t0.elapsed_time(t1)
    sample_ms = [a.elapsed_time(b) for a, b in sample_events]
    if world > 1:
        dist.barrier()
    ms_max = D.max_over_ranks(ms_rank, dev)
    ms_all = [ms_rank]
    if world > 1:
        tt = torch.tensor([ms_rank], dtype=torch.float64, device=dev)
        got = [torch.zeros_like(tt) for _ in range(world)]
        dist.all_gather(got, tt)
        ms_all = [float(g.item()) for g in got]
    finite = all(bool(torch.isfinite(h["out"]).all()) for h in host)
    outs = torch.cat([h["out"] for h in host]).to(dev) if host else torch.zeros((0, CH), device=dev)
    D.gather_rows(outs, dst=0)  # latents to rank 0 (outside the timed region)
    if rank == 0:
        h2d = sum(h["coords"].numel() * 4 + h["x"].numel() * 4 + h["ctx"].numel() * 2 for h in host)
        value = CFG4_IMAGES / (ms_max / 1000.0)
        result = {
            "metric": "SLat flow images/s, config 4 (64 ragged images, 25-step CFG sampler each)",
            "value": round(value, 3), "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_total": round(ms_max, 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulate/residual",
            "data": "synthetic: seeded ragged sphere shells, per-image N(0,1) noise and condition tokens, "
                    "random-init weights",
            "config": {"workload": "config4: 64 images, LPT over ranks, varlen CFG packs per rank",
                       "voxels_total": sum(sizes), "voxels_min": min(sizes), "voxels_max": max(sizes),
                       "pack_voxels_max": CFG4_PACK_VOXELS, "parallelism": f"dp{world} (images)"},
            "per_step_ms_rank0": round(sum(sample_ms) / max(1, len(sample_ms) * args.steps), 3),
            "packs_rank0": len(host), "rank_ms": [round(v, 1) for v in ms_all],
            "imbalance_measured": round(max(ms_all) / (sum(ms_all) / len(ms_all)), 4),
            "imbalance_planned_cost": round(D.imbalance(plan, [cfg4_cost(v) for v in sizes]), 4),
            "imbalance_planned_voxels": round(D.imbalance(plan, sizes), 4),
            "latents_finite_rank0": finite, "gpu_launches_rank0": int(launches), "clocks": clk,
            "e2e": {"value": round(value, 3), "unit": "images/s", "h2d_bytes_rank0": int(h2d),
                    "includes": "per pack: H2D coords/noise/conditions from pinned memory, topology prepare, "
                                "25 sampler steps (one captured step graph per pack shape), D2H latents"},
        }
        print(json.dumps(result), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------- reference arm

def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import reflib
    if not reflib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libp3dref.so not built (needs the "
                          "reference sources at build time)"}))
        return
    samples = []
    det = None
    for i in range(args.warmup + args.steps):
        step_s, det = cpu_baseline_sample()
        if i >= args.warmup:
            samples.append(step_s)
    step = statistics.median(samples)
    value = 1.0 / step
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 8), "unit": "steps/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step * 1000.0, 1),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (as ours)",
           "config": {"workload": "config2: full SLat-flow sampler step, CFG batch 2",
                      "method": "extrapolated from bounded samples of the reference CPU ops"},
           "cpu_baseline": {"value": round(value, 8), "unit": "steps/s", "cores": det["threads"],
                            "kind": "reference",
                            "sample": "reference block at 256 voxels x2 (scaled by N) + reference attention "
                                      "at 512 x2 (scaled by N^2) to N=4092 + conv slab scaled by neighbour pairs",
                            "details": det},
           "e2e": {"value": round(value, 8), "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.steps is None:
        args.steps = 25 if args.workload == "cfg4" else 20
    if args.workload == "cfg1":
        (run_reference_cfg1 if args.impl == "reference" else run_cfg1)(args)
        return
    if args.workload in ("cfg3", "cascade"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "workload": args.workload,
                              "unavailable": "the config-3 decoder has no reference implementation; the reference's "
                                             "cascade decoder (ggml GPU graph) cannot be built (empty ggml submodule)"}))
            return
        (run_cfg3 if args.workload == "cfg3" else run_cascade)(args)
        return
    if args.workload == "cfg4":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "workload": "cfg4",
                              "unavailable": "config 4 has no reference arm: 64 images x 25 steps of the CPU path "
                                             "would take days (the per-step figure is the config-2 reference arm)"}))
            return
        run_cfg4(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
