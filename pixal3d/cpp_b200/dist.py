"""Data-parallel plumbing for the SLat sampler on N GPUs (one process per GPU).

Images are independent and the two CFG branches of an image stay together
(batch items [0, I) conditional, [I, 2I) unconditional on one GPU), so the
path shards with no collective inside the step loop.
- Before timing: rank 0's condition tokens are broadcast.
- After timing: the sampled latents are gathered to rank 0, and the step time
  is reduced as the max over ranks.

Every rank takes the same collective calls in the same order.  The functions
work with any torch.distributed backend: NCCL on the GPU box, gloo in the CPU
tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def lpt_assign(sizes: list[int], world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of images (cost ~ voxel
    count) to `world` ranks: largest image first, each to the least loaded
    rank (ties -> lowest rank).  Deterministic, so every rank computes the
    same plan without communicating."""
    loads = [0] * world
    plan: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(sizes)), key=lambda j: (-sizes[j], j)):
        r = min(range(world), key=lambda k: (loads[k], k))
        plan[r].append(i)
        loads[r] += sizes[i]
    for p in plan:
        p.sort()
    return plan


def imbalance(plan: list[list[int]], sizes: list[int]) -> float:
    """max rank load / mean rank load (1.0 = perfectly balanced)."""
    loads = [sum(sizes[i] for i in p) for p in plan]
    mean = sum(loads) / max(len(loads), 1)
    return max(loads) / mean if mean > 0 else 1.0


def world_rank() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def broadcast_(t: torch.Tensor, src: int = 0) -> torch.Tensor:
    """In-place broadcast of rank `src`'s tensor (no-op on one process)."""
    world, _ = world_rank()
    if world > 1:
        dist.broadcast(t, src=src)
    return t


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """The max of a per-rank scalar (a device-timed duration) over all ranks."""
    world, _ = world_rank()
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(x: torch.Tensor, dst: int = 0) -> list[torch.Tensor] | None:
    """Gather each rank's [rows_r, C] tensor to rank `dst` (rows may differ per
    rank: padded to the max for the collective, trimmed after).  Returns the
    list on `dst`, None elsewhere."""
    world, rank = world_rank()
    if world == 1:
        return [x]
    n = torch.tensor([x.shape[0]], dtype=torch.int64, device=x.device)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    counts = [int(c.item()) for c in counts]
    rows = max(counts)
    pad = x.new_zeros((rows,) + tuple(x.shape[1:]))
    pad[: x.shape[0]] = x
    bufs = [torch.empty_like(pad) for _ in range(world)] if rank == dst else None
    dist.gather(pad, bufs, dst=dst)
    if rank != dst:
        return None
    return [b[:c] for b, c in zip(bufs, counts)]
