"""The N>1 host path of bench.py / the data-parallel sampler on CPU: two gloo
ranks (world_size 2) run the same collective sequence as the GPU ranks.
1. Broadcast of rank 0's condition tokens.
2. A per-rank, per-image update of each rank's own LPT share of ragged images.
   The update is a stand-in for the device sampler.
3. Max-over-ranks timing and a ragged gather of the latents to rank 0.
The gathered result must equal the single-process result bit for bit.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from pixal3d.cpp_b200 import dist as D  # noqa: E402

SIZES = [5000, 812, 3100, 2999, 64, 4096, 1500, 7]  # ragged voxel counts per image
CH = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _images():
    rng = np.random.default_rng(0)
    return [torch.from_numpy(rng.standard_normal((n, CH)).astype(np.float32)) for n in SIZES]


def _fake_sample(x: torch.Tensor, cond: torch.Tensor, steps: int = 3) -> torch.Tensor:
    # deterministic stand-in for the per-image CFG sampler
    for s in range(steps):
        x = x - 0.1 * (x - cond[: x.shape[1]].sum() * 1e-3 * (s + 1))
    return x


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cond = torch.randn(1029 * 4) if rank == 0 else torch.zeros(1029 * 4)
        D.broadcast_(cond, src=0)
        plan = D.lpt_assign(SIZES, world)
        imgs = _images()
        mine = [_fake_sample(imgs[i], cond) for i in plan[rank]]
        local = torch.cat(mine) if mine else torch.zeros((0, CH))
        t = D.max_over_ranks(float(rank + 1))
        got = D.gather_rows(local, dst=0)
        if rank == 0:
            torch.save({"cond": cond, "parts": got, "plan": plan, "tmax": t}, os.path.join(out_dir, "r0.pt"))
        else:
            assert got is None
            torch.save({"tmax": t}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_lpt_assign_balances_and_is_deterministic():
    plan = D.lpt_assign(SIZES, 2)
    assert sorted(i for p in plan for i in p) == list(range(len(SIZES)))
    assert plan == D.lpt_assign(SIZES, 2)
    assert D.imbalance(plan, SIZES) < 1.01
    plan8 = D.lpt_assign(list(range(8000, 60000, 800)), 8)
    assert D.imbalance(plan8, list(range(8000, 60000, 800))) < 1.05
    assert D.lpt_assign([3, 1], 4) == [[0], [1], [], []]


def test_two_gloo_ranks_match_single_process(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0 = torch.load(tmp_path / "r0.pt")
    r1 = torch.load(tmp_path / "r1.pt")
    assert r0["tmax"] == 2.0 and r1["tmax"] == 2.0
    cond = r0["cond"]
    imgs = _images()
    for rank, part in enumerate(r0["parts"]):
        idx = r0["plan"][rank]
        exp = torch.cat([_fake_sample(imgs[i], cond) for i in idx]) if idx else torch.zeros((0, CH))
        assert torch.equal(part, exp), f"rank {rank} latents differ"
