"""Multi-process host logic on the CPU (gloo, world size 2, 127.0.0.1): the rank/shard layer that
bench.py uses for one process per GPU.  Each rank reconstructs its contiguous shard of the batch
with the float64 oracle; the gathered shards equal the whole batch computed in one process (chains
are independent: no exchange on the hot path), and the max-over-ranks reduction returns the
slowest rank's time."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, batch: int, points: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import nerf64

    d = bench.Dist(world, device_needed=False)
    try:
        lo, hi = bench.shard(batch, d.world, d.rank)
        inp = bench.make_inputs(batch, points, seed=0)
        part = {k: v[lo:hi].double() for k, v in inp.items()}
        xyz = nerf64.reconstruct64(part["lengths"], part["angles"], part["dihedrals"])
        # uneven shards: pad to the largest, gather, trim
        per = -(-batch // world)
        padded = torch.zeros(per, points, 3, dtype=torch.float64)
        padded[: hi - lo] = xyz
        gathered = [torch.empty_like(padded) for _ in range(world)]
        d.pg.all_gather(gathered, padded)
        slowest = d.max(float(10 + rank))
        if d.rank == 0:
            pieces = []
            for r in range(world):
                a, b = bench.shard(batch, world, r)
                pieces.append(gathered[r][: b - a])
            torch.save({"xyz": torch.cat(pieces), "slowest": slowest}, os.path.join(out_dir, "result.pt"))
    finally:
        d.close()


@pytest.mark.parametrize("batch", [7, 8])
def test_two_ranks_shard_and_max(tmp_path, batch):
    world, points = 2, 40
    mp.start_processes(_worker, args=(world, _free_port(), batch, points, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    res = torch.load(tmp_path / "result.pt")
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle import nerf64

    inp = bench.make_inputs(batch, points, seed=0)
    whole = nerf64.reconstruct64(inp["lengths"].double(), inp["angles"].double(), inp["dihedrals"].double())
    assert torch.equal(res["xyz"], whole)
    assert res["slowest"] == 11.0
