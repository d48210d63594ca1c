# SPDX-License-Identifier: Unlicense
"""The multi-GPU host logic of bench.py on two gloo ranks (CPU): each rank
gets a disjoint block of tile pairs, the barrier passes, and the reported
time is the maximum over ranks (the device times of a weak-scaling run)."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    import bench

    r, w, local = bench.dist_setup(world)
    bench.barrier(w)
    worst = bench.allmax(w, 10.0 * (r + 1))
    seeds = bench.rank_tile_seeds(r, 3)
    everyone = [None] * w
    dist.all_gather_object(everyone, seeds)
    q.put((r, w, local, worst, everyone))
    dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_two_ranks_shard_tiles_and_take_the_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=150) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, (rank, world, local, worst, everyone) in enumerate(res):
        assert (rank, world, local) == (r, 2, r)
        assert worst == 20.0
        flat = [s for block in everyone for s in block]
        assert len(flat) == len(set(flat)) == 6
