"""Host logic of the head-sharded multi-GPU path, on two gloo ranks (CPU).

bench.py --gpus N runs one process per GPU, each on a contiguous shard of the
heads, with no collective on the data path; the step statistics are reduced
once (time: max over ranks, work: sum).  These tests run that logic with the
gloo backend on CPU processes."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sparsepr_b200.sharding import head_shard, reduce_step_stats
from sparsepr_b200.synthetic import random_init_indices


def test_head_shards_cover_all_heads_once():
    for world in (1, 2, 4, 5, 8):
        covered = []
        for rank in range(world):
            h0, h1 = head_shard(40, world, rank)
            covered += list(range(h0, h1))
        assert covered == list(range(40))
    with pytest.raises(ValueError):
        head_shard(40, 3, 0)
    with pytest.raises(ValueError):
        head_shard(40, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        heads, n, k = 6, 500, 16
        h0, h1 = head_shard(heads, world, rank)
        # A shard starts k-means from its rows of the all-heads cold-start draw.
        mine = random_init_indices(heads, n, k, seed=3)[h0:h1]
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        # Per-rank step statistics: the job time is the slowest rank's, work adds up.
        times, work = reduce_step_stats([10.0 + rank, 5.0 - rank], [float(h1 - h0), 100.0 * (rank + 1)])
        if rank == 0:
            out.put((torch.cat(gathered).tolist(), times, work))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_stats_and_share_the_init_draw():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    init_rows, times, work = out.get(timeout=10)
    assert init_rows == random_init_indices(6, 500, 16, seed=3).tolist()
    assert times == [11.0, 5.0]
    assert work == [6.0, 300.0]
