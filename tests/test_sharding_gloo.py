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


def _ulysses_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from sparsepr_b200.ulysses import UlyssesSparseAttention, head_to_seq, seq_to_head

        g = torch.Generator().manual_seed(7)
        b, n, h, d = 1, 12, 4, 8
        x = torch.randn(b, n, h, d, generator=g)  # full tensor, BLHD
        ns, hs = n // world, h // world
        mine = x[:, rank * ns:(rank + 1) * ns].contiguous()
        heads = seq_to_head(mine)
        ok_heads = torch.equal(heads, x.permute(0, 2, 1, 3)[:, rank * hs:(rank + 1) * hs])
        ok_back = torch.equal(head_to_seq(heads), mine)

        # A head-local stand-in for the layer: per head, mix every token (cumulative
        # sum over the sequence) and tag the head, so a wrong token or head order shows.
        def layer(q, k, v):
            tag = torch.arange(q.shape[1], dtype=q.dtype).view(1, -1, 1, 1) + rank * hs
            return q.cumsum(dim=2) + 100 * tag + k - v

        got = UlyssesSparseAttention(attention=layer)(mine, mine, mine)
        full = x.permute(0, 2, 1, 3).cumsum(dim=2) + 100 * torch.arange(h, dtype=x.dtype).view(1, -1, 1, 1)
        want = full.permute(0, 2, 1, 3)[:, rank * ns:(rank + 1) * ns]
        out.put((rank, ok_heads, ok_back, bool(torch.allclose(got, want))))
    finally:
        dist.destroy_process_group()


def test_ulysses_exchange_on_two_gloo_ranks():
    """Sequence shards -> head shards (all tokens) -> layer -> sequence shards,
    over all_to_all on two gloo ranks, against the same computation unsharded."""
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = sorted(out.get(timeout=10) for _ in range(world))
    assert all(r[1:] == (True, True, True) for r in results), results
