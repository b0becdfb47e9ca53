"""Head sharding across ranks (one process per GPU).

Every step of the SparsePR layer is per head (per-head k-means, selection,
attention and repair), so N ranks split the heads into N contiguous shards and
run with no collective on the data path.  Only the step statistics cross
ranks: times as the maximum over ranks (the job is as slow as its slowest
rank), work as the sum.
"""

from __future__ import annotations

import torch

__all__ = ["head_shard", "reduce_step_stats"]


def head_shard(heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous head range ``[h0, h1)`` of ``rank``; heads must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if heads % world:
        raise ValueError(f"{heads} heads do not shard over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def reduce_step_stats(times: list[float], work: list[float], device=None) -> tuple[list[float], list[float]]:
    """All-reduce per-rank step statistics: max of ``times``, sum of ``work``.

    Works on any initialised process group (NCCL on GPUs, gloo on CPU); with
    no process group it returns the inputs."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(times), list(work)
    t = torch.tensor(times, dtype=torch.float64, device=device)
    w = torch.tensor(work, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(w, op=dist.ReduceOp.SUM)
    return t.tolist(), w.tolist()
