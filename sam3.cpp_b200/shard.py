"""Data-parallel plumbing of the encoder across GPUs (one process per GPU).

The path shards by image: sam3.cpp encodes one image per sam3_state, so N
GPUs run N independent encoder replicas with no collective on the data path.
These helpers are the whole of the host-side multi-GPU logic and are shared
by bench.py and the tests.
"""
from __future__ import annotations


def image_shard(batch: int, rank: int, world: int) -> list[int]:
    """Images of a step's batch that `rank` of `world` encodes: r, r+N, r+2N, ...

    Every image goes to exactly one rank; ranks differ by at most one image.
    """
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"bad shard request: batch={batch} rank={rank} world={world}")
    return list(range(rank, batch, world))


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar over the default process group (identity when
    no group is initialised).  `device` is where the reduction tensor lives:
    the rank's GPU under NCCL, the CPU under gloo."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
