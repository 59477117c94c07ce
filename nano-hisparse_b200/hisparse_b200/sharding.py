"""Request-level data parallelism: one process per GPU, requests sharded.

Requests are independent, so the hot path needs no collective: each rank owns
its pool, pinned host store and tables (configuration 4 of the reference's
headline: requests partitioned across the GPUs of one box). The only
cross-rank operation is reporting — the slowest rank's time.
"""

from __future__ import annotations

import numpy as np
import torch


def requests_for_rank(request_ids, rank: int, world: int) -> list:
    """Round-robin shard of `request_ids` owned by `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return list(request_ids)[rank::world]


def lognormal_lengths(count: int, median: int, low: int, high: int, seed: int) -> list[int]:
    """Seeded prompt lengths, lognormal around `median`, clipped to [low, high]."""
    rng = np.random.default_rng(seed)
    values = np.exp(rng.normal(np.log(median), 0.75, size=count))
    return [int(v) for v in np.clip(np.round(values), low, high)]


def max_over_ranks(value: float, device=None) -> float:
    """Largest `value` over all ranks (identity without a process group)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
