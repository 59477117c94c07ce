"""Request-level data parallelism: one process per GPU, requests sharded.

Requests are independent, so the hot path needs no collective: each rank owns
its pool, pinned host store and tables (configuration 4 of the reference's
headline: requests partitioned across the GPUs of one box). The only
cross-rank operation is reporting — the slowest rank's time.
"""

from __future__ import annotations

import os
from pathlib import Path

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


def parse_cpulist(text: str) -> set[int]:
    """CPU ids of a sysfs cpulist such as "0-55,112-167"."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def pci_local_cpus(domain: int, bus: int, device: int,
                   sysfs: str | Path = "/sys/bus/pci/devices") -> set[int] | None:
    """CPUs of the NUMA node a PCI device hangs off (its sysfs local_cpulist),
    or None when the file is not there."""
    path = Path(sysfs) / f"{domain:04x}:{bus:02x}:{device:02x}.0" / "local_cpulist"
    try:
        return parse_cpulist(path.read_text())
    except (OSError, ValueError):
        return None


def bind_to_device_node(device_index: int, sysfs: str | Path = "/sys/bus/pci/devices"):
    """Restrict this process to the CPUs next to CUDA device `device_index`, so
    pinned host memory it allocates afterwards (placed on first touch) sits on
    the GPU's own NUMA node and its gathers cross no socket link. Returns the
    CPU set now in use, or None when the topology is unknown (nothing changes)."""
    props = torch.cuda.get_device_properties(device_index)
    local = pci_local_cpus(props.pci_domain_id, props.pci_bus_id, props.pci_device_id, sysfs)
    if not local:
        return None
    allowed = local & os.sched_getaffinity(0)
    if not allowed:
        return None
    os.sched_setaffinity(0, allowed)
    return allowed
