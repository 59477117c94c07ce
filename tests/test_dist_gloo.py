"""Data-parallel plumbing on CPU: two gloo ranks shard requests with no
overlap and agree on the slowest rank's time (bench.py's reporting path)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "nano-hisparse_b200"))
    from hisparse_b200.sharding import max_over_ranks, requests_for_rank

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = requests_for_rank(range(256), rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        slowest = max_over_ranks(10.0 + rank)
        out[rank] = (sorted(sum(gathered, [])) == list(range(256)), slowest)
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_reduce():
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world,
                       start_method="spawn", join=True)
    assert dict(out) == {0: (True, 11.0), 1: (True, 11.0)}
