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


def _sharded_worker(rank, world, port, out):
    import sys
    from pathlib import Path

    import numpy as np

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "nano-hisparse_b200"))
    sys.path.insert(0, str(root))
    import oracle
    from hisparse_b200.sharded import head_slice

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(3)
        hq, hkv, d, p, length, top = 8, 4, 32, 16, 4000, 12
        pages = -(-length // p)
        q = torch.randn(hq, d, generator=gen)
        keys = torch.randn(pages, 4, hkv, d, generator=gen)
        mn, mx = keys.amin(1), keys.amax(1)
        ks, qs = head_slice(hkv, hq, rank, world)
        # this rank's undivided head sums (the oracle stands in for the kernel)
        part = oracle.quest_sharded_scores(q[qs], mn[:, ks], mx[:, ks], pages, 1) * np.float32(
            hq // world)
        mine = torch.from_numpy(part)
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        out[rank] = [t.numpy().tobytes() for t in gathered]
    finally:
        dist.destroy_process_group()


def test_two_ranks_exchange_partial_scores_in_rank_order():
    """Head-sharded selection's exchange: every rank ends with the partials of
    all ranks in rank order (the bytes the shared top-k is computed from)."""
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_sharded_worker, args=(world, _free_port(), out), nprocs=world,
                       start_method="spawn", join=True)
    assert out[0] == out[1] and len(out[0]) == world and out[0][0] != out[0][1]


def _agreement_worker(rank, world, port, out):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "nano-hisparse_b200"))
    from hisparse_b200.sharded import group_world, same_on_every_rank

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        group = dist.group.WORLD
        out[rank] = (
            group_world(None),                                  # no group: this rank alone
            group_world(group),
            same_on_every_rank(group, (2048, 32768, 16, 128)),  # equal on both ranks
            same_on_every_rank(group, (2048 + rank, 32768)),    # table lengths differ
            same_on_every_rank(group, (7, -3 * rank)),          # one negative value differs
        )
    finally:
        dist.destroy_process_group()


def test_head_sharded_exchange_checks_agreement_and_needs_a_named_group():
    """An initialised default group does not make a selection head-sharded
    (group=None is one rank), and ranks whose exchange sizes differ are caught
    on every rank before the all-gather."""
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_agreement_worker, args=(world, _free_port(), out), nprocs=world,
                       start_method="spawn", join=True)
    assert out[0] == out[1] == (1, 2, True, False, False)
