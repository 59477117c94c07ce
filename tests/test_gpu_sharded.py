"""Head-sharded Quest selection (configuration 5): per-shard partial scores,
the shard-ordered combine and the shared top-k, vs the unsharded kernel, the
oracle's restatement of the sharded order and the reference's selections."""

import math
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from helpers import full_quest_inputs, near_tie_report, pages_to_tokens
from hisparse_b200 import _lib, quest_selection
from hisparse_b200.sharded import head_slice, sharded_quest_selection

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _emulated(q, mn, mx, length, page_size, top_pages, keep_sink, shards):
    """W shards run one after another on one GPU: partials, stack, select."""
    lib = _lib.load()
    hq, hkv = q.shape[0], mn.shape[1]
    max_pages = mn.shape[0]
    lengths = torch.tensor([length], dtype=torch.int32, device=DEV)
    partials = torch.empty((shards, max_pages), dtype=torch.float32, device=DEV)
    status, stream = _lib.status_word(DEV).data_ptr(), _lib.stream_of(DEV)
    for r in range(shards):
        ks, qs = head_slice(hkv, hq, r, shards)
        qr = q[qs].contiguous()
        mr, xr = mn[:, ks].contiguous(), mx[:, ks].contiguous()
        ptrs = torch.tensor([mr.data_ptr(), xr.data_ptr()], dtype=torch.int64, device=DEV)
        _lib.check(lib.hs_quest_partial_scores_batched(
            1, qr.data_ptr(), 0, _lib.dtype_code(qr.dtype), ptrs[0:1].data_ptr(),
            ptrs[1:2].data_ptr(), _lib.dtype_code(mr.dtype), lengths.data_ptr(), qr.shape[0],
            mr.shape[1], qr.shape[1], max_pages, page_size, partials[r].data_ptr(), status,
            stream))
        torch.cuda.synchronize()  # mr/xr/ptrs are freed at the end of the iteration
    width = top_pages * page_size
    tokens = torch.empty(width, dtype=torch.int32, device=DEV)
    count = torch.empty(1, dtype=torch.int32, device=DEV)
    nbytes = lib.hs_quest_workspace_bytes(1, max_pages)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    _lib.check(lib.hs_quest_select_partials(
        shards, partials.data_ptr(), 1, lengths.data_ptr(), hq, max_pages, page_size,
        top_pages, int(keep_sink), tokens.data_ptr(), width, count.data_ptr(), ws.data_ptr(),
        nbytes, status, stream))
    torch.cuda.synchronize()
    return [t for t in tokens.tolist()[:int(count.item())]], partials


def _metadata(gen, pages, hkv, d, dtype):
    keys = torch.randn(pages, 4, hkv, d, generator=gen).to(dtype)
    return keys.float().amin(1).to(dtype), keys.float().amax(1).to(dtype)


def test_one_shard_equals_unsharded_selection():
    gen = torch.Generator().manual_seed(5)
    for hq, hkv, d, p, length, top, dtype in [(32, 8, 128, 16, 32768, 128, torch.bfloat16),
                                              (8, 2, 32, 16, 150, 4, torch.float32),
                                              (6, 2, 24, 7, 1000, 9, torch.float16)]:
        pages = math.ceil(length / p)
        q = torch.randn(hq, d, generator=gen).to(dtype).to(DEV)
        mn, mx = (t.to(DEV) for t in _metadata(gen, pages, hkv, d, dtype))
        for sink in (True, False):
            ref = quest_selection(q, mn, mx, length, p, top, sink)
            got = sharded_quest_selection(q, mn, mx, length, p, top, sink)
            assert torch.equal(ref.device_tokens, got.device_tokens)
    assert not _lib.device_flags(DEV)


@pytest.mark.parametrize("shards", [2, 4])
@pytest.mark.parametrize("hq,hkv,d,p,length,top,dtype", [
    (28, 4, 128, 64, 1048576, 128, torch.bfloat16),   # configuration 5
    (32, 8, 128, 16, 32768, 128, torch.bfloat16),
    (8, 4, 64, 16, 5000, 17, torch.float16),
])
def test_emulated_shards_match_oracle(shards, hq, hkv, d, p, length, top, dtype):
    if hkv % shards:
        pytest.skip("KV heads do not split evenly")
    gen = torch.Generator().manual_seed(6 + shards)
    pages = math.ceil(length / p)
    q = torch.randn(hq, d, generator=gen).to(dtype)
    mn, mx = _metadata(gen, pages, hkv, d, dtype)
    got, partials = _emulated(q.to(DEV), mn.to(DEV), mx.to(DEV), length, p, top, True, shards)
    scores = oracle.quest_sharded_scores(q, mn, mx, pages, shards)
    tokens, count = oracle.quest_select(scores, length, p, top, True)
    assert got == tokens[:count].tolist()
    # each shard's partial is the oracle's undivided head sum of its slice
    ks, qs = head_slice(hkv, hq, shards - 1, shards)
    part = oracle.quest_sharded_scores(q[qs], mn[:, ks], mx[:, ks], pages, 1) * np.float32(
        hq // shards)
    np.testing.assert_allclose(partials[-1, :pages].cpu().numpy(), part, rtol=1e-6, atol=1e-6)
    assert not _lib.device_flags(DEV)


def test_sharded_selection_agrees_with_reference(golden):
    """The reference averages over all heads in torch's order; the sharded
    fixed-order sum picks the same pages on every recorded case."""
    checked = 0
    for case in golden("quest_cases"):
        hq, hkv = case["query"].shape[0], case["minimum"].shape[1]
        if hkv % 2 or "tokens_1" not in case:
            continue
        q, mn, mx = (case[k].to(DEV) for k in ("query", "minimum", "maximum"))
        got, _ = _emulated(q, mn, mx, case["length"], case["page_size"], case["top_pages"],
                           True, 2)
        pages = math.ceil(case["length"] / case["page_size"])
        if case["top_pages"] >= pages:
            continue
        assert list(got) == list(case["tokens_1"]), f"{case['name']}: " + near_tie_report(
            case["tokens_1"], got, case["query"], case["minimum"], case["maximum"],
            case["length"], case["page_size"], case["top_pages"], True)
        checked += 1
    assert checked >= 5


@pytest.mark.parametrize("shards", [2, 4])
def test_sharded_full_size_equals_reference(golden, shards):
    """Configuration 5 at full size (16,389 pages, 28 / 4 heads split over 2 or
    4 shards): the shard-ordered selection equals the reference's recorded
    selection page for page, sink on and off."""
    checked = 0
    for case in golden("quest_full_cases"):
        if not case["name"].startswith("config5"):
            continue
        q, mn, mx, digest = full_quest_inputs(case["q_heads"], case["kv_heads"],
                                              case["head_dim"], case["page_size"],
                                              case["max_pages"], case["seed"])
        assert digest == case["digest"], f"{case['name']}: input generator changed"
        p, top, length = case["page_size"], case["top_pages"], case["length"]
        for sink in (1, 0):
            got, _ = _emulated(q.to(DEV), mn.to(DEV), mx.to(DEV), length, p, top, bool(sink),
                               shards)
            want = pages_to_tokens(case[f"pages_{sink}"], length, p)
            assert got == want, f"{case['name']} sink={sink} shards={shards}: " + \
                near_tie_report(want, got, q, mn, mx, length, p, top, bool(sink))
            checked += 1
    assert checked == 6
    assert not _lib.device_flags(DEV)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q, mn, mx, length, p, top, out):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "nano-hisparse_b200"))
    import datetime

    import torch.distributed as dist

    from hisparse_b200.sharded import head_slice as hs_slice
    from hisparse_b200.sharded import sharded_quest_selection as sqs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        ks, qs = hs_slice(mn.shape[1], q.shape[0], rank, world)
        sel = sqs(q[qs].to(dev), mn[:, ks].contiguous().to(dev), mx[:, ks].contiguous().to(dev),
                  length, p, top, group=dist.group.WORLD)
        out[rank] = sel.device_tokens.cpu().tolist()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nccl_agree_with_emulation():
    import torch.multiprocessing as mp

    gen = torch.Generator().manual_seed(9)
    hq, hkv, d, p, length, top = 28, 4, 128, 64, 262144, 128
    pages = math.ceil(length / p)
    q = torch.randn(hq, d, generator=gen).to(torch.bfloat16)
    mn, mx = _metadata(gen, pages, hkv, d, torch.bfloat16)
    expected, _ = _emulated(q.to(DEV), mn.to(DEV), mx.to(DEV), length, p, top, True, 2)
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_rank, args=(2, _free_port(), q, mn, mx, length, p, top, out), nprocs=2,
                       start_method="spawn", join=True)
    for rank in range(2):
        assert [t for t in out[rank] if t >= 0] == expected


def _batch_rank(rank, world, port, q, keys, length, p, top, out):
    """One rank of a head-sharded DecodeBatch layer over its KV-head slice."""
    import sys
    from pathlib import Path

    import numpy as np

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "nano-hisparse_b200"))
    import datetime

    import torch.distributed as dist

    from hisparse_b200 import CacheConfig, DecodeBatch, HotConfig, RowCache
    from hisparse_b200 import _lib as lib_
    from hisparse_b200.sharded import head_slice as hs_slice

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        ks, qs = hs_slice(keys.shape[3], q.shape[0], rank, world)
        kv = keys[:, :, :, ks].contiguous()                  # [n, 2, P, Hkv_l, D]
        n, hkv, d = kv.shape[0], kv.shape[3], kv.shape[4]
        hot = HotConfig(top * p, 2 * top * p)
        hb = hot.hot_blocks(p)
        resident = np.full(n, -1)
        resident[[0, n - 2, n - 1]] = [0, 1, 2]
        config = CacheConfig(gpu_pages=3 + hb, host_pages=n, page_size=p, kv_heads=hkv,
                             head_dim=d, device=str(dev), dtype=kv.dtype)
        cache = RowCache(config, hot, host=kv.pin_memory())
        cache.pool.zero_()
        cache.pool[:3] = kv[[0, n - 2, n - 1]].to(dev)
        cache.add_layer(0, 0, length, np.arange(n), resident, list(range(3, 3 + hb)))
        mins = kv[:, 0].float().amin(1).to(kv.dtype)[None].to(dev)
        maxs = kv[:, 0].float().amax(1).to(kv.dtype)[None].to(dev)
        batch = DecodeBatch(cache, [0], 1, {0: mins}, {0: maxs}, top, q[qs].shape[0],
                            group=dist.group.WORLD)
        counts = torch.zeros((1, 3), dtype=torch.int64, device=dev)
        with torch.cuda.stream(batch.compute):
            o = batch.layer(0, q[qs][None].to(dev).contiguous(), counts=counts)
        torch.cuda.synchronize(dev)
        eager_tokens = batch.tokens[0].cpu().tolist()
        # the same selection from a segmented step graph: the layer's two
        # captured pieces with the all-gather issued between them at replay
        from hisparse_b200.batched import DecodeGraph

        streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        gbatch = DecodeBatch(cache, [0], 1, {0: mins}, {0: maxs}, top, q[qs].shape[0],
                             group=dist.group.WORLD, streams=streams)
        graph = DecodeGraph([gbatch], 1)
        graph.queries[0][0].copy_(q[qs][None].to(dev))
        graph.replay()
        torch.cuda.synchronize(dev)
        graph_result = (graph.segmented, gbatch.tokens[0].cpu().tolist(),
                        bool(torch.isfinite(graph.outputs[0]).all()))
        del graph
        out[rank] = (eager_tokens, counts.cpu().tolist(), bool(torch.isfinite(o).all()),
                     lib_.device_flags(dev), graph_result)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_sharded_decode_batch_on_two_ranks():
    """DecodeBatch with a process group: both ranks select the same pages (the
    emulated sharded selection of the whole request), make the same plan and
    attend over their own heads."""
    import torch.multiprocessing as mp

    gen = torch.Generator().manual_seed(12)
    hq, hkv, d, p, length, top = 8, 4, 64, 16, 3000, 12
    n = math.ceil(length / p)
    q = torch.randn(hq, d, generator=gen).to(torch.bfloat16)
    keys = torch.randn(n, 2, p, hkv, d, generator=gen).to(torch.bfloat16)
    mn = keys[:, 0].float().amin(1).to(torch.bfloat16)
    mx = keys[:, 0].float().amax(1).to(torch.bfloat16)
    expected, _ = _emulated(q.to(DEV), mn.to(DEV), mx.to(DEV), length, p, top, True, 2)
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_batch_rank, args=(2, _free_port(), q, keys, length, p, top, out),
                       nprocs=2, start_method="spawn", join=True)
    assert [t for t in out[0][0] if t >= 0] == expected
    assert out[0][0] == out[1][0] and out[0][1] == out[1][1]
    assert out[0][2] and out[1][2] and not out[0][3] and not out[1][3]
    for r in range(2):
        assert out[r][4] == (True, out[r][0], True)
