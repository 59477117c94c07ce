"""RowCache (resolve stream/event protocol) and DecodeBatch end to end."""

import math

import numpy as np
import pytest
import torch

import oracle
from helpers import TOL, rebuild_host
from hisparse_b200 import (CacheConfig, DecodeBatch, HotConfig, LogicalTopK, RowCache, _lib,
                           quest_selection, row_attention)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _scenario(golden, name):
    return next(s for s in golden("scenarios") if s["name"] == name)


@pytest.mark.parametrize("name", ["row_misses_and_resident_hits", "late_hits_protected"])
def test_row_attention_through_row_cache(golden, name):
    """Consecutive row_attention calls with no appends in between: the cache's
    own tag/LRU state carries from call to call, as in the reference's
    tests/test_hybrid.py:42-93."""
    scenario = _scenario(golden, name)
    recs = scenario["records"]
    first = recs[0]
    pool0 = first["pool_before"]
    _, _, p, hkv, d = pool0.shape
    host = torch.zeros((first["host_pages"], *pool0.shape[1:]), dtype=pool0.dtype)
    for rec in recs:
        h = rebuild_host(rec)
        if rec["host_blocks"].numel():
            host[rec["host_blocks"]] = h[rec["host_blocks"]]
    config = CacheConfig(gpu_pages=pool0.shape[0], host_pages=first["host_pages"], page_size=p,
                         kv_heads=hkv, head_dim=d, device=DEV, dtype=pool0.dtype)
    cache = RowCache(config, HotConfig(4, 4), host=host.pin_memory())
    cache.pool.copy_(pool0)
    tables = cache.add_layer("a", 0, first["length"], first["source"], first["resident"],
                             first["hot"].tolist())
    tables.tags.copy_(first["tags"])
    tables.lru.copy_(first["lru"])
    for i, rec in enumerate(recs):
        out = row_attention(rec["query"].to(DEV), cache, "a", 0,
                            LogicalTopK(rec["positions"].to(DEV)))
        torch.testing.assert_close(out.cpu().double(), rec["out"].double(),
                                   **TOL[pool0.dtype], msg=f"{name}[{i}]")
        assert tables.tags.tolist() == rec["tags_after"].tolist()
    assert cache.snapshot()["row_stats"] == scenario["row_stats"]
    assert not tables.busy


def test_lease_rejects_double_resolve_and_double_release():
    config = CacheConfig(gpu_pages=4, host_pages=8, page_size=4, kv_heads=1, head_dim=8,
                         device=DEV)
    cache = RowCache(config, HotConfig(4, 4))
    cache.add_layer("a", 0, 12, [0, 1, 2], [-1, -1, 3], [0])
    lease = cache.resolve("a", 0, LogicalTopK(torch.tensor([0, 5], device=DEV)))
    with pytest.raises(RuntimeError, match="already leased"):
        cache.resolve("a", 0, LogicalTopK(torch.tensor([1], device=DEV)))
    lease.release()
    with pytest.raises(RuntimeError, match="released"):
        lease.release()
    with pytest.raises(ValueError, match="max_union_rows"):
        cache.resolve("a", 0, LogicalTopK(torch.arange(5, device=DEV)))


def _build(seed, requests, layers, length, p, hkv, d, hot_rows, resident_fraction, dtype):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    n = math.ceil(length / p)
    hot = HotConfig(hot_rows // 2, hot_rows)
    hot_blocks = hot.hot_blocks(p)
    resident_pages = max(2, int(n * resident_fraction))
    gpu_pages = requests * layers * (resident_pages + hot_blocks)
    config = CacheConfig(gpu_pages=gpu_pages, host_pages=requests * layers * n, page_size=p,
                         kv_heads=hkv, head_dim=d, device=DEV, dtype=dtype)
    host = torch.randn(config.host_pages, 2, p, hkv, d, generator=gen).to(dtype)
    placement, meta = {}, {}
    next_block = 0
    for r in range(requests):
        mins, maxs = [], []
        for layer in range(layers):
            base = (r * layers + layer) * n
            source = np.arange(base, base + n)
            chosen = set(rng.choice(n - 2, size=resident_pages - 2, replace=False).tolist())
            chosen |= {n - 2, n - 1}
            resident = np.full(n, -1)
            for pg in sorted(chosen):
                resident[pg] = next_block
                next_block += 1
            hot_list = list(range(next_block, next_block + hot_blocks))
            next_block += hot_blocks
            placement[r, layer] = (source, resident, hot_list)
            keys = host[base:base + n, 0].float()  # [n, P, Hkv, D]
            mins.append(keys.amin(1).to(dtype))
            maxs.append(keys.amax(1).to(dtype))
        meta[r] = (torch.stack(mins), torch.stack(maxs))
    return config, hot, host, placement, meta


def _cache(config, hot, host, placement, length):
    cache = RowCache(config, hot, host=host.pin_memory())
    cache.pool.zero_()
    for (r, layer), (source, resident, hot_list) in placement.items():
        cache.add_layer(r, layer, length, source, resident, hot_list)
        for pg in np.nonzero(resident >= 0)[0]:
            cache.pool[int(resident[pg])] = host[int(source[pg])].to(DEV)
    return cache


def test_decode_batch_matches_per_request_api():
    b, layers, length, p, hkv, d, hq, top = 3, 2, 2000, 16, 8, 128, 32, 16
    args = _build(0, b, layers, length, p, hkv, d, 512, 0.25, torch.bfloat16)
    config, hot, host, placement, meta = args
    cache_a = _cache(config, hot, host, placement, length)
    cache_b = _cache(config, hot, host, placement, length)
    mins = {r: meta[r][0].to(DEV) for r in range(b)}
    maxs = {r: meta[r][1].to(DEV) for r in range(b)}
    batch = DecodeBatch(cache_a, list(range(b)), layers, mins, maxs, top, hq)
    gen = torch.Generator().manual_seed(9)
    for step in range(3):
        for layer in range(layers):
            q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16).to(DEV)
            out = batch.layer(layer, q)
            for r in range(b):
                sel = quest_selection(q[r], mins[r][layer], maxs[r][layer], length, p, top)
                single = cache_b.attention(q[r], r, layer, sel)
                torch.testing.assert_close(out[r], single, **TOL[torch.bfloat16])
                ta, tb = cache_a.tables[r, layer], cache_b.tables[r, layer]
                assert torch.equal(ta.tags, tb.tags) and torch.equal(ta.lru, tb.lru)
    assert not _lib.device_flags(DEV)


def test_decode_batch_against_oracle_full_step():
    """One layer of configuration-2 shape (4 requests) against the oracle's
    whole-path restatement: selection, plans, gathered rows and outputs."""
    b, length, p, hkv, d, hq, top = 4, 32768, 16, 8, 128, 32, 128
    config, hot, host, placement, meta = _build(1, b, 1, length, p, hkv, d, 4096, 0.25,
                                                torch.bfloat16)
    cache = _cache(config, hot, host, placement, length)
    mins = {r: meta[r][0].to(DEV) for r in range(b)}
    maxs = {r: meta[r][1].to(DEV) for r in range(b)}
    batch = DecodeBatch(cache, list(range(b)), 1, mins, maxs, top, hq)
    pool_cpu = cache.pool.cpu()
    tags = [cache.tables[r, 0].tags.cpu().numpy().astype(np.int64) for r in range(b)]
    lrus = [cache.tables[r, 0].lru.cpu().numpy().copy() for r in range(b)]
    gen = torch.Generator().manual_seed(3)
    for step in range(2):
        q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16)
        out = batch.layer(0, q.to(DEV)).cpu()
        outs, counts = oracle.decode_layer_batched(
            [q[r] for r in range(b)], [meta[r][0][0] for r in range(b)],
            [meta[r][1][0] for r in range(b)], [length] * b, p, top, meta[0][0].shape[1],
            [placement[r, 0][0] for r in range(b)], [placement[r, 0][1] for r in range(b)],
            [np.array(placement[r, 0][2]) for r in range(b)], tags, lrus, host, pool_cpu)
        for r in range(b):
            torch.testing.assert_close(out[r].double(), torch.from_numpy(outs[r]),
                                       **TOL[torch.bfloat16])
            assert cache.tables[r, 0].tags.tolist() == tags[r].tolist()
            assert cache.tables[r, 0].lru.tolist() == lrus[r].tolist()
        assert batch.last_counts()[0].tolist() == counts.tolist()
    assert torch.equal(cache.pool.cpu(), pool_cpu)


def test_decode_batch_with_external_positions_matches_quest_path():
    """layer(positions=...) resolves a given selection instead of running Quest:
    fed the tokens Quest chose, it leaves the same outputs, counts, tags and LRU
    as the Quest path; bad shapes are rejected."""
    b, length, p, hkv, d, hq, top = 3, 4000, 16, 8, 128, 32, 16
    config, hot, host, placement, meta = _build(4, b, 1, length, p, hkv, d, 512, 0.25,
                                                torch.bfloat16)
    cache_a = _cache(config, hot, host, placement, length)
    cache_b = _cache(config, hot, host, placement, length)
    mins = {r: meta[r][0].to(DEV) for r in range(b)}
    maxs = {r: meta[r][1].to(DEV) for r in range(b)}
    batch_a = DecodeBatch(cache_a, list(range(b)), 1, mins, maxs, top, hq)
    batch_b = DecodeBatch(cache_b, list(range(b)), 1, mins, maxs, top, hq)
    gen = torch.Generator().manual_seed(5)
    for step in range(3):
        q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16).to(DEV)
        out_a = batch_a.layer(0, q).clone()
        tokens = batch_a.tokens.clone()
        out_b = batch_b.layer(0, q, positions=tokens).clone()
        assert torch.equal(out_a, out_b)
        assert torch.equal(batch_a.last_counts(), batch_b.last_counts())
        for r in range(b):
            ta, tb = cache_a.tables[r, 0], cache_b.tables[r, 0]
            assert torch.equal(ta.tags, tb.tags) and torch.equal(ta.lru, tb.lru)
    with pytest.raises(ValueError, match="positions"):
        batch_b.layer(0, q, positions=tokens[:, :-1].contiguous())
    with pytest.raises(ValueError, match="positions"):
        batch_b.layer(0, q, positions=tokens.long())
    assert not _lib.device_flags(DEV)


@pytest.mark.parametrize("segmented", [False, True])
def test_decode_graph_replay_matches_eager_steps(segmented):
    """A whole step captured as a CUDA graph (two micro-batches on their own
    streams) gives the same outputs, counts and tables as eager DecodeBatch
    calls on an identical cache; so does the segmented capture (each layer
    as two graphs split where a head-sharded batch exchanges its scores)."""
    from hisparse_b200.batched import DecodeGraph

    b, layers, length, p, hkv, d, hq, top = 4, 2, 3000, 16, 8, 128, 32, 16
    config, hot, host, placement, meta = _build(5, b, layers, length, p, hkv, d, 512, 0.25,
                                                torch.bfloat16)
    caches = [_cache(config, hot, host, placement, length) for _ in range(2)]
    mins = {r: meta[r][0].to(DEV) for r in range(b)}
    maxs = {r: meta[r][1].to(DEV) for r in range(b)}
    groups = [[0, 2], [1, 3]]

    def batches(cache):
        out = []
        for g in groups:
            streams = (torch.cuda.Stream(), torch.cuda.Stream())
            with torch.cuda.stream(streams[0]):
                out.append(DecodeBatch(cache, g, layers, {r: mins[r] for r in g},
                                       {r: maxs[r] for r in g}, top, hq, streams=streams))
        return out

    eager, captured = batches(caches[0]), batches(caches[1])
    # runs two eager warm-up steps on caches[1]; gather launches timed inside the graph
    graph = DecodeGraph(captured, layers, timing=False if segmented else ("gather",),
                        segmented=segmented)
    assert graph.segmented == segmented
    gen = torch.Generator().manual_seed(11)
    warm = [torch.randn(layers, b, hq, d, generator=gen).to(torch.bfloat16) for _ in range(2)]
    steps = [torch.randn(layers, b, hq, d, generator=gen).to(torch.bfloat16) for _ in range(3)]
    torch.cuda.synchronize()

    def eager_step(q):
        outs = []
        for layer in range(layers):
            for i, bt in enumerate(eager):
                with torch.cuda.stream(bt.compute):
                    outs.append((i, layer, bt.layer(layer, q[layer][groups[i]].to(DEV).contiguous())))
        torch.cuda.synchronize()
        return outs

    # the graph's warm-up used zero queries: replay them on the eager side too
    zeros = torch.zeros(layers, b, hq, d, dtype=torch.bfloat16)
    for _ in range(2):
        eager_step(zeros)
    for q in steps:
        ref = eager_step(q)
        for i, g in enumerate(groups):
            graph.queries[i].copy_(q[:, g].to(DEV))
        graph.replay()
        torch.cuda.synchronize()
        for i, layer, out in ref:
            assert torch.equal(graph.outputs[i][layer], out)
        if not segmented:
            assert len(graph.timing) == layers * len(groups)
            assert all(name == "gather" and a.elapsed_time(b_) >= 0
                       for name, a, b_ in graph.timing)
    for key in caches[0].tables:
        assert torch.equal(caches[0].tables[key].tags, caches[1].tables[key].tags)
        assert torch.equal(caches[0].tables[key].lru, caches[1].tables[key].lru)
    assert torch.equal(caches[0].pool, caches[1].pool)
    del warm
    assert not _lib.device_flags(DEV)
