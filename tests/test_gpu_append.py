"""KV append kernel (pool rows, host mirror, K min/max, mean-K summary) vs the
reference's recorded HostStore.append chunks and the oracle."""

import numpy as np
import pytest
import torch

import oracle
from hisparse_b200 import CacheConfig, MappedHost, _lib
from hisparse_b200.append import append_chunks, append_page

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _config(block, dtype):
    _, p, hkv, d = block.shape
    return CacheConfig(gpu_pages=1, host_pages=1, page_size=p, kv_heads=hkv, head_dim=d,
                       device=DEV, dtype=dtype)


def _records(golden):
    for case in golden("append_cases"):
        for record in case["records"]:
            yield case["name"], record["chunks"]


def test_batched_append_matches_reference_chunks(golden):
    """All chunks of one recorded HostStore.append in one batched launch (each
    chunk on its own block): pool, host mirror, min/max and summary equal the
    reference's bit for bit."""
    for name, chunks in _records(golden):
        n, dtype = len(chunks), chunks[0]["k"].dtype
        config = _config(chunks[0]["block_before"], dtype)
        pool = torch.stack([c["block_before"] for c in chunks]).to(DEV)
        host = torch.stack([c["host_before"] for c in chunks]).pin_memory()
        mn = torch.stack([c["min_before"] for c in chunks]).to(DEV)
        mx = torch.stack([c["max_before"] for c in chunks]).to(DEV)
        sm = torch.stack([c["summary_before"] for c in chunks]).to(DEV)
        t = max(c["count"] for c in chunks)
        k = torch.zeros((n, t, config.kv_heads, config.head_dim), dtype=dtype)
        v = torch.zeros_like(k)
        for i, c in enumerate(chunks):
            k[i, :c["count"]], v[i, :c["count"]] = c["k"], c["v"]
        within = torch.tensor([c["within"] for c in chunks], dtype=torch.int32, device=DEV)
        count = torch.tensor([c["count"] for c in chunks], dtype=torch.int32, device=DEV)
        blocks = torch.arange(n, dtype=torch.int64, device=DEV)

        def ptrs(t_):
            return torch.tensor([t_[i].data_ptr() for i in range(n)], dtype=torch.int64,
                                device=DEV)

        append_chunks(k.to(DEV), v.to(DEV), within, count, blocks, pool, ptrs(mn), ptrs(mx),
                      ptrs(sm), config, MappedHost(host), blocks.clone())
        torch.cuda.synchronize()
        for i, c in enumerate(chunks):
            assert torch.equal(pool[i].cpu().view(torch.uint8),
                               c["block_after"].view(torch.uint8)), name
            assert torch.equal(host[i].view(torch.uint8), c["host_after"].view(torch.uint8)), name
            assert torch.equal(mn[i].cpu(), c["min_after"]), name
            assert torch.equal(mx[i].cpu(), c["max_after"]), name
            assert torch.equal(sm[i].cpu(), c["summary_after"]), name
    assert not _lib.device_flags(DEV)


def test_append_page_replays_reference_sessions_in_order(golden):
    """The one-chunk form, chunk after chunk as HostStore.append issued them,
    on a pool/host holding the recorded slots."""
    for name, chunks in _records(golden):
        dtype = chunks[0]["k"].dtype
        config = _config(chunks[0]["block_before"], dtype)
        for c in chunks:
            pool = c["block_before"].unsqueeze(0).to(DEV)
            host = c["host_before"].unsqueeze(0).pin_memory()
            mn, mx = c["min_before"].to(DEV), c["max_before"].to(DEV)
            sm = c["summary_before"].to(DEV)
            append_page(pool, c["k"].to(DEV), c["v"].to(DEV), 0, c["within"], mn, mx, sm,
                        config, MappedHost(host), 0)
            torch.cuda.synchronize()
            assert torch.equal(pool[0].cpu().view(torch.uint8),
                               c["block_after"].view(torch.uint8)), name
            assert torch.equal(host[0].view(torch.uint8), c["host_after"].view(torch.uint8))
            assert torch.equal(mn.cpu(), c["min_after"]) and torch.equal(mx.cpu(), c["max_after"])
            assert torch.equal(sm.cpu(), c["summary_after"]), name


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_decode_append_batch_matches_oracle(dtype):
    """A decode step's append at configuration 2's shape: one token for each of
    16 requests, at random offsets of their tail pages, no mirror for some."""
    gen = torch.Generator().manual_seed(21)
    b, p, hkv, d, blocks = 16, 16, 8, 128, 64
    config = CacheConfig(gpu_pages=blocks, host_pages=blocks, page_size=p, kv_heads=hkv,
                         head_dim=d, device=DEV, dtype=dtype)
    pool_cpu = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(dtype)
    host_cpu = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(dtype)
    slots = torch.randperm(blocks, generator=gen)[:b]
    host_slots = torch.randperm(blocks, generator=gen)[:b]
    host_slots[::5] = -1
    within = torch.randint(0, p, (b,), generator=gen)
    k = torch.randn(b, 1, hkv, d, generator=gen).to(dtype)
    v = torch.randn(b, 1, hkv, d, generator=gen).to(dtype)
    mn_cpu = torch.randn(b, hkv, d, generator=gen).to(dtype)
    mx_cpu = (mn_cpu.float() + 1).to(dtype)
    sm_cpu = torch.randn(b, hkv, d, generator=gen)
    pool, host = pool_cpu.to(DEV), host_cpu.pin_memory()
    mn, mx, sm = mn_cpu.to(DEV), mx_cpu.to(DEV), sm_cpu.to(DEV)
    ptrs = [torch.tensor([t[i].data_ptr() for i in range(b)], dtype=torch.int64, device=DEV)
            for t in (mn, mx, sm)]
    append_chunks(k.to(DEV), v.to(DEV), within.to(torch.int32).to(DEV),
                  torch.ones(b, dtype=torch.int32, device=DEV), slots.to(DEV), pool, *ptrs,
                  config, MappedHost(host), host_slots.to(DEV))
    torch.cuda.synchronize()
    for i in range(b):
        s, h, w = int(slots[i]), int(host_slots[i]), int(within[i])
        blk, hst, omn, omx, osm = oracle.append_rows(
            k[i], v[i], w, pool_cpu[s], None if h < 0 else host_cpu[h], mn_cpu[i], mx_cpu[i],
            sm_cpu[i].numpy())
        assert np.array_equal(oracle.as_array(pool[s].cpu())[0], blk)
        if h >= 0:
            assert np.array_equal(oracle.as_array(host[h])[0], hst)
        assert np.array_equal(oracle.as_array(mn[i].cpu())[0], omn)
        assert np.array_equal(oracle.as_array(mx[i].cpu())[0], omx)
        assert np.array_equal(sm[i].cpu().numpy(), osm)
    untouched = set(range(blocks)) - {int(x) for x in host_slots if x >= 0}
    for h in list(untouched)[:8]:
        assert torch.equal(host[h], host_cpu[h])
    assert not _lib.device_flags(DEV)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_host_only_chunks_match_oracle(dtype):
    """Chunks of pages that hold no pool block (pool_block -1): the rows go to
    the host block only and the mean reads the page's earlier rows there;
    pooled chunks of the same launch are unaffected, and a chunk with neither
    block is skipped and flagged."""
    gen = torch.Generator().manual_seed(23)
    b, p, hkv, d, blocks = 12, 16, 2, 64, 32
    config = CacheConfig(gpu_pages=blocks, host_pages=blocks, page_size=p, kv_heads=hkv,
                         head_dim=d, device=DEV, dtype=dtype)
    pool_cpu = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(dtype)
    host_cpu = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(dtype)
    slots = torch.randperm(blocks, generator=gen)[:b]
    slots[::2] = -1
    host_slots = torch.randperm(blocks, generator=gen)[:b]
    within = torch.randint(0, p - 3, (b,), generator=gen)
    count = torch.randint(1, 4, (b,), generator=gen)
    k = torch.randn(b, 3, hkv, d, generator=gen).to(dtype)
    v = torch.randn(b, 3, hkv, d, generator=gen).to(dtype)
    mn_cpu = torch.full((b, hkv, d), float("inf")).to(dtype)
    mx_cpu = torch.full((b, hkv, d), float("-inf")).to(dtype)
    sm_cpu = torch.zeros(b, hkv, d)
    pool, host = pool_cpu.to(DEV), host_cpu.pin_memory()
    mn, mx, sm = mn_cpu.to(DEV), mx_cpu.to(DEV), sm_cpu.to(DEV)
    ptrs = [torch.tensor([t[i].data_ptr() for i in range(b)], dtype=torch.int64, device=DEV)
            for t in (mn, mx, sm)]
    append_chunks(k.to(DEV), v.to(DEV), within.to(torch.int32).to(DEV),
                  count.to(torch.int32).to(DEV), slots.to(DEV), pool, *ptrs, config,
                  MappedHost(host), host_slots.to(DEV))
    torch.cuda.synchronize()
    for i in range(b):
        s, h, w, c = int(slots[i]), int(host_slots[i]), int(within[i]), int(count[i])
        blk, hst, omn, omx, osm = oracle.append_rows(
            k[i, :c], v[i, :c], w, None if s < 0 else pool_cpu[s], host_cpu[h], mn_cpu[i],
            mx_cpu[i], sm_cpu[i].numpy())
        if s >= 0:
            assert np.array_equal(oracle.as_array(pool[s].cpu())[0], blk)
        assert np.array_equal(oracle.as_array(host[h])[0], hst)
        assert np.array_equal(oracle.as_array(mn[i].cpu())[0], omn)
        assert np.array_equal(oracle.as_array(mx[i].cpu())[0], omx)
        assert np.array_equal(sm[i].cpu().numpy(), osm)
    untouched = set(range(blocks)) - {int(x) for x in slots if x >= 0}
    for s in untouched:
        assert torch.equal(pool[s].cpu(), pool_cpu[s])
    assert not _lib.device_flags(DEV)
    # neither a pool nor a host block: skipped, flagged, nothing written
    before = mn.clone()
    append_chunks(k[:1].to(DEV), v[:1].to(DEV), torch.zeros(1, dtype=torch.int32, device=DEV),
                  torch.ones(1, dtype=torch.int32, device=DEV),
                  torch.tensor([-1], dtype=torch.int64, device=DEV), pool,
                  *[t[:1] for t in ptrs], config, MappedHost(host),
                  torch.tensor([-1], dtype=torch.int64, device=DEV))
    torch.cuda.synchronize()
    assert _lib.device_flags(DEV) == [_lib.DEVICE_FLAGS[1]]
    assert torch.equal(mn, before)


def test_append_rejects_chunks_leaving_their_page():
    config = CacheConfig(gpu_pages=2, host_pages=2, page_size=4, kv_heads=1, head_dim=8,
                         device=DEV, dtype=torch.float32)
    pool = torch.zeros(2, 2, 4, 1, 8, device=DEV)
    meta = [torch.zeros(1, 8, device=DEV) for _ in range(3)]
    with pytest.raises(ValueError):
        append_page(pool, torch.ones(2, 1, 8, device=DEV), torch.ones(2, 1, 8, device=DEV), 0, 3,
                    *meta, config)
    # a chunk past its page in the batched form is skipped on the device and flagged
    ptrs = [torch.tensor([m.data_ptr()], dtype=torch.int64, device=DEV) for m in meta]
    append_chunks(torch.ones(1, 2, 1, 8, device=DEV), torch.ones(1, 2, 1, 8, device=DEV),
                  torch.tensor([3], dtype=torch.int32, device=DEV),
                  torch.tensor([2], dtype=torch.int32, device=DEV),
                  torch.tensor([0], dtype=torch.int64, device=DEV), pool, *ptrs, config)
    torch.cuda.synchronize()
    assert _lib.device_flags(DEV) == [_lib.DEVICE_FLAGS[1]]
    assert torch.count_nonzero(pool) == 0
