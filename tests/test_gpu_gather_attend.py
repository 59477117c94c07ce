"""Miss gather and row attention kernels vs the reference's recorded results and
the oracle; the recorded cache sessions replayed call by call."""

import numpy as np
import pytest
import torch

import oracle
from helpers import TOL, raw_numpy, rebuild_host, same_bytes
from hisparse_b200 import (CacheConfig, LogicalTopK, MappedHost, RowPlan, _lib, attend_rows,
                           gather_rows, resolve_rows)
from hisparse_b200.row_kernels import attend_into

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _config(pool):
    _, _, p, hkv, d = pool.shape
    return CacheConfig(gpu_pages=pool.shape[0], host_pages=1, page_size=p, kv_heads=hkv,
                       head_dim=d, device=DEV, dtype=pool.dtype)


def test_attention_reference_fixtures(golden):
    for case in golden("attention_cases"):
        pool = case["pool"].to(DEV)
        rows = case["rows"].to(DEV)
        out = attend_rows(case["query"].to(DEV), pool, rows, _config(pool))
        torch.testing.assert_close(out.cpu().double(), case["out"].double(),
                                   **TOL[case["query"].dtype], msg=case["name"])
        ref = oracle.attend_rows(case["query"], case["pool"], case["rows"].numpy(),
                                 case["page_size"])
        torch.testing.assert_close(out.cpu().double(), torch.from_numpy(ref),
                                   **TOL[case["query"].dtype], msg=case["name"])
    assert not _lib.device_flags(DEV)


def test_scenarios_replay_call_by_call(golden):
    """Each resolve/gather/attention call HybridKVCache made in the recorded
    sessions (restating the reference's cache tests and trace replays)."""
    for scenario in golden("scenarios"):
        totals = torch.zeros(3, dtype=torch.int64)
        for i, rec in enumerate(scenario["records"]):
            tag = f"{scenario['name']}[{i}]"
            t = {k: rec[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
            cols = None if rec["head_columns"] is None else rec["head_columns"].to(DEV)
            plan = resolve_rows(LogicalTopK(rec["positions"].to(DEV), cols), t["source"],
                                t["resident"], t["hot"], t["tags"], t["lru"], rec["length"],
                                rec["page_size"])
            assert plan.physical_rows.tolist() == rec["physical"].tolist(), tag
            assert plan.miss_host_rows.tolist() == rec["miss_host"].tolist(), tag
            assert plan.miss_device_rows.tolist() == rec["miss_device"].tolist(), tag
            assert plan.counts.tolist() == rec["counts"].tolist(), tag
            assert t["tags"].tolist() == rec["tags_after"].tolist(), tag
            assert t["lru"].tolist() == rec["lru_after"].tolist(), tag
            totals += plan.counts.cpu()
            host = rebuild_host(rec).pin_memory()
            pool = rec["pool_before"].to(DEV)
            config = _config(pool)
            gather_rows(MappedHost(host), pool, plan, config)
            assert same_bytes(raw_numpy(pool.cpu()), raw_numpy(rec["pool_after"])), tag
            q = rec["query"].to(DEV)
            out = attend_rows(q, pool, plan.physical_rows, config)
            torch.testing.assert_close(out.cpu().double(), rec["out"].double(),
                                       **TOL[q.dtype], msg=tag)
        stats = scenario["row_stats"]
        assert totals.tolist() == [stats["resident_hits"], stats["hot_hits"], stats["misses"]]
    assert not _lib.device_flags(DEV)


@pytest.mark.parametrize("dtype,p,hkv,d", [
    (torch.bfloat16, 16, 8, 128),  # 2 KiB rows: 16-byte vectors
    (torch.float32, 4, 1, 8),      # 32 B rows
    (torch.float16, 7, 2, 24),     # 96 B rows
    (torch.float16, 3, 1, 3),      # 6 B rows: 2-byte copies
    (torch.bfloat16, 64, 4, 128),  # configuration 5 rows
])
def test_gather_against_oracle(dtype, p, hkv, d):
    rng = np.random.default_rng(p * 31 + d)
    host_blocks, pool_blocks, count = 97, 53, 300
    gen = torch.Generator().manual_seed(7)
    host = torch.randn(host_blocks, 2, p, hkv, d, generator=gen).to(dtype).pin_memory()
    pool = torch.randn(pool_blocks, 2, p, hkv, d, generator=gen).to(dtype)
    misses = min(count, pool_blocks * p)
    mh = np.full(count, -1, dtype=np.int64)
    md = np.full(count, -1, dtype=np.int64)
    used = misses - 17
    mh[:used] = rng.choice(host_blocks * p, size=used, replace=False)
    md[:used] = rng.choice(pool_blocks * p, size=used, replace=False)
    expected = raw_numpy(pool)
    oracle.gather_rows(raw_numpy(host), expected, mh, md, p)
    dpool = pool.to(DEV)
    plan = RowPlan(None, torch.tensor(mh, device=DEV), torch.tensor(md, device=DEV), None)
    gather_rows(MappedHost(host), dpool, plan, _config(dpool))
    assert same_bytes(raw_numpy(dpool.cpu()), expected)
    assert not _lib.device_flags(DEV)


def test_gather_skips_and_flags_out_of_range_rows():
    host = torch.randn(4, 2, 4, 1, 8).pin_memory()
    pool = torch.zeros(2, 2, 4, 1, 8, device=DEV)
    plan = RowPlan(None, torch.tensor([1, 100, 2], device=DEV), torch.tensor([0, 1, 50],
                                                                            device=DEV), None)
    gather_rows(MappedHost(host), pool, plan, _config(pool))
    flags = _lib.device_flags(DEV)
    assert flags and "beyond" in flags[0]
    assert torch.equal(pool[0, :, 0].cpu(), host[0, :, 1])
    assert pool[0, :, 1:].abs().sum().item() == 0 and pool[1].abs().sum().item() == 0


def test_mapped_host_requires_pinned_memory():
    with pytest.raises(ValueError, match="pinned"):
        MappedHost(torch.zeros(4))


@pytest.mark.parametrize("hq,hkv,d,p,k,dtype", [
    (32, 8, 128, 16, 2048, torch.bfloat16),   # configuration 2
    (32, 8, 128, 64, 4096, torch.bfloat16),   # configuration 3
    (28, 4, 128, 64, 8192, torch.bfloat16),   # configuration 5
    (8, 2, 32, 16, 64, torch.float32),        # configuration 1
    (6, 2, 24, 7, 33, torch.float16),
    (12, 1, 256, 4, 100, torch.bfloat16),     # group of 12 (> 8 heads per CTA), head_dim 256
])
def test_attention_full_size_against_oracle(hq, hkv, d, p, k, dtype):
    gen = torch.Generator().manual_seed(k + d)
    blocks = (k + p - 1) // p + 16
    pool = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(dtype)
    q = torch.randn(hq, d, generator=gen).to(dtype)
    rows = torch.randperm(blocks * p, generator=gen)[:k]
    rows[torch.rand(k, generator=gen) < 0.1] = -1
    out = attend_rows(q.to(DEV), pool.to(DEV), rows.to(DEV), _config(pool))
    ref = oracle.attend_rows(q, pool, rows.numpy(), p)
    torch.testing.assert_close(out.cpu().double(), torch.from_numpy(ref), **TOL[dtype])


def test_attention_batched_matches_single():
    gen = torch.Generator().manual_seed(4)
    b, hq, hkv, d, p, k = 6, 32, 8, 128, 16, 1024
    pool = torch.randn(200, 2, p, hkv, d, generator=gen).to(torch.bfloat16).to(DEV)
    q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16).to(DEV)
    rows = torch.stack([torch.randperm(200 * p, generator=gen)[:k] for _ in range(b)]).to(DEV)
    rows[:, ::7] = -1
    out = torch.empty_like(q)
    attend_into(out, q, pool, rows[:, None, :].expand(b, hq, k), _config(pool), batch=b)
    for i in range(b):
        single = attend_rows(q[i], pool, rows[i], _config(pool))
        torch.testing.assert_close(out[i], single, **TOL[torch.bfloat16])


def test_attention_all_rows_invalid_gives_zeros():
    pool = torch.randn(3, 2, 4, 1, 8, device=DEV)
    out = attend_rows(torch.randn(2, 8, device=DEV), pool, torch.full((4,), -1, device=DEV),
                      _config(pool))
    assert out.abs().sum().item() == 0


def _phase_attention(q, pool, counts, phases):
    """hs_attend_rows_phase over the leading valid rows of each phase's rows
    ([B, K]) selected by a (first, n) component range of `counts` ([B, 3]),
    then hs_attend_merge."""
    lib = _lib.load()
    b, hq, d = q.shape
    _, _, p, hkv, _ = pool.shape
    k = phases[0][0].shape[1]
    out = torch.empty_like(q)
    nbytes = lib.hs_attend_workspace_bytes(b, hq, hkv, d, k)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    status, stream = _lib.status_word(DEV).data_ptr(), torch.cuda.current_stream().cuda_stream
    code = _lib.dtype_code(q.dtype)
    for phase, (r, first, n) in enumerate(phases):
        _lib.check(lib.hs_attend_rows_phase(
            b, q.data_ptr(), hq * d, code, pool.data_ptr(), pool.shape[0], code, r.data_ptr(),
            k, k, counts.data_ptr(), 3, first, n, phase, hq, hkv, d, p, ws.data_ptr(), nbytes,
            status, stream))
    _lib.check(lib.hs_attend_merge(b, len(phases), out.data_ptr(), hq * d, code, hq, hkv, d, k,
                                   ws.data_ptr(), nbytes, status, stream))
    return out


@pytest.mark.parametrize("hq,hkv,b,k", [
    (32, 8, 8, 2048),    # configuration 2 shape, 8 requests of a micro-batch
    (28, 4, 1, 8192),    # configuration 5 on one GPU
    (14, 2, 1, 8192),    # configuration 5, heads split over 2 ranks
    (7, 1, 1, 8192),     # configuration 5, heads split over 4 ranks
    (32, 8, 64, 512),    # a wide batch
    (8, 8, 5, 300),      # one query head per KV head
    (16, 2, 3, 1000),    # eight query heads per KV head
])
def test_attention_two_phase_uneven_requests(hq, hkv, b, k):
    """The two-phase attention (ready rows, then gathered rows, then the merge)
    over requests with uneven, empty and full valid counts, rows both in whole
    pages (consecutive pool rows) and scattered: every request's output equals
    the oracle's attention over its valid rows of both phases."""
    gen = torch.Generator().manual_seed(hq * 100 + b)
    d, p = 128, 16
    blocks = 4 * k // p + 8
    pool = torch.randn(blocks, 2, p, hkv, d, generator=gen).to(torch.bfloat16)
    q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16)

    def rows_like_a_selection():
        # whole pages (runs of consecutive rows) for the first half, single rows after
        pages = torch.randperm(blocks, generator=gen)[:k // (2 * p) + 1]
        runs = (pages[:, None] * p + torch.arange(p)).reshape(-1)[:k // 2]
        single = torch.randperm(blocks * p, generator=gen)[:k - runs.numel()]
        return torch.cat([runs, single])

    ready = torch.stack([rows_like_a_selection() for _ in range(b)])
    missed = torch.stack([torch.randperm(blocks * p, generator=gen)[:k] for _ in range(b)])
    counts = torch.zeros(b, 3, dtype=torch.int64)
    for i in range(b):
        kind = i % 4
        r_hits = [k, 0, k // 3, 1][kind] if b > 1 else k * 3 // 4
        misses = [0, k, k // 5, k - 1][kind] if b > 1 else k // 4
        counts[i] = torch.tensor([r_hits // 2, r_hits - r_hits // 2, misses])
    if b > 2:
        counts[2] = 0                      # an empty request
    ready[0, 3] = -1                        # a skipped row inside the valid range
    dq, dpool = q.to(DEV), pool.to(DEV)
    dready, dmissed, dcounts = ready.to(DEV), missed.to(DEV), counts.to(DEV)
    out = _phase_attention(dq, dpool, dcounts, [(dready, 0, 2), (dmissed, 2, 1)])
    for i in range(b):
        nr, nm = int(counts[i, :2].sum()), int(counts[i, 2])
        rows = torch.cat([ready[i, :nr], missed[i, :nm]])
        if rows.numel() == 0 or (rows < 0).all():
            assert out[i].abs().sum().item() == 0, i
            continue
        ref = oracle.attend_rows(q[i], pool, rows.numpy(), p)
        torch.testing.assert_close(out[i].cpu().double(), torch.from_numpy(ref),
                                   **TOL[torch.bfloat16], msg=f"request {i}")
    assert not _lib.device_flags(DEV)
