"""Row resolver kernel vs the reference's recorded results and the oracle."""

import math

import numpy as np
import pytest
import torch

import oracle
from hisparse_b200 import LogicalTopK, _lib, resolve_rows

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _run(case, dtype=None):
    t = {k: case[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
    if dtype is not None:
        t = {k: v.to(dtype) if k != "lru" else v for k, v in t.items()}
    pos = case["positions"].to(DEV)
    plan = resolve_rows(LogicalTopK(pos), t["source"], t["resident"], t["hot"], t["tags"],
                        t["lru"], case["length"], case["page_size"])
    return plan, t


def test_reference_fixtures_bit_exact(golden):
    for case in golden("resolver_cases"):
        plan, t = _run(case)
        name = case["name"]
        assert plan.physical_rows.tolist() == case["physical"].tolist(), name
        assert plan.miss_host_rows.tolist() == case["miss_host"].tolist(), name
        assert plan.miss_device_rows.tolist() == case["miss_device"].tolist(), name
        assert plan.counts.tolist() == case["counts"].tolist(), name
        assert t["tags"].tolist() == case["tags_after"].tolist(), name
        assert t["lru"].tolist() == case["lru_after"].tolist(), name
    assert not _lib.device_flags(DEV)


def test_int64_tables_are_updated_in_place(golden):
    case = golden("resolver_cases")[0]  # the known-answer vector uses int64 tables
    assert case["tags"].dtype == torch.int64
    plan, t = _run(case)
    assert t["tags"].dtype == torch.int64 and t["tags"][0].item() == 37
    assert plan.physical_rows.tolist() == [24, 5, 30, -1, 14, -1]


def _random_case(rng, k, h, p, length, resident_fraction=0.25, tag_fraction=0.6):
    n = math.ceil(length / p)
    source = rng.choice(max(4 * n, 64), size=n, replace=False).astype(np.int64)
    if n > 4:
        source[rng.choice(n - 2, size=max(1, n // 64), replace=False)] = -1
    hot_blocks = math.ceil(h / p)
    blocks = rng.permutation(hot_blocks + n + 8)
    hot = blocks[:hot_blocks]
    resident = np.full(n, -1, dtype=np.int64)
    rp = rng.choice(n, size=int(n * resident_fraction), replace=False)
    resident[rp] = blocks[hot_blocks:hot_blocks + len(rp)]
    pages = rng.choice(n, size=min(n, max(1, k // p)), replace=False)
    pos = (pages[:, None] * p + np.arange(p)).reshape(-1)[:k]
    pos = np.concatenate([pos, rng.integers(-2, length + 3, size=k - len(pos))])
    pos = rng.permutation(pos)
    wanted = [int(source[t // p]) * p + t % p for t in pos
              if 0 <= t < length and source[t // p] >= 0 and resident[t // p] < 0]
    wanted = list(dict.fromkeys(wanted))
    rng.shuffle(wanted)
    n_tags = int(h * tag_fraction)
    pool = list(dict.fromkeys(wanted[: n_tags // 2] +
                              rng.choice(max(4 * n, 64) * p, size=n_tags).tolist()))[:n_tags]
    tags = np.full(h, -1, dtype=np.int64)
    tags[rng.choice(h, size=len(pool), replace=False)] = pool
    lru = rng.permutation(h).astype(np.int64)
    return dict(positions=torch.tensor(pos, dtype=torch.int32), source=torch.tensor(source),
                resident=torch.tensor(resident), hot=torch.tensor(hot),
                tags=torch.tensor(tags), lru=torch.tensor(lru), length=length, page_size=p)


@pytest.mark.parametrize("k,h,p,length", [
    (2048, 4096, 16, 32768),     # configuration 2 (Llama-3-8B shape, 32k context)
    (4096, 8192, 16, 131072),    # configuration 3, page 16
    (4096, 8192, 64, 131072),    # configuration 3, page 64
    (8192, 16384, 64, 1048576),  # configuration 5 (1M tokens)
    (32768, 32768, 16, 600000),  # maximum hot_rows; scratch in global workspace
    (1, 1, 1, 1), (7, 9, 3, 20),
])
def test_full_size_against_oracle(k, h, p, length):
    rng = np.random.default_rng(k * 7 + h)
    case = _random_case(rng, k, h, p, length)
    for dtype in (torch.int32, torch.int64):
        plan, t = _run(case, dtype)
        ref = oracle.resolve_rows(case["positions"].numpy(), case["source"].numpy(),
                                  case["resident"].numpy(), case["hot"].numpy(),
                                  case["tags"].numpy(), case["lru"].numpy(), length, p)
        assert plan.physical_rows.cpu().numpy().tolist() == ref["physical"].tolist()
        assert plan.miss_host_rows.tolist() == ref["miss_host"].tolist()
        assert plan.miss_device_rows.tolist() == ref["miss_device"].tolist()
        assert plan.counts.tolist() == ref["counts"].tolist()
        assert t["tags"].tolist() == ref["tags"].tolist()
        assert t["lru"].tolist() == ref["lru"].tolist()
    assert not _lib.device_flags(DEV)


def test_repeated_calls_chain_tables():
    """Two steps in a row: the second sees the first's tag/LRU update."""
    rng = np.random.default_rng(3)
    case = _random_case(rng, 512, 1024, 16, 8192)
    tags = case["tags"].numpy().copy()
    lru = case["lru"].numpy().copy()
    t = {k: case[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
    t["tags"] = t["tags"].int()
    for step in range(3):
        pos = torch.tensor(np.sort(rng.integers(0, 8192, size=512)), dtype=torch.int32)
        plan = resolve_rows(LogicalTopK(pos.to(DEV)), t["source"], t["resident"], t["hot"],
                            t["tags"], t["lru"], 8192, 16)
        ref = oracle.resolve_rows(pos.numpy(), case["source"].numpy(), case["resident"].numpy(),
                                  case["hot"].numpy(), tags, lru, 8192, 16)
        tags, lru = ref["tags"], ref["lru"]
        assert plan.physical_rows.tolist() == ref["physical"].tolist(), step
        assert t["tags"].tolist() == tags.tolist(), step
        assert t["lru"].tolist() == lru.tolist(), step


def test_legacy_head_columns():
    rng = np.random.default_rng(11)
    case = _random_case(rng, 64, 128, 4, 400)
    cols = torch.tensor(rng.integers(-1, 66, size=(6, 20)), dtype=torch.int64)
    t = {k: case[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
    plan = resolve_rows(LogicalTopK(case["positions"].to(DEV), cols.to(DEV)), t["source"],
                        t["resident"], t["hot"], t["tags"], t["lru"], 400, 4)
    ref = oracle.resolve_rows(case["positions"].numpy(), case["source"].numpy(),
                              case["resident"].numpy(), case["hot"].numpy(),
                              case["tags"].numpy(), case["lru"].numpy(), 400, 4)
    c = cols.numpy()
    expected = np.where((c >= 0) & (c < 64), ref["physical"][np.clip(c, 0, 63)], -1)
    assert plan.physical_rows.tolist() == expected.tolist()


def test_corrupt_lru_leaves_tables_and_flags():
    case = _random_case(np.random.default_rng(5), 16, 32, 4, 200)
    t = {k: case[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
    t["lru"][3] = 99
    before = t["tags"].clone()
    plan = resolve_rows(LogicalTopK(case["positions"].to(DEV)), t["source"], t["resident"],
                        t["hot"], t["tags"], t["lru"], 200, 4)
    assert plan.physical_rows.tolist() == [-1] * 16
    assert torch.equal(before, t["tags"])
    assert any("LRU" in f for f in _lib.device_flags(DEV))


def test_resolver_graph_capture_without_cpu_readback():
    """Same property as the reference's tests/test_hybrid.py:192-217."""
    rng = np.random.default_rng(9)
    case = _random_case(rng, 64, 128, 4, 256, resident_fraction=0.0, tag_fraction=0.0)
    t = {k: case[k].to(DEV) for k in ("source", "resident", "hot", "tags", "lru")}
    t["tags"] = t["tags"].int()
    logical = LogicalTopK(torch.arange(0, 256, 4, dtype=torch.int32, device=DEV))

    def resolve():
        return resolve_rows(logical, t["source"], t["resident"], t["hot"], t["tags"], t["lru"],
                            256, 4)

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            resolve()
    torch.cuda.current_stream().wait_stream(stream)
    tags_before, lru_before = t["tags"].cpu().numpy(), t["lru"].cpu().numpy()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        result = resolve()
    t["tags"].copy_(torch.tensor(tags_before, device=DEV))
    t["lru"].copy_(torch.tensor(lru_before, device=DEV))
    new = torch.arange(1, 256, 4, dtype=torch.int32)
    logical.positions.copy_(new.to(DEV))
    graph.replay()
    ref = oracle.resolve_rows(new.numpy(), case["source"].numpy(), case["resident"].numpy(),
                              case["hot"].numpy(), tags_before, lru_before, 256, 4)
    assert result.counts.tolist() == ref["counts"].tolist()
    assert result.physical_rows.tolist() == ref["physical"].tolist()


@pytest.mark.parametrize("batch", [8, 48])
def test_batched_cluster_forms_against_oracle(batch):
    """hs_resolve_rows_batched at configuration-3 size (4096 positions, 8192
    hot rows: scratch for a cluster of CTAs). A batch of 8 runs clusters of 4
    CTAs; 48 requests would need more than one wave of those, so they run
    clusters of 2 with larger parts. Every request equals the oracle."""
    k, h, p, length = 4096, 8192, 16, 131072
    rng = np.random.default_rng(batch)
    cases = [_random_case(rng, k, h, p, length) for _ in range(batch)]
    for c in cases:  # Quest-like input: sorted, -1 padded
        pos = np.sort(c["positions"].numpy())
        c["positions"] = torch.tensor(np.where((pos >= 0) & (pos < length), pos, -1),
                                      dtype=torch.int32)
        c["positions"] = torch.cat([c["positions"][c["positions"] >= 0],
                                    c["positions"][c["positions"] < 0]])
    n = max(len(c["source"]) for c in cases)

    def table(name, dtype, size):
        out = []
        for c in cases:
            t = torch.full((size,), -1, dtype=dtype)
            t[:len(c[name])] = c[name].to(dtype)
            out.append(t.to(DEV))
        return out

    src, res = table("source", torch.int32, n), table("resident", torch.int32, n)
    hot = [c["hot"].to(torch.int32).to(DEV) for c in cases]
    tags = [c["tags"].to(torch.int32).to(DEV) for c in cases]
    lru = [c["lru"].to(DEV) for c in cases]

    def ptrs(ts):
        return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=DEV)

    positions = torch.stack([c["positions"] for c in cases]).to(DEV).contiguous()
    lengths = torch.full((batch,), length, dtype=torch.int32, device=DEV)
    phys = torch.empty((batch, k), dtype=torch.int64, device=DEV)
    mh, md = torch.empty_like(phys), torch.empty_like(phys)
    counts = torch.empty((batch, 3), dtype=torch.int64, device=DEV)
    lib = _lib.load()
    ws_bytes = lib.hs_resolve_workspace_bytes(batch, k, h)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=DEV)
    status = _lib.status_word(torch.device(DEV))
    hot_blocks = len(cases[0]["hot"])
    # the pointer arrays stay referenced until the kernel has read them
    arrays = [ptrs(x) for x in (src, res, hot, tags, lru)]
    _lib.check(lib.hs_resolve_rows_batched(
        batch, positions.data_ptr(), k, arrays[0].data_ptr(), arrays[1].data_ptr(), n,
        arrays[2].data_ptr(), hot_blocks, arrays[3].data_ptr(), arrays[4].data_ptr(), h,
        lengths.data_ptr(), p, phys.data_ptr(), mh.data_ptr(), md.data_ptr(),
        counts.data_ptr(), None, ws.data_ptr(), ws_bytes, status.data_ptr(),
        _lib.stream_of(torch.device(DEV))))
    torch.cuda.synchronize()
    for b, c in enumerate(cases):
        ref = oracle.resolve_rows(c["positions"].numpy(), c["source"].numpy(),
                                  c["resident"].numpy(), c["hot"].numpy(), c["tags"].numpy(),
                                  c["lru"].numpy(), length, p)
        assert phys[b].tolist() == ref["physical"].tolist(), b
        assert mh[b].tolist() == ref["miss_host"].tolist(), b
        assert md[b].tolist() == ref["miss_device"].tolist(), b
        assert counts[b].tolist() == ref["counts"].tolist(), b
        assert tags[b].tolist() == ref["tags"].tolist(), b
        assert lru[b].tolist() == ref["lru"].tolist(), b
    assert not _lib.device_flags(DEV)
