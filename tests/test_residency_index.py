"""Indexed residency control against the REAL reference (CPU; skipped where
the reference checkout is absent, e.g. on a GPU box).

hisparse_b200.residency replaces four scans of the reference's
HybridKVCache (resolve's page pinning, update_residency's resident count,
_historical_pages and _unpin_clean_pages per layer; hybrid.py:204-296,
412-469) with per-layer indexes of resident and of pinned pages kept beside
the allocator. The policy must not change: the
reference's own test suite passes with the index installed, and scripted
random sessions (appends, sparse attention with reuse, reclaim, hot
transitions, capacity pressure, releases) give identical outputs, counters,
tables and allocator state with and without it."""

from __future__ import annotations

import os
import random
import subprocess
import sys
from pathlib import Path

import pytest
import torch

REFERENCE = Path(os.environ.get("NANO_HISPARSE_REFERENCE", "/root/reference"))
ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.skipif(not (REFERENCE / "nano_hisparse").is_dir(),
                                reason="reference checkout not available")


@pytest.fixture(scope="module")
def ref():
    sys.dont_write_bytecode = True  # the checkout may be read-only
    if str(REFERENCE) not in sys.path:
        sys.path.insert(0, str(REFERENCE))
    import nano_hisparse

    return nano_hisparse


def test_reference_suite_passes_with_the_index():
    """The reference's CPU tests (residency, hybrid, storage, engine, trace,
    ...) with the indexed methods installed at start-up."""
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([str(REFERENCE), str(ROOT / "tests"),
                                           str(ROOT / "nano-hisparse_b200")]))
    result = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
         "-p", "residency_index_plugin", "--rootdir", str(REFERENCE),
         str(REFERENCE / "tests")],
        cwd=str(REFERENCE), env=env, capture_output=True, text=True, timeout=900)
    tail = result.stdout[-3000:] + result.stderr[-2000:]
    assert result.returncode == 0, tail
    assert " passed" in result.stdout and "failed" not in result.stdout, tail
    assert "indexed residency installed: DeviceAllocator.bind" in result.stdout, tail
    assert "HybridKVCache._unpin_clean_pages" in result.stdout, tail


def _state(cache):
    """Everything the policy decides: counters, per-layer tables and flags,
    allocator ownership and orders, page placement."""
    alloc, storage = cache.allocator, cache.storage
    tables = {g: (t.source.tolist(), t.resident.tolist(), t.hot.tolist(), t.tags.tolist(),
                  t.lru.tolist(), list(t.blocks), t.hot_required, t.trigger, t.busy)
              for g, t in cache.tables.items()}
    pages = {k: (p.slot, p.location.value, p.host_slot, p.valid_tokens, p.content_version,
                 p.host_committed_version) for k, p in storage.pages.items()}
    return {"stats": dict(storage.stats), "row_stats": cache.row_stats.tolist(),
            "tables": tables, "pages": pages, "lru": list(alloc.lru.items()),
            "reclaimable": list(alloc.reclaimable), "free": sorted(alloc.free),
            "refs": [(s.owner, s.ref_cnt) for s in alloc.slots],
            "pending": sorted(cache.pending_clean)}


def _session(ref, seed, check_index=None):
    """A scripted random session on a small pool; returns its log of
    outputs, errors and states."""
    from nano_hisparse.config import CacheConfig, CapacityError
    from nano_hisparse.hybrid import HotConfig, HybridKVCache
    from nano_hisparse.selection import Selection

    rng = random.Random(seed)
    torch.manual_seed(seed)
    P, kv, D, hq = 4, 2, 8, 4
    cfg = CacheConfig(gpu_pages=rng.choice([14, 18, 24]), host_pages=400, page_size=P,
                      kv_heads=kv, head_dim=D, device="cpu")
    hot = HotConfig(8, 8, resident_window_pages=rng.choice([2, 3, 6]),
                    transition_watermark=rng.choice([None, 0, 2]))
    cache = HybridKVCache(cfg, hot)
    log, live, last = [], {}, {}
    for op in range(90):
        choice = rng.random()
        try:
            if choice < 0.12 or not live:
                name = f"r{op}"
                layers = rng.choice([1, 2])
                cache.reserve(name, 120, layers)
                live[name] = layers
                log.append(("reserve", name))
            elif choice < 0.55:
                name = rng.choice(sorted(live))
                layer = rng.randrange(live[name])
                count = rng.choice([1, 1, 2, 5, 9])
                length = cache.storage.requests[name].lengths[layer]
                if length + count > 120:
                    continue
                k, v = torch.randn(2, count, kv, D).unbind(0)
                cache.write(name, layer, k, v)
                log.append(("write", name, layer, count))
            elif choice < 0.85:
                name = rng.choice(sorted(live))
                layer = rng.randrange(live[name])
                length = cache.storage.requests[name].lengths[layer]
                if length < 1:
                    continue
                picks = sorted({rng.randrange(length) for _ in range(rng.randint(1, 8))})
                if (name, layer) in last and rng.random() < 0.5:  # reuse: hot hits
                    picks = last[name, layer]
                last[name, layer] = picks
                q = torch.randn(hq, D)
                out = cache.attention(q, name, layer, Selection.from_tokens(picks, length, P, hq))
                log.append(("attend", name, layer, out.tolist()))
            elif choice < 0.93:
                name = rng.choice(sorted(live))
                layer = rng.randrange(live[name])
                cache.reclaim_history(name, layer, evict=rng.random() < 0.3)
                log.append(("reclaim", name, layer))
            else:
                name = rng.choice(sorted(live))
                cache.release_request(name)
                del live[name]
                log.append(("release", name))
        except (CapacityError, RuntimeError, ValueError) as error:
            log.append(("error", type(error).__name__, str(error)))
        cache.storage.synchronize()
        log.append(_state(cache))
        if check_index is not None:
            check_index(cache)
    return log


def _index_matches_scan(cache):
    from hisparse_b200 import residency

    for group in cache.tables:
        scanned = [k for k in cache.allocator.lru if k[2] >= 0 and k[:2] == group]
        assert list(residency.resident_keys(cache, group)) == scanned
        resident = [p.key for p in cache.storage.pages.values()
                    if p.key[:2] == group and p.slot is not None]
        assert sorted(resident) == sorted(scanned)
        pinned = [k for k in scanned if cache.allocator.lru[k] not in cache.allocator.reclaimable]
        assert sorted(residency._state(cache.allocator)[1].get(group, {})) == sorted(pinned)


@pytest.mark.parametrize("seed", range(12))
def test_sessions_identical_with_and_without_index(ref, seed):
    from hisparse_b200 import residency

    baseline = _session(ref, seed)
    residency.install(ref)
    try:
        indexed = _session(ref, seed, check_index=_index_matches_scan)
    finally:
        residency.uninstall(ref)
    assert len(indexed) == len(baseline)
    for i, (a, b) in enumerate(zip(baseline, indexed)):
        assert a == b, (seed, i)
    assert any(entry[0] == "attend" for entry in baseline if isinstance(entry, tuple))


def test_index_built_for_caches_created_before_install(ref):
    """A cache that already holds resident pages is indexed from its
    allocator's LRU at the first indexed call."""
    from nano_hisparse.config import CacheConfig
    from nano_hisparse.hybrid import HotConfig, HybridKVCache

    from hisparse_b200 import residency

    cache = HybridKVCache(CacheConfig(gpu_pages=12, host_pages=64, page_size=4, kv_heads=1,
                                      head_dim=8, device="cpu"), HotConfig(4, 4))
    cache.reserve("a", 40, 1)
    cache.write("a", 0, torch.randn(22, 1, 8), torch.randn(22, 1, 8))
    residency.install(ref)
    try:
        _index_matches_scan(cache)
        cache.write("a", 0, torch.randn(5, 1, 8), torch.randn(5, 1, 8))
        _index_matches_scan(cache)
    finally:
        residency.uninstall(ref)
