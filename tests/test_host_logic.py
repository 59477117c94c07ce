"""Host-side logic of the drop-in surface (no GPU): Selection / LogicalTopK
semantics, configuration validation, the plugin binding and sharding."""

import sys
import types

import pytest
import torch

from hisparse_b200 import CacheConfig, HotConfig, LogicalTopK, Selection, quest_selection
from hisparse_b200 import plugin
from hisparse_b200.sharding import lognormal_lengths, requests_for_rank


def test_per_head_masks_and_invalid_positions():
    # restates the reference's tests/test_selection.py:8-15
    selected = Selection.from_tokens([[3, 1, 1, -1], [0]], 4, 2, 2)
    assert selected.positions == ((1, 3), (0,))
    topk = LogicalTopK.from_selection(selected, "cpu")
    assert topk.positions.tolist() == [0, 1, 3]
    assert topk.head_columns.tolist() == [[1, 2], [0, -1]]
    for rows in [[4], [-2], [-1], [1.2], []]:
        with pytest.raises((ValueError, TypeError)):
            Selection.from_tokens(rows, 4, 2, 2)


def test_shared_selection_and_pages():
    sel = Selection.from_pages([0, 2], 10, 4, 3)
    assert sel.positions == ((0, 1, 2, 3, 8, 9),) * 3
    assert sel.pages == [0, 2]
    topk = LogicalTopK.from_selection(sel, "cpu")
    assert topk.head_columns is None and topk.positions.dtype == torch.int32
    with pytest.raises(ValueError, match="invalid logical page"):
        Selection.from_pages([3], 10, 4, 1)


def test_quest_budget_covering_history_needs_no_kernel():
    sel = quest_selection(torch.randn(4, 8), torch.zeros(10, 2, 8), torch.zeros(10, 2, 8), 37,
                          4, 10)
    assert sel.positions[0] == tuple(range(37)) and sel.source == "quest"
    with pytest.raises(ValueError, match="invalid page budget"):
        quest_selection(torch.randn(6, 8), torch.zeros(10, 4, 8), torch.zeros(10, 4, 8), 37, 4, 2)


def test_validate_messages():
    topk = LogicalTopK(torch.arange(5, dtype=torch.int32))
    with pytest.raises(ValueError, match="max_union_rows"):
        topk.validate("cpu", 4)
    with pytest.raises(ValueError, match="nonempty device integer vector"):
        LogicalTopK(torch.zeros(0, dtype=torch.int32)).validate("cpu", 4)
    with pytest.raises(ValueError, match="head columns"):
        LogicalTopK(torch.arange(2), torch.zeros(2, 2, dtype=torch.int32)).validate("cpu", 4)


def test_configs():
    assert HotConfig(4).hot_rows == 8
    with pytest.raises(ValueError):
        HotConfig(8, 4)
    with pytest.raises(ValueError):
        HotConfig(4, 40000)
    assert HotConfig(2048, 4096).admission_blocks(16, 32) == 32 * (256 + 2)
    with pytest.raises(ValueError):
        CacheConfig(page_size=0)
    with pytest.raises(ValueError):
        CacheConfig(dtype=torch.int8)
    assert CacheConfig(kv_heads=8, head_dim=128, dtype=torch.bfloat16).row_bytes == 2048


def test_plugin_rebinds_and_restores_reference_names():
    pkg = types.ModuleType("fake_reference")
    pkg.__path__ = []
    originals = {}
    for sub, names in [("selection", ["quest_selection"]), ("model", ["quest_selection"]),
                       ("hybrid", ["resolve_rows", "LogicalTopK"]),
                       ("row_kernels", ["MappedHost", "gather_rows", "attend_rows"]),
                       ("storage", [])]:
        mod = types.ModuleType(f"fake_reference.{sub}")
        for name in names:
            value = object()
            setattr(mod, name, value)
            originals[sub, name] = value
        sys.modules[mod.__name__] = mod
        setattr(pkg, sub, mod)
    store_append = lambda self, *args: None  # noqa: E731
    sys.modules["fake_reference.storage"].HostStore = type("HostStore", (),
                                                           {"append": store_append})
    sys.modules["fake_reference"] = pkg
    try:
        bound = plugin.install(pkg, indexed_residency=False)
        assert len(bound) == 8
        import hisparse_b200 as hs
        from hisparse_b200.append import host_store_append

        store_cls = sys.modules["fake_reference.storage"].HostStore
        assert store_cls.append is host_store_append

        assert sys.modules["fake_reference.hybrid"].resolve_rows is hs.resolve_rows
        assert sys.modules["fake_reference.row_kernels"].attend_rows is hs.attend_rows
        assert sys.modules["fake_reference.model"].quest_selection is hs.quest_selection
        plugin.uninstall(pkg)
        for (sub, name), value in originals.items():
            assert getattr(sys.modules[f"fake_reference.{sub}"], name) is value
        assert store_cls.__dict__["append"] is store_append
    finally:
        for key in [k for k in sys.modules if k.startswith("fake_reference")]:
            del sys.modules[key]


def test_sharding_helpers():
    ids = list(range(10))
    shards = [requests_for_rank(ids, r, 4) for r in range(4)]
    assert sorted(sum(shards, [])) == ids
    assert [len(s) for s in shards] == [3, 3, 2, 2]
    lengths = lognormal_lengths(256, 16384, 4096, 131072, seed=4)
    assert min(lengths) >= 4096 and max(lengths) <= 131072
    assert 8000 < sorted(lengths)[128] < 32000
    assert lengths == lognormal_lengths(256, 16384, 4096, 131072, seed=4)


def test_numa_topology_parsing(tmp_path):
    from hisparse_b200.sharding import parse_cpulist, pci_local_cpus

    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert parse_cpulist("") == set()
    node = tmp_path / "0000:53:00.0"
    node.mkdir()
    (node / "local_cpulist").write_text("56-111,168-223\n")
    cpus = pci_local_cpus(0, 0x53, 0, tmp_path)
    assert len(cpus) == 112 and 56 in cpus and 223 in cpus and 0 not in cpus
    assert pci_local_cpus(0, 0x54, 0, tmp_path) is None


def test_bench_host_store_budget(monkeypatch):
    """bench.py sizes each rank's pinned host store to half the free host RAM
    shared by the node's ranks, and refuses when not even four pages' worth
    of contexts fit."""
    import bench

    page = 64 * 1024
    wanted = 16 * 32 * 2048  # configuration 2: REQUESTS x LAYERS x pages
    monkeypatch.setattr(bench, "available_host_bytes", lambda: 1 << 40)  # 1 TiB free
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    assert bench.host_store_pages(wanted, page, lambda m: None) == wanted
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    monkeypatch.setattr(bench, "available_host_bytes", lambda: 1 << 39)  # 512 GiB free
    shared = bench.host_store_pages(wanted, page, lambda m: None)
    assert shared == (1 << 39) // 2 // 8 // page < wanted
    monkeypatch.setattr(bench, "available_host_bytes", lambda: None)  # unknown: no cap
    assert bench.host_store_pages(wanted, page, lambda m: None) == wanted
    monkeypatch.setattr(bench, "available_host_bytes", lambda: 1 << 30)
    with pytest.raises(RuntimeError, match="host RAM"):
        bench.host_store_pages(wanted, page, lambda m: None)


def test_bench_clock_window(tmp_path):
    """Clock samples are kept for the timed window; throttle reasons are
    collected from the samples inside it."""
    import datetime
    import time

    import bench

    sampler = bench.ClockSampler(0)
    sampler.path = tmp_path / "clocks.csv"
    now = time.time()
    lines = []
    for k in range(12):
        stamp = datetime.datetime.fromtimestamp(now - 0.6 + 0.1 * k).strftime(
            "%Y/%m/%d %H:%M:%S.%f")[:-3]
        reason = "Active" if k == 3 else "Not Active"   # before the window
        lines.append(f"{stamp}, 0, {1900 + k}, 1965, 700.0, 0x0, Not Active, Not Active, "
                     f"Not Active, {reason}")
    sampler.path.write_text("\n".join(lines))

    class Done:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            pass

    sampler.proc = Done()
    sampler.window(now - 0.05, now + 0.25)
    clocks = sampler.stop()
    assert clocks["window"] == "timed region" and clocks["samples"] >= 3
    assert clocks["reasons"] == [] and clocks["sm_max_mhz"] == 1965.0
