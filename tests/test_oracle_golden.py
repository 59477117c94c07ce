"""Pins the CPU oracle against the reference: known-answer vectors transcribed
from the reference's tests, and fixtures recorded by running the reference
(tests/golden/make_fixtures.py). CPU only."""

import numpy as np
import pytest
import torch

import oracle
from helpers import (TOL, full_quest_inputs, near_tie_report, pages_to_tokens, raw_numpy,
                     rebuild_host, same_bytes)


def test_resolver_known_answer_vector():
    # tests/test_selection.py:36-50 and examples/inspect_indices.py:22-34 of the reference
    out = oracle.resolve_rows([9, 2, 6, 9, 14, -1], [5, 2, 9, 4], [-1, 7, -1, 3], [6, 1],
                              [-1, -1, -1, -1, -1, 22, -1, -1], [0, 1, 2, 3, 4, 6, 7, 5], 16, 4)
    assert out["physical"].tolist() == [24, 5, 30, -1, 14, -1]
    assert out["counts"].tolist() == [2, 1, 1]
    assert out["miss_host"].tolist() == [37, -1, -1, -1, -1, -1]
    assert out["miss_device"].tolist() == [24, -1, -1, -1, -1, -1]
    assert out["tags"][0] == 37 and out["tags"][5] == 22


def test_quest_known_answers():
    # tests/test_selection.py:18-22: a page whose mean cancels is kept
    low = np.array([[[-10.0, 0.0]], [[1.0, 0.0]], [[0.0, 0.0]]], dtype=np.float32)
    high = np.array([[[10.0, 0.0]], [[1.0, 0.0]], [[0.0, 0.0]]], dtype=np.float32)
    q = np.array([[1.0, 0.0]], dtype=np.float32)
    tokens = oracle.quest_tokens(q, low, high, 5, 2, 2, keep_sink=False)
    assert sorted({t // 2 for t in tokens}) == [0, 2]
    # tests/test_selection.py:25-33: head mean before top-k
    bounds = np.array([[[9.0, 0.0]], [[0.0, 10.0]], [[-1.0, -1.0]]], dtype=np.float32)
    tokens = oracle.quest_tokens(np.eye(2, dtype=np.float32), bounds, bounds, 5, 2, 2,
                                 keep_sink=False)
    assert tokens == [2, 3, 4]


def test_resolver_matches_reference_fixtures(golden):
    for case in golden("resolver_cases"):
        out = oracle.resolve_rows(case["positions"].numpy(), case["source"].numpy(),
                                  case["resident"].numpy(), case["hot"].numpy(),
                                  case["tags"].numpy(), case["lru"].numpy(), case["length"],
                                  case["page_size"])
        name = case["name"]
        assert out["physical"].tolist() == case["physical"].tolist(), name
        assert out["miss_host"].tolist() == case["miss_host"].tolist(), name
        assert out["miss_device"].tolist() == case["miss_device"].tolist(), name
        assert out["counts"].tolist() == case["counts"].tolist(), name
        assert out["tags"].tolist() == case["tags_after"].tolist(), name
        assert out["lru"].tolist() == case["lru_after"].tolist(), name


def test_quest_matches_reference_fixtures(golden):
    """Every recorded selection, token for token (a difference is reported with
    the fp64 scores of the pages involved)."""
    checked = 0
    for case in golden("quest_cases"):
        for sink in (0, 1):
            key = f"tokens_{sink}"
            if key not in case:
                continue
            got = oracle.quest_tokens(case["query"], case["minimum"], case["maximum"],
                                      case["length"], case["page_size"], case["top_pages"],
                                      keep_sink=bool(sink))
            assert got == list(case[key]), f"{case['name']} sink={sink}: " + near_tie_report(
                case[key], got, case["query"], case["minimum"], case["maximum"],
                case["length"], case["page_size"], case["top_pages"], bool(sink))
            checked += 1
    assert checked == 62


def test_quest_full_size_matches_reference(golden):
    """The reference's selections at the sizes the bench runs (configuration 2:
    2,048-2,050 pages, configuration 3: 8,192 / 2,048, configuration 5:
    16,389), regenerated from their seeds: the oracle's fixed-order fp32 sums
    pick the same pages, with and without the sink page."""
    cases = golden("quest_full_cases")
    assert len(cases) == 13
    for case in cases:
        q, mn, mx, digest = full_quest_inputs(case["q_heads"], case["kv_heads"],
                                              case["head_dim"], case["page_size"],
                                              case["max_pages"], case["seed"])
        assert digest == case["digest"], f"{case['name']}: input generator changed"
        for sink in (1, 0):
            got = oracle.quest_tokens(q, mn, mx, case["length"], case["page_size"],
                                      case["top_pages"], bool(sink))
            want = pages_to_tokens(case[f"pages_{sink}"], case["length"], case["page_size"])
            assert got == want, f"{case['name']} sink={sink}: " + near_tie_report(
                want, got, q, mn, mx, case["length"], case["page_size"], case["top_pages"],
                bool(sink))


def test_attention_matches_reference_fixtures(golden):
    for case in golden("attention_cases"):
        out = oracle.attend_rows(case["query"], case["pool"], case["rows"].numpy(),
                                 case["page_size"])
        expected = case["out"].double()
        tol = TOL[case["query"].dtype]
        torch.testing.assert_close(torch.from_numpy(out), expected, **tol, msg=case["name"])


def test_scenarios_replay_through_the_oracle(golden):
    """Every resolve/gather/attention call the reference's HybridKVCache made in
    the recorded sessions: bit-exact plans, tables and gathered bytes; attention
    within tolerance; summed counts equal the reference's row counters."""
    for scenario in golden("scenarios"):
        totals = np.zeros(3, dtype=np.int64)
        for i, rec in enumerate(scenario["records"]):
            tag = f"{scenario['name']}[{i}]"
            out = oracle.resolve_rows(rec["positions"].numpy(), rec["source"].numpy(),
                                      rec["resident"].numpy(), rec["hot"].numpy(),
                                      rec["tags"].numpy(), rec["lru"].numpy(), rec["length"],
                                      rec["page_size"])
            physical = out["physical"]
            if rec["head_columns"] is not None:
                cols = rec["head_columns"].numpy()
                physical = np.where((cols >= 0) & (cols < physical.size),
                                    physical[np.clip(cols, 0, physical.size - 1)], -1)
            assert physical.tolist() == rec["physical"].tolist(), tag
            assert out["miss_host"].tolist() == rec["miss_host"].tolist(), tag
            assert out["miss_device"].tolist() == rec["miss_device"].tolist(), tag
            assert out["counts"].tolist() == rec["counts"].tolist(), tag
            assert out["tags"].tolist() == rec["tags_after"].tolist(), tag
            assert out["lru"].tolist() == rec["lru_after"].tolist(), tag
            totals += out["counts"]
            host = raw_numpy(rebuild_host(rec))
            pool = raw_numpy(rec["pool_before"])
            oracle.gather_rows(host, pool, out["miss_host"], out["miss_device"],
                               rec["page_size"])
            assert same_bytes(pool, raw_numpy(rec["pool_after"])), tag
            att = oracle.attend_rows(rec["query"], rec["pool_after"], physical, rec["page_size"])
            torch.testing.assert_close(torch.from_numpy(att), rec["out"].double(),
                                       **TOL[rec["query"].dtype], msg=tag)
        stats = scenario["row_stats"]
        assert totals.tolist() == [stats["resident_hits"], stats["hot_hits"], stats["misses"]]


def test_scenario_counters_match_reference_tests(golden):
    """Counters the reference's own tests assert (test_hybrid.py:58,73,93,274;
    test_residency.py:195; test_trace.py:18-56)."""
    stats = {s["name"]: s["row_stats"] for s in golden("scenarios")}
    assert stats["row_misses_and_resident_hits"] == {
        "resident_hits": 2, "hot_hits": 3, "misses": 3, "h2d_bytes": 192}
    assert stats["late_hits_protected"]["misses"] == 5
    assert stats["invalid_padding_only"]["misses"] == 0
    assert [stats["all_miss_minimum_hot"][k] for k in ("resident_hits", "hot_hits", "misses")] \
        == [0, 0, 64]
    table = {"trace_reuse_4": (28, 4), "trace_alternating_4": (0, 32),
             "trace_alternating_8": (24, 8), "trace_streaming_8": (0, 32),
             "trace_packed_4": (28, 4)}
    for name, (hits, misses) in table.items():
        assert (stats[name]["hot_hits"], stats[name]["misses"]) == (hits, misses), name
        assert stats[name]["h2d_bytes"] == misses * 64


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_oracle_gather_is_a_byte_copy(dtype):
    gen = torch.Generator().manual_seed(5)
    host = torch.randn(6, 2, 3, 2, 4, generator=gen).to(dtype)
    pool = torch.zeros(4, 2, 3, 2, 4, dtype=dtype)
    hn, pn = raw_numpy(host), raw_numpy(pool)
    oracle.gather_rows(hn, pn, [0, 17, 5, -1], [11, 3, 0, -1], 3)
    expected = pool.clone()
    for h, d in ((0, 11), (17, 3), (5, 0)):
        expected[d // 3, :, d % 3] = host[h // 3, :, h % 3]
    assert same_bytes(pn, raw_numpy(expected))


def test_oracle_append_matches_reference_fixtures(golden):
    """The metadata producer + host mirror restatement reproduces every page
    chunk HostStore.append wrote in the recorded sessions: pool block and
    host block bytes, K min/max and the mean-K summary bit for bit."""
    chunks = 0
    for case in golden("append_cases"):
        for record in case["records"]:
            for c in record["chunks"]:
                blk, host, mn, mx, summ = oracle.append_rows(
                    c["k"], c["v"], c["within"], c["block_before"], c["host_before"],
                    c["min_before"], c["max_before"], c["summary_before"].numpy())
                assert np.array_equal(blk, oracle.as_array(c["block_after"])[0]), case["name"]
                assert np.array_equal(host, oracle.as_array(c["host_after"])[0]), case["name"]
                assert np.array_equal(mn, oracle.as_array(c["min_after"])[0]), case["name"]
                assert np.array_equal(mx, oracle.as_array(c["max_after"])[0]), case["name"]
                # rows added in order, then one division: torch's CPU mean gives
                # the same fp32 bits on every recorded chunk
                assert np.array_equal(summ, c["summary_after"].numpy()), case["name"]
                chunks += 1
    assert chunks > 60


def test_oracle_select_ranking_rule():
    """The oracle's ranking, which every selection kernel matches token for
    token, is the rule the header states: forced tail (and sink) pages, then
    the highest scores with -0 equal to +0, NaN above +inf and equal scores
    taking the lower page; checked against a plain sort on random scores with
    ties, signed zeros, infinities and NaN."""
    rng = np.random.default_rng(3)
    for trial in range(400):
        n = int(rng.integers(2, 400))
        top = int(rng.integers(1, n + 3))
        p = int(rng.integers(1, 9))
        length = (n - 1) * p + int(rng.integers(1, p + 1))
        kind = trial % 4
        if kind == 0:
            s = rng.normal(200, 20, n)
        elif kind == 1:
            s = rng.integers(0, 3, n).astype(float)
        elif kind == 2:
            s = rng.choice([0.0, -0.0, 1.0, -1.0], n)
        else:
            s = rng.normal(0, 1e3, n)
            s[rng.integers(0, n, 4)] = np.nan
            s[rng.integers(0, n, 3)] = np.inf
            s[rng.integers(0, n, 3)] = -np.inf
        s = s.astype(np.float32)
        sink = bool(rng.integers(0, 2))
        tokens, count = oracle.quest_select(s, length, p, top, sink, max(top * p, length))
        if top >= n:
            pages = list(range(n))
        else:
            def rank(page):
                if page == n - 1 or (sink and top > 1 and page == 0):
                    return (0, 0.0, page)
                v = float(s[page])
                return (1, 0.0, page) if np.isnan(v) else (2, -(v + 0.0), page)
            pages = sorted(sorted(range(n), key=rank)[:top])
        want = [t for pg in pages for t in range(pg * p, min(pg * p + p, length))]
        assert tokens[:count].tolist() == want, (trial, n, top, sink)
        assert set(tokens[count:].tolist()) <= {-1}
