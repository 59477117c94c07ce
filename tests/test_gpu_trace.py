"""Trace replay through the kernels against the reference's own replay
reports (trace.py:109-216), recorded by tests/golden/make_fixtures.py."""

import pytest
import torch

from conftest import load_golden
from hisparse_b200.trace import replay_trace

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

# The locality table of the reference's README (README.md:135-139) and
# tests/test_trace.py:18-56: (resident hits, hot hits, misses, h2d bytes).
README_COUNTERS = {
    ("reuse", 4): (0, 28, 4, 256),
    ("alternating", 4): (0, 0, 32, 2048),
    ("alternating", 8): (0, 24, 8, 512),
    ("streaming", 8): (0, 0, 32, 2048),
    ("packed", 4): (0, 28, 4, 256),
}


def _lists(value):
    """Tuples -> lists, recursively (the fixtures store lists)."""
    if isinstance(value, (list, tuple)):
        return [_lists(v) for v in value]
    return value


@pytest.fixture(scope="module")
def cases():
    return load_golden("trace_reports")


@pytest.mark.parametrize("index", range(11))
def test_replay_matches_reference_report(cases, index):
    """Every report field the reference computes from the replay (counters,
    hot contents as logical tokens, Jaccard, density, reuse gaps, summary)
    equals the reference's, and the attention stays within the replay's
    own tolerance of a dense fp32 attention over the selected rows."""
    case = cases[index]
    report = replay_trace(case["trace"], case["capacity"], DEV)
    expected = case["report"]
    error = report["summary"].pop("max_abs_error")
    tolerance = 3e-5 if case["trace"]["prefill"]["k"].dtype == torch.float32 else 8e-3
    assert error <= 2 * tolerance, case["name"]
    assert report.pop("device").startswith("cuda")
    events = report.pop("events")
    assert report == {k: v for k, v in expected.items() if k != "events"}, case["name"]
    assert len(events) == len(expected["events"])
    for got, want in zip(events, expected["events"]):
        got.pop("max_abs_error")
        got["positions"] = _lists(got["positions"])
        assert got == want, (case["name"], got["step"])


@pytest.mark.parametrize("pattern,capacity", sorted(README_COUNTERS))
def test_readme_locality_table(cases, pattern, capacity):
    """The README's synthetic-trace counters, reproduced by the kernels."""
    case = next(c for c in cases if c["name"] == f"synthetic_{pattern}_{capacity}")
    summary = replay_trace(case["trace"], capacity, DEV)["summary"]
    got = tuple(summary[k] for k in ("resident_hits", "hot_hits", "misses", "h2d_bytes"))
    assert got == README_COUNTERS[pattern, capacity]
