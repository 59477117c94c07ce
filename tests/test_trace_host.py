"""Trace format, generator and validation on the CPU (trace.py:22-102)."""

import pytest
import torch

from conftest import load_golden
from hisparse_b200.trace import (load_trace, replay_trace, save_trace, synthetic_trace,
                                 validate_trace)


def test_synthetic_traces_equal_the_reference_traces():
    """synthetic_trace draws the reference's tensors in the reference's order:
    the recorded traces come back bit for bit."""
    for case in load_golden("trace_reports"):
        if not case["name"].startswith("synthetic_"):
            continue
        pattern = case["trace"]["source"]["pattern"]
        ours, theirs = synthetic_trace(pattern), case["trace"]
        assert ours["source"] == theirs["source"] and ours["page_size"] == theirs["page_size"]
        for name in ("k", "v"):
            assert torch.equal(ours["prefill"][name], theirs["prefill"][name])
        for a, b in zip(ours["events"], theirs["events"], strict=True):
            assert a["positions"] == b["positions"]
            for name in ("q", "k", "v"):
                assert torch.equal(a[name], b[name])


def test_validate_returns_the_reference_union_bound():
    for case in load_golden("trace_reports"):
        assert validate_trace(case["trace"]) == case["report"]["max_union_rows"], case["name"]


def test_validation_messages(tmp_path):
    trace = synthetic_trace("reuse", steps=2)
    with pytest.raises(ValueError, match="unknown access pattern"):
        synthetic_trace("random")
    with pytest.raises(ValueError, match="2..8 steps"):
        synthetic_trace("reuse", steps=9)
    with pytest.raises(ValueError, match="schema_version"):
        validate_trace({**trace, "schema_version": 3})
    with pytest.raises(ValueError, match="at least one event"):
        validate_trace({**trace, "events": []})
    bad = {**trace, "prefill": {"k": trace["prefill"]["k"], "v": trace["prefill"]["v"][:3]}}
    with pytest.raises(ValueError, match="invalid prefill KV"):
        validate_trace(bad)
    event = {**trace["events"][0], "q": torch.randn(2, 7)}
    with pytest.raises(ValueError, match="incompatible event"):
        validate_trace({**trace, "events": [event]})
    event = {**trace["events"][0], "positions": [[0, 1]]}
    with pytest.raises(ValueError, match="one shared token ID list"):
        validate_trace({**trace, "events": [event]})
    event = {**trace["events"][0], "positions": [0, 65]}
    with pytest.raises(ValueError, match="noncausal"):
        validate_trace({**trace, "events": [event]})
    path = tmp_path / "t" / "trace.pt"
    save_trace(trace, path)
    again = load_trace(path)
    assert torch.equal(again["prefill"]["k"], trace["prefill"]["k"])


def test_replay_has_no_cpu_path():
    with pytest.raises(ValueError, match="no CPU path"):
        replay_trace(synthetic_trace("reuse"), 4, "cpu")
