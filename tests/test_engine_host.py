"""BatchedEngine's scheduler against the REAL reference Engine (CPU; skipped
where the reference checkout is absent, e.g. on a GPU box).

Both engines run on the same fakes: a token source that is a fixed function
of (request, tokens emitted so far) and a cache with a fixed number of
admission slots. Scripted sessions (admission deferral, EOS, cancelling
waiting and running requests, validation errors, a pool that can never
admit) must give the same emitted list, the same queues and the same
request records after every step (engine.py:48-143).
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

REFERENCE = Path(os.environ.get("NANO_HISPARSE_REFERENCE", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REFERENCE / "nano_hisparse").is_dir(),
                                reason="reference checkout not available")

VOCAB, LAYERS, KV_HEADS, HEAD_DIM, PAGE = 64, 2, 2, 8, 4


@pytest.fixture(scope="module")
def ref():
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(REFERENCE))
    try:
        yield SimpleNamespace(engine=importlib.import_module("nano_hisparse.engine"),
                              config=importlib.import_module("nano_hisparse.config"))
    finally:
        sys.path.remove(str(REFERENCE))


def next_token(request_id, emitted):
    return (sum(map(ord, request_id)) * 7 + emitted * 13) % VOCAB


def one_hot(token):
    logits = torch.zeros(VOCAB)
    logits[token] = 1.0
    return logits


class RefModel:
    """What the reference Engine calls (model.py:162-221), as fakes."""

    def __init__(self):
        self.config = SimpleNamespace(num_hidden_layers=LAYERS, vocab_size=VOCAB,
                                      num_key_value_heads=KV_HEADS, head_dim=HEAD_DIM)
        self.device, self.dtype, self.emitted = torch.device("cpu"), torch.float32, {}

    def prefill(self, tokens, cache, request_id):
        self.emitted[request_id] = 1
        return one_hot(next_token(request_id, 0))

    def decode(self, token, request_id, cache, top_k=None, backend="auto", selector="quest"):
        n = self.emitted[request_id]
        self.emitted[request_id] = n + 1
        return one_hot(next_token(request_id, n))


class SlotCache:
    """A cache with `slots` admissions (the reference's or ours, by error class)."""

    def __init__(self, slots, capacity_error, host_pages=10**6):
        self.config = SimpleNamespace(kv_heads=KV_HEADS, head_dim=HEAD_DIM, page_size=PAGE,
                                      host_pages=host_pages, index_budget_bytes=10**9)
        from hisparse_b200.config import HotConfig

        self.hot_config = HotConfig(64)
        self.pool = torch.empty(0)
        self.slots, self.live, self.error = slots, [], capacity_error
        self.storage = SimpleNamespace(retired=[])
        self.rows = SimpleNamespace(synchronize=lambda: None)

    @property
    def budget(self):
        return max(self.slots, 1)

    def collect(self, wait=False):
        pass

    def admission_blocks(self, layers):
        return 1

    def index_reservation_bytes(self, max_tokens, layers):
        return 0

    def reserve(self, request_id, max_tokens, layers):
        if len(self.live) >= self.slots:
            raise self.error("no slot")
        self.live.append(request_id)

    def release_request(self, request_id, wait=True):
        self.live.remove(request_id)


def ours(slots, eos=None, host_pages=10**6):
    from hisparse_b200.config import CapacityError
    from hisparse_b200.engine import BatchedEngine, DecoderConfig, DecoderWeights

    class FakeForward(BatchedEngine):
        def _prefill(self, request):
            return next_token(request.request_id, 0)

        def _decode(self, requests):
            return [next_token(r.request_id, len(r.generated)) for r in requests]

    weights = DecoderWeights.random(
        DecoderConfig(vocab_size=VOCAB, hidden_size=32, intermediate_size=64,
                      num_hidden_layers=LAYERS, num_attention_heads=4,
                      num_key_value_heads=KV_HEADS), 0, device="cpu", dtype=torch.float32)
    cache = SlotCache(slots, CapacityError, host_pages)
    return FakeForward(weights, cache, top_k=2, eos_token_id=eos), cache


def theirs(ref, slots, eos=None, host_pages=10**6):
    cache = SlotCache(slots, ref.config.CapacityError, host_pages)
    return ref.engine.Engine(RefModel(), cache, top_k=2, eos_token_id=eos), cache


def state(engine, cache):
    return ([r.request_id for r in engine.waiting], [r.request_id for r in engine.running],
            {k: (r.generated, r.prefill_count, r.decode_count, r.finished, r.cancelled)
             for k, r in engine.requests.items()}, list(cache.live))


SESSIONS = {
    # step -> actions taken before that step
    "deferral_and_cancel": {
        0: [("add", "a", 9, 3), ("add", "b", 5, 5), ("add", "c", 7, 1), ("add", "d", 4, 4),
            ("add", "e", 6, 6)],
        2: [("cancel", "e")],
        4: [("cancel", "b"), ("add", "f", 3, 2)],
    },
    "eos": {0: [("add", "x", 4, 8), ("add", "yy", 6, 8), ("add", "z", 5, 8)]},
    "late_arrivals": {0: [("add", "a", 3, 4)], 3: [("add", "b", 2, 2), ("add", "c", 2, 3)],
                      5: [("cancel", "a"), ("cancel", "a")]},
}


@pytest.mark.parametrize("name,slots", [("deferral_and_cancel", 2), ("eos", 3),
                                        ("late_arrivals", 1), ("deferral_and_cancel", 5)])
def test_batched_engine_schedules_like_the_reference(ref, name, slots):
    eos = next_token("yy", 3) if name == "eos" else None
    mine, my_cache = ours(slots, eos)
    other, other_cache = theirs(ref, slots, eos)
    script = SESSIONS[name]
    for step in range(40):
        for action in script.get(step, []):
            for engine in (mine, other):
                if action[0] == "add":
                    engine.add_request(action[1], list(range(action[2])), action[3])
                else:
                    engine.cancel(action[1])
        if not (mine.waiting or mine.running or other.waiting or other.running) and \
                step > max(script):
            break
        assert mine.step() == other.step(), f"step {step}"
        assert state(mine, my_cache) == state(other, other_cache), f"step {step}"
    assert mine.run() == other.run()


def test_validation_and_capacity_errors_match(ref):
    from hisparse_b200.config import CapacityError

    cases = [("a", [1, 2], 0), ("a", [], 2), ("a", [VOCAB], 2), ("a", [-1], 2)]
    for rid, prompt, max_new in cases:
        mine, _ = ours(2)
        other, _ = theirs(ref, 2)
        with pytest.raises(ValueError) as e_mine:
            mine.add_request(rid, prompt, max_new)
        with pytest.raises(ValueError) as e_other:
            other.add_request(rid, prompt, max_new)
        assert str(e_mine.value) == str(e_other.value)
    mine, _ = ours(2)
    other, _ = theirs(ref, 2)
    mine.add_request("a", [1], 1)
    other.add_request("a", [1], 1)
    with pytest.raises(ValueError):
        mine.add_request("a", [1], 1)
    with pytest.raises(ValueError):
        other.add_request("a", [1], 1)
    # host pool too small for the request at all
    mine, _ = ours(2, host_pages=3)
    other, _ = theirs(ref, 2, host_pages=3)
    with pytest.raises(CapacityError):
        mine.add_request("a", list(range(10)), 4)
    with pytest.raises(ref.config.CapacityError):
        other.add_request("a", list(range(10)), 4)
    # a pool that can never admit, nothing running: the step raises
    mine, _ = ours(0)
    other, _ = theirs(ref, 0)
    mine.add_request("a", [1, 2], 2)
    other.add_request("a", [1, 2], 2)
    with pytest.raises(CapacityError):
        mine.step()
    with pytest.raises(ref.config.CapacityError):
        other.step()
