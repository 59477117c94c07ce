"""BatchedEngine against the reference Engine (engine.py:76-136).

The fixtures hold every step of the reference's Engine.run on the CPU at
configuration 1 and variants (tests/golden/make_fixtures.py engine_cases),
on weights that DecoderWeights.random rebuilds here bit for bit. The batched
engine must emit the same (request, token) list at every step: the same
admissions, the same tokens, the same finishing order. fp32 throughout; the
fixture records the reference's smallest top-2 logit margin (>= 2.8e-3) and
Quest boundary gap (>= 7.8e-5 of the largest page score), far above the
~1e-6 relative differences of device vs CPU fp32 arithmetic.
"""

from __future__ import annotations

import pytest
import torch

from helpers import weights_digest

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _cases():
    from pathlib import Path

    path = Path(__file__).parent / "golden" / "engine_cases.pt"
    return {c["name"]: c for c in torch.load(path, weights_only=True)}


CASES = _cases()


def _engine(case, dtype=torch.float32, gpu_pages=None):
    from hisparse_b200.config import CacheConfig, HotConfig
    from hisparse_b200.engine import BatchedEngine, DecoderConfig, DecoderWeights, ServingCache

    weights = DecoderWeights.random(DecoderConfig(**case["model"]), case["seed"], device=DEV,
                                    dtype=dtype)
    cache = ServingCache(
        CacheConfig(gpu_pages=gpu_pages or case["gpu_pages"], host_pages=case["host_pages"],
                    page_size=case["page_size"], kv_heads=case["model"]["num_key_value_heads"],
                    head_dim=case["model"]["hidden_size"] // case["model"]["num_attention_heads"],
                    device=DEV, dtype=dtype),
        HotConfig(case["union"], case["hot_rows"]))
    engine = BatchedEngine(weights, cache, top_k=case["top_k"],
                           eos_token_id=case["eos_token_id"])
    for rid, prompt, max_new in case["requests"]:
        engine.add_request(rid, prompt, max_new)
    return engine, weights, cache


@pytest.mark.parametrize("name", sorted(CASES))
def test_engine_steps_equal_the_reference_engine(name):
    case = CASES[name]
    engine, weights, cache = _engine(case)
    cpu_weights = type(weights)(weights.config, weights.state_dict(), "cpu", torch.float32)
    assert weights_digest(cpu_weights) == case["weights_sha256"]
    for index, expected in enumerate(case["steps"]):
        got = engine.step()
        want = [(rid, tok) for rid, tok, _ in expected]
        assert got == want, (f"{name} step {index}: {got} != {want} (reference top-2 logit "
                             f"margins {[m for *_, m in expected]})")
        if index % 8 == 3:
            cache.assert_invariants()
    assert not engine.waiting and not engine.running
    assert {r: engine.requests[r].generated for r in case["generated"]} == case["generated"]
    assert all(r.prefill_count == 1 for r in engine.requests.values())
    cache.assert_invariants()
    assert not cache.requests and len(cache.free_pool) == case["gpu_pages"]
    from hisparse_b200 import _lib

    assert not _lib.device_flags(DEV)


def test_engine_tight_pool_reads_history_through_the_gather():
    """Configuration 1's pool (one request's credits) keeps no history
    resident: every selected history row is a miss gathered from the host
    store, and the tokens still equal the reference's."""
    case = CASES["config1"]
    engine, _, cache = _engine(case)
    out = engine.run()
    assert out == case["generated"]
    stats = cache.snapshot()
    assert stats["row_stats"]["misses"] > 0
    assert stats["placement"]["host_only_pages"] > 0


def test_engine_wide_pool_borrows_and_revokes():
    """A pool with spare blocks: prompt history borrows them, and an
    admission that needs credits revokes borrowed blocks (tokens unchanged)."""
    case = CASES["config1_wide"]
    # room for the three requests' credits (72) plus a few borrowed blocks:
    # the third admission must take some back
    engine, _, cache = _engine(case, gpu_pages=80)
    assert engine.run() == case["generated"]
    stats = cache.snapshot()["placement"]
    assert stats["borrowed"] > 0 and stats["revoked"] > 0


def test_engine_bf16_runs_with_cancellation():
    """bf16 serving at configuration 1's shape: a cancelled running request
    frees its blocks, the others finish, and no device flag is raised."""
    case = CASES["config1_wide"]
    engine, _, cache = _engine(case, dtype=torch.bfloat16)
    for _ in range(5):
        engine.step()
    engine.cancel("b")
    assert engine.requests["b"].cancelled and "b" not in cache.requests
    cache.assert_invariants()
    out = engine.run()
    assert len(out["a"]) == 33 and len(out["c"]) == 33 and len(out["b"]) < 33
    assert all(0 <= t < case["model"]["vocab_size"] for toks in out.values() for t in toks)
    from hisparse_b200 import _lib

    assert not _lib.device_flags(DEV)
