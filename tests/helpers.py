"""Helpers shared by the CPU (oracle) and GPU (kernel) parity tests."""

from __future__ import annotations

import math

import numpy as np
import torch

# Attention tolerances: fp32 as the reference's own tests (tests/test_hybrid.py:56-57),
# half precision as its trace replay (trace.py:146-147); the bf16 bound is the
# stated 2e-2 absolute, with no relative slack.
TOL = {
    torch.float32: dict(atol=1e-5, rtol=2e-5),
    torch.float16: dict(atol=8e-3, rtol=8e-3),
    torch.bfloat16: dict(atol=2e-2, rtol=0.0),
}


def raw_numpy(t: torch.Tensor) -> np.ndarray:
    """Byte-exact numpy copy of a CPU tensor (16-bit floats as uint16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def same_bytes(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality (uninitialised pool memory may hold NaN patterns)."""
    return a.shape == b.shape and np.array_equal(
        np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(b).view(np.uint8))


def rebuild_host(record) -> torch.Tensor:
    """Host store of a recorded resolve call: the blocks its gather read, zeros
    elsewhere (the gather reads nothing else)."""
    data = record["host_data"]
    host = torch.zeros((record["host_pages"], *data.shape[1:]), dtype=data.dtype)
    blocks = record["host_blocks"]
    if blocks.numel():
        host[blocks] = data
    return host


def expected_physical(record):
    """Reference physical rows: [K] shared, or [Hq, W] for per-head columns."""
    return record["physical"]


def quest_scores_fp64(query, minimum, maximum, pages):
    q = query.double().numpy()
    mn = minimum[:pages].double().numpy()
    mx = maximum[:pages].double().numpy()
    hq, hkv = q.shape[0], mn.shape[1]
    g = hq // hkv
    lo = np.repeat(mn, g, axis=1)  # [pages, hq, d]
    hi = np.repeat(mx, g, axis=1)
    s = np.maximum(q[None] * lo, q[None] * hi).sum(-1)  # [pages, hq]
    return s.mean(1)


def forced_pages(pages, top_pages, keep_sink):
    forced = {pages - 1}
    if keep_sink and top_pages > 1 and pages > 1:
        forced.add(0)
    return forced


def quest_sets_agree(expected_tokens, got_tokens, query, minimum, maximum, length, page_size,
                     top_pages, keep_sink, rel=1e-5):
    """Selections agree exactly, or differ only in pages whose exact (fp64)
    scores tie with the k-th score to within `rel` (fp32 summation order is
    left unspecified by the reference). Returns (ok, detail)."""
    if list(expected_tokens) == list(got_tokens):
        return True, "identical"
    pages = math.ceil(length / page_size)
    a = {t // page_size for t in expected_tokens}
    b = {t // page_size for t in got_tokens}
    if len(a) != len(b):
        return False, f"page counts differ: {len(a)} vs {len(b)}"
    scores = quest_scores_fp64(query, minimum, maximum, pages)
    forced = forced_pages(pages, top_pages, keep_sink)
    chosen = sorted((p for p in a if p not in forced), key=lambda p: scores[p])
    if not chosen:
        return False, "forced pages differ"
    kth = scores[chosen[0]]
    scale = max(abs(kth), np.abs(scores).max() * 1e-3, 1e-30)
    for p in a ^ b:
        if p in forced or abs(scores[p] - kth) > rel * scale:
            return False, f"page {p} score {scores[p]!r} vs k-th {kth!r}"
    return True, f"near-tie pages {sorted(a ^ b)}"
