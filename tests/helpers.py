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


def full_quest_inputs(q_heads, kv_heads, head_dim, page_size, pages, seed,
                      dtype=torch.bfloat16, chunk=1024):
    """Seeded Quest inputs at full configuration sizes, regenerated wherever a
    test needs them (the metadata of one configuration-5 layer is 33 MB, too
    large to commit): q ~ N(0,1) [q_heads, head_dim]; K ~ N(0,1) drawn page
    chunk by page chunk as [chunk, page_size, kv_heads, head_dim]; the page
    bounds are K's min/max over each page's tokens, in `dtype`.
    Returns (q, minimum, maximum, digest), digest = sha256 of their bytes,
    which a fixture records so a changed generator is caught, not mistaken
    for a parity failure."""
    import hashlib

    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(q_heads, head_dim, generator=gen).to(dtype)
    mn = torch.empty((pages, kv_heads, head_dim), dtype=dtype)
    mx = torch.empty_like(mn)
    for lo in range(0, pages, chunk):
        n = min(chunk, pages - lo)
        keys = torch.randn(n, page_size, kv_heads, head_dim, generator=gen).to(dtype)
        mn[lo:lo + n] = keys.amin(1)
        mx[lo:lo + n] = keys.amax(1)
    h = hashlib.sha256()
    for t in (q, mn, mx):
        h.update(raw_numpy(t).tobytes())
    return q, mn, mx, h.hexdigest()


def pages_to_tokens(pages, length, page_size):
    """Selection.from_pages' expansion: every token of the pages in ascending
    order, the last page clipped at `length`."""
    return [t for p in sorted(pages)
            for t in range(p * page_size, min((p + 1) * page_size, length))]


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


def near_tie_report(expected_tokens, got_tokens, query, minimum, maximum, length,
                    page_size, top_pages, keep_sink):
    """Explains a selection that differs from the reference's: the pages in
    which they differ, each with its exact (fp64) score and its relative gap
    to the k-th chosen score. Selections must be identical; this only names
    what differs, for the failure message."""
    pages = math.ceil(length / page_size)
    a = {t // page_size for t in expected_tokens}
    b = {t // page_size for t in got_tokens}
    if len(a) != len(b):
        return f"page counts differ: {len(a)} vs {len(b)}"
    scores = quest_scores_fp64(query, minimum, maximum, pages)
    forced = forced_pages(pages, top_pages, keep_sink)
    chosen = sorted((p for p in a if p not in forced), key=lambda p: scores[p])
    if not chosen:
        return "forced pages differ"
    kth = scores[chosen[0]]
    return ", ".join(f"page {p}: fp64 score {scores[p]!r}, gap to k-th "
                     f"{(scores[p] - kth) / max(abs(kth), 1e-30):+.3e} (relative)"
                     + (" [forced]" if p in forced else "")
                     for p in sorted(a ^ b))


def weights_digest(weights) -> str:
    """sha256 of a DecoderWeights' reference state_dict (fp32 bytes, sorted
    names): pins that seeded weights come out the same on every machine."""
    import hashlib

    h = hashlib.sha256()
    for name, tensor in sorted(weights.state_dict().items()):
        h.update(name.encode())
        h.update(tensor.numpy().tobytes())
    return h.hexdigest()
