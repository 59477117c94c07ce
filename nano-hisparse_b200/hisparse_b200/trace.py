"""Token-row traces replayed through the hot-path kernels.

Drop-in for nano_hisparse/trace.py:22-216: the same trace format (schema 1
or 2: a prefill K/V, then events of one query, one appended K/V row and the
selected token positions), the same validation and messages, and a
``replay_trace`` that returns the reference's report — per event the
length, union rows, selected pages, row/page Jaccard against the previous
event, page density, resident/hot/miss counts, host->device bytes, the hot
buffer's contents as logical tokens and the attention error; the summary
of those — so a recorded trace is a regression fixture for the resolver's
locality counters on the GPU.

The replay runs every event through the kernels: the appended row through
``hs_append_rows`` (pool tail block, host store, page min/max), the
selection through the resolver, the miss gather and the row attention
(``ServingCache`` -> ``RowCache.attention``). The placement is the
reference's replay placement (trace.py:126-147): a pool of exactly the
admission blocks (the hot region plus two tail blocks), so after the
prefill the history is host-only, the two pages at the write tail stay
resident and the hot buffer starts empty; each new page takes the block of
the page two behind it. The attention error column compares the kernel
output with a dense fp32 torch attention over the same selected rows
(selection.py:94-102), a diagnostic like the reference's, which
synchronises every event: the replay is not a timing tool.
"""

from __future__ import annotations

from math import ceil
from statistics import mean

import torch

from .config import CacheConfig, HotConfig
from .selection import Selection

PATTERNS = ("reuse", "alternating", "streaming", "packed")


def synthetic_trace(pattern, steps=8, seed=42):
    """The four controlled access patterns of trace.py:22-55 on a 64-row
    prefill of one KV head (head_dim 8, page 4), K/V and queries drawn from
    one CPU generator in the same order, so the trace's tensors are the
    reference's. Rows per step: reuse {0,4,8,12}; alternating shifts them by
    step % 2; streaming {s, 16+s, 32+s, 48+s}; packed {0,1,2,3}."""
    if pattern not in PATTERNS:
        raise ValueError("unknown access pattern")
    if not 2 <= steps <= 8:
        raise ValueError("synthetic traces support 2..8 steps")
    generator = torch.Generator().manual_seed(seed)

    def draw(count):
        return torch.randn(count, 1, 8, generator=generator)

    prefill_k = draw(64)
    prefill_v = draw(64)
    events = []
    for step in range(steps):
        if pattern == "packed":
            rows = [0, 1, 2, 3]
        elif pattern == "streaming":
            rows = [step, 16 + step, 32 + step, 48 + step]
        else:
            shift = step % 2 if pattern == "alternating" else 0
            rows = [shift, 4 + shift, 8 + shift, 12 + shift]
        q = torch.randn(2, 8, generator=generator)
        k = draw(1)
        v = draw(1)
        events.append({"q": q, "k": k, "v": v, "positions": rows})
    return {"schema_version": 2,
            "source": {"kind": "synthetic", "pattern": pattern, "seed": seed},
            "page_size": 4, "prefill": {"k": prefill_k, "v": prefill_v}, "events": events}


def validate_trace(trace):
    """trace.py:58-90: checks the schema, the prefill and every event; returns
    the largest union of selected rows over the events (the hot buffer's
    default capacity)."""
    if trace.get("schema_version") not in (1, 2) or not isinstance(trace.get("source"), dict):
        raise ValueError("trace requires schema_version=1 or 2 and source metadata")
    if not trace.get("events"):
        raise ValueError("trace needs at least one event")
    k, v = trace["prefill"]["k"], trace["prefill"]["v"]
    if k.ndim != 3 or k.shape != v.shape or min(k.shape) < 1 or k.dtype != v.dtype:
        raise ValueError("invalid prefill KV")
    if k.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError("unsupported KV dtype")
    kv_heads, head_dim = k.shape[1], k.shape[2]
    length, union = k.shape[0], 0
    for event in trace["events"]:
        q, new_k, new_v = event["q"], event["k"], event["v"]
        shapes_ok = (tuple(new_k.shape) == (1, kv_heads, head_dim)
                     and new_v.shape == new_k.shape
                     and new_k.dtype == k.dtype and new_v.dtype == k.dtype)
        query_ok = (q.ndim == 2 and q.shape[1] == head_dim and q.shape[0] >= 1
                    and q.shape[0] % kv_heads == 0 and q.dtype == k.dtype)
        if not (shapes_ok and query_ok):
            raise ValueError("incompatible event Q/K/V")
        length += 1
        positions = event["positions"]
        if trace["schema_version"] == 2 and (
                not isinstance(positions, (list, tuple))
                or not all(isinstance(t, int) for t in positions)):
            raise ValueError("schema_version=2 requires one shared token ID list per query")
        selection = Selection.from_tokens(positions, length, trace["page_size"], q.shape[0])
        union = max(union, len(set().union(*selection.positions)))
    return union


def save_trace(trace, path):
    """Validates, then writes with torch.save (trace.py:93-96)."""
    validate_trace(trace)
    path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(trace, path)


def load_trace(path):
    """Loads with weights_only=True and validates (trace.py:99-102)."""
    trace = torch.load(path, map_location="cpu", weights_only=True)
    validate_trace(trace)
    return trace


def _jaccard(current, previous):
    if previous is None:
        return None
    return len(current & previous) / len(current | previous)


def _selected_attention(q, k, v, selection):
    """Dense fp32 attention of each query head over its selected rows (the
    sparse output of selection.py:94-102), in the query's dtype."""
    heads, kv_heads = q.shape[0], k.shape[1]
    group = heads // kv_heads
    keys = k.float().repeat_interleave(group, 1)
    values = v.float().repeat_interleave(group, 1)
    scores = torch.einsum("hd,thd->ht", q.float(), keys) / q.shape[-1] ** 0.5
    mask = torch.zeros_like(scores, dtype=torch.bool)
    for head, rows in enumerate(selection.positions):
        mask[head, list(rows)] = True
    weights = scores.masked_fill(~mask, float("-inf")).softmax(-1)
    return torch.einsum("ht,thd->hd", weights, values).to(q.dtype)


@torch.inference_mode()
def replay_trace(trace, hot_rows=None, device="cuda"):
    """Replays a trace through the kernels and reports its locality
    (trace.py:109-216; same report keys and meanings). ``device`` must be a
    CUDA device: there is no CPU path."""
    from .engine import ServingCache

    union_bound = validate_trace(trace)
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("replay_trace runs the CUDA kernels; there is no CPU path")
    page_size, schema = trace["page_size"], trace["schema_version"]
    k = trace["prefill"]["k"].to(device)
    v = trace["prefill"]["v"].to(device)
    prefill, kv_heads, head_dim = k.shape
    maximum = prefill + len(trace["events"])
    hot = HotConfig(union_bound, union_bound if hot_rows is None else hot_rows)
    config = CacheConfig(gpu_pages=hot.admission_blocks(page_size),
                         host_pages=ceil(maximum / page_size), page_size=page_size,
                         kv_heads=kv_heads, head_dim=head_dim, dtype=k.dtype, device=device)
    cache = ServingCache(config, hot)
    rows_cache = cache.rows
    row_bytes = 2 * kv_heads * head_dim * k.element_size()
    tolerance = 3e-5 if k.dtype == torch.float32 else 0.008
    records, last_seen, gaps = [], {}, []
    previous_rows = previous_pages = None
    with torch.cuda.device(device), torch.cuda.stream(cache.compute):
        res = cache.reserve("trace", maximum, 1)
        try:
            pages = ceil(prefill / page_size)
            within, count, meta = cache.plan_prompt("trace", prefill)
            pad = pages * page_size - prefill
            padded = [torch.nn.functional.pad(t, (0, 0, 0, 0, 0, pad))
                      .view(pages, page_size, kv_heads, head_dim) for t in (k, v)]
            cache.append(0, padded[0], padded[1], within, count, meta)
            cache.advance("trace", prefill)
            # host block -> logical page, to report hot tags as logical tokens
            page_of = {int(block): page for page, block in enumerate(res.host[0])}
            cache.reset_stats()
            for step, event in enumerate(trace["events"]):
                q, new_k, new_v = (event[name].to(device) for name in ("q", "k", "v"))
                _, within, count, _, meta = cache.plan_decode(["trace"], [0])
                cache.append(0, new_k[None], new_v[None], within, count, meta)
                cache.advance("trace", 1)
                k, v = torch.cat((k, new_k)), torch.cat((v, new_v))
                length = k.shape[0]
                selection = Selection.from_tokens(event["positions"], length, page_size,
                                                  q.shape[0])
                rows = set().union(*selection.positions)
                selected_pages = {t // page_size for t in rows}
                before = rows_cache.row_stats.clone()
                actual = rows_cache.attention(q, "trace", 0, selection)
                expected = _selected_attention(q, k, v, selection)
                error = (actual.float() - expected.float()).abs().max().item()
                torch.testing.assert_close(actual, expected, atol=tolerance, rtol=tolerance)
                resident, hits, misses = (rows_cache.row_stats - before).cpu().tolist()
                if resident + hits + misses != len(rows):
                    raise RuntimeError("resolver counts do not cover the selected rows")
                for token in rows:
                    if token in last_seen:
                        gaps.append(step - last_seen[token])
                    last_seen[token] = step
                tags = rows_cache.tables["trace", 0].tags.cpu().tolist()
                slots = [None if tag < 0
                         else page_of[tag // page_size] * page_size + tag % page_size
                         for tag in tags]
                density = len(rows) / sum(min(page_size, length - p * page_size)
                                          for p in selected_pages)
                records.append({
                    "step": step,
                    "length": length,
                    "positions": selection.positions[0] if schema == 2
                    else selection.positions,
                    "union_rows": sorted(rows),
                    "selected_pages": sorted(selected_pages),
                    "row_jaccard": _jaccard(rows, previous_rows),
                    "page_jaccard": _jaccard(selected_pages, previous_pages),
                    "page_density": density,
                    "resident_hits": resident,
                    "hot_hits": hits,
                    "misses": misses,
                    "h2d_bytes": misses * row_bytes,
                    "hot_slots": slots,
                    "max_abs_error": error,
                })
                previous_rows, previous_pages = rows, selected_pages
            totals = cache.snapshot()["row_stats"]
        finally:
            cache.release_request("trace", wait=True)
    later = records[1:]
    nonresident = totals["hot_hits"] + totals["misses"]
    summary = {
        **totals,
        "hot_hit_rate": totals["hot_hits"] / nonresident if nonresident else None,
        "unique_rows": len(last_seen),
        "mean_reuse_gap_steps": mean(gaps) if gaps else None,
        "mean_row_jaccard": mean(r["row_jaccard"] for r in later) if later else None,
        "mean_page_jaccard": mean(r["page_jaccard"] for r in later) if later else None,
        "mean_page_density": mean(r["page_density"] for r in records),
        "max_abs_error": max(r["max_abs_error"] for r in records),
    }
    return {
        "schema_version": schema,
        "source": trace["source"],
        "device": str(device),
        "dtype": str(k.dtype),
        "page_size": page_size,
        "row_bytes": row_bytes,
        "max_union_rows": union_bound,
        "hot_rows": hot.hot_rows,
        "gpu_blocks": config.gpu_pages,
        "initial_residency": "history evicted; two tail pages retained; hot empty",
        "summary": summary,
        "events": records,
    }
