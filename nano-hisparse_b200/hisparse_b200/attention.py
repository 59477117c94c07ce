"""Row attention entry point (drop-in for nano_hisparse/attention.py:6-35)."""

from __future__ import annotations

import torch

from .row_kernels import attend_rows

BACKENDS = ("auto", "cuda")


@torch.inference_mode()
def row_attention(query, cache, request_id, layer, topk, backend="auto"):
    """Resolve the selection (lookups, LRU, miss gather) through
    ``cache.resolve`` and attend over the physical rows.

    Same checks and error messages as the reference; ``backend`` is "auto" or
    "cuda" (both run libhisparse: there is no Triton or torch path).
    """
    if backend not in BACKENDS:
        raise ValueError("invalid attention backend")
    if query.ndim != 2 or query.shape[1] != cache.config.head_dim:
        raise ValueError("invalid query shape")
    if query.shape[0] % cache.config.kv_heads or query.device != cache.pool.device:
        raise ValueError("query GQA/device mismatch")
    if topk.head_columns is not None and topk.head_columns.shape[0] != query.shape[0]:
        raise ValueError("selection must have one row per query head")
    if query.device.type != "cuda":
        raise ValueError("hisparse_b200 operators take CUDA tensors; there is no CPU path")
    with cache.resolve(request_id, layer, topk) as lease:
        rows = lease.plan.physical_rows
        if rows.ndim == 1:
            rows = rows[None, :].expand(query.shape[0], -1)
        return attend_rows(query, cache.pool, rows, cache.config)
