"""Batched decode hot path: B requests of one layer per launch.

The reference decodes requests one at a time (engine.py:76-126). Here one
``DecodeBatch.layer`` call runs the whole per-layer hot path for B requests
with four batched libhisparse launches — Quest selection, resolver, miss
gather, attention — and the same ordering protocol as ``RowCache.resolve``:
the gather runs on the transfer stream after the resolver and after the
previous readers of the layer's hot rows; attention waits for the gather.
Per-request tables stay separate tensors (the per-request API keeps working
on them); the batch passes them to the kernels as device pointer arrays built
once. No host synchronisation happens inside ``layer``.
"""

from __future__ import annotations

import torch

from . import _lib
from .cache import RowCache


def _pointers(tensors, device):
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device=device)


class _LayerState:
    def __init__(self, batch: DecodeBatch, layer: int):
        cache, ids, device = batch.cache, batch.request_ids, batch.device
        tables = [cache.tables[r, layer] for r in ids]
        self.tables = tables
        self.min_ptrs = _pointers([batch.minimum[r][layer] for r in ids], device)
        self.max_ptrs = _pointers([batch.maximum[r][layer] for r in ids], device)
        self.src_ptrs = _pointers([t.source for t in tables], device)
        self.res_ptrs = _pointers([t.resident for t in tables], device)
        self.hot_ptrs = _pointers([t.hot for t in tables], device)
        self.tag_ptrs = _pointers([t.tags for t in tables], device)
        self.lru_ptrs = _pointers([t.lru for t in tables], device)
        self.table_pages = min(int(t.source.numel()) for t in tables)
        self.lengths = torch.tensor([cache.lengths[r, layer] for r in ids], dtype=torch.int32,
                                    device=device)
        self.counts = torch.zeros((len(ids), 3), dtype=torch.int64, device=device)
        self.ready = None
        self.last_use = None


class DecodeBatch:
    """Decode hot path for a fixed set of requests of a RowCache.

    minimum / maximum: {request_id: [layers, pages, Hkv, D]} Quest metadata.
    """

    def __init__(self, cache: RowCache, request_ids, layers, minimum, maximum, top_pages,
                 q_heads, keep_sink=True):
        self.cache, self.request_ids = cache, list(request_ids)
        self.device, self.config = cache.device, cache.config
        self.minimum, self.maximum = minimum, maximum
        self.top_pages, self.keep_sink, self.q_heads = top_pages, keep_sink, q_heads
        self.batch = len(self.request_ids)
        cfg, b, dev = cache.config, self.batch, self.device
        self.width = top_pages * cfg.page_size
        if self.width > cache.hot_config.max_union_rows:
            raise ValueError("top-k width/union exceeds the admitted max_union_rows")
        self.max_pages = min(int(minimum[r].shape[1]) for r in self.request_ids)
        self.hot_rows = cache.hot_config.hot_rows
        self.layers = [_LayerState(self, layer) for layer in range(layers)]
        lib = _lib.load()
        self.tokens = torch.empty((b, self.width), dtype=torch.int32, device=dev)
        self.token_counts = torch.empty(b, dtype=torch.int32, device=dev)
        self.physical = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.miss_host = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.miss_device = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.quest_ws_bytes = lib.hs_quest_workspace_bytes(b, self.max_pages)
        self.quest_ws = _lib.workspace(self.quest_ws_bytes, dev, zeroed=True)
        self.resolve_ws_bytes = lib.hs_resolve_workspace_bytes(b, self.width, self.hot_rows)
        self.resolve_ws = _lib.workspace(self.resolve_ws_bytes, dev)
        self.attend_ws_bytes = lib.hs_attend_workspace_bytes(b, q_heads, cfg.kv_heads,
                                                             cfg.head_dim, self.width)
        self.attend_ws = _lib.workspace(self.attend_ws_bytes, dev)
        self.status = _lib.status_word(dev)
        self._dtype = _lib.dtype_code(cfg.dtype)
        self._row_bytes = cfg.row_bytes

    def set_lengths(self, layer: int, lengths: torch.Tensor):
        """Device int32 [B] context lengths of `layer` (after an append)."""
        self.layers[layer].lengths.copy_(lengths)

    def layer(self, layer: int, query: torch.Tensor, out: torch.Tensor | None = None,
              counts: torch.Tensor | None = None, timing: list | None = None) -> torch.Tensor:
        """Hot path of `layer` for query [B, Hq, D] (CUDA, contiguous) on the
        cache's compute stream; returns attention output [B, Hq, D].

        counts: optional int64 [B, 3] CUDA tensor receiving the resolver counts
        (default: the layer's own buffer, see last_counts). timing: optional
        list; when given, (name, start, end) CUDA-event pairs recorded on each
        launch's own stream are appended for the four stages."""
        cache, cfg, st, lib = self.cache, self.config, self.layers[layer], _lib.load()
        cache.check_stream()
        b, hq, d = query.shape
        if b != self.batch or hq != self.q_heads or d != cfg.head_dim:
            raise ValueError("query must be [batch, q_heads, head_dim]")
        if out is None:
            out = torch.empty_like(query)
        compute, transfer = cache.compute, cache.transfer
        stream = compute.cuda_stream
        status = self.status.data_ptr()
        if counts is None:
            counts = st.counts
        elif counts.shape != (b, 3) or counts.dtype != torch.int64 or not counts.is_contiguous():
            raise ValueError("counts must be a contiguous int64 [batch, 3] tensor")

        def mark(stream_):
            if timing is None:
                return None
            event = torch.cuda.Event(enable_timing=True)
            event.record(stream_)
            return event

        if st.ready is not None:
            compute.wait_event(st.ready)
        t0 = mark(compute)
        _lib.check(lib.hs_quest_select_batched(
            b, query.data_ptr(), hq * d, _lib.dtype_code(query.dtype), st.min_ptrs.data_ptr(),
            st.max_ptrs.data_ptr(), self._dtype, st.lengths.data_ptr(), hq, cfg.kv_heads, d,
            self.max_pages, cfg.page_size, self.top_pages, int(self.keep_sink),
            self.tokens.data_ptr(), self.width, self.token_counts.data_ptr(),
            _lib.ptr(self.quest_ws), self.quest_ws_bytes, status, stream))
        t1 = mark(compute)
        _lib.check(lib.hs_resolve_rows_batched(
            b, self.tokens.data_ptr(), self.width, st.src_ptrs.data_ptr(), st.res_ptrs.data_ptr(),
            st.table_pages, st.hot_ptrs.data_ptr(), cache.hot_blocks, st.tag_ptrs.data_ptr(),
            st.lru_ptrs.data_ptr(), self.hot_rows, st.lengths.data_ptr(), cfg.page_size,
            self.physical.data_ptr(), self.miss_host.data_ptr(), self.miss_device.data_ptr(),
            counts.data_ptr(), _lib.ptr(self.resolve_ws), self.resolve_ws_bytes, status,
            stream))
        t2 = mark(compute)
        resolved = torch.cuda.Event()
        resolved.record(compute)
        transfer.wait_event(resolved)
        if st.last_use is not None:
            transfer.wait_event(st.last_use)
        t3 = mark(transfer)
        _lib.check(lib.hs_gather_rows(
            cache.mapped.data_ptr(), cache.host.shape[0], cache.pool.data_ptr(),
            cache.pool.shape[0], self.miss_host.data_ptr(), self.miss_device.data_ptr(),
            b * self.width, self.width, cfg.page_size, self._row_bytes, status,
            transfer.cuda_stream))
        t4 = mark(transfer)
        st.ready = torch.cuda.Event()
        st.ready.record(transfer)
        compute.wait_event(st.ready)
        t5 = mark(compute)
        _lib.check(lib.hs_attend_rows(
            b, query.data_ptr(), hq * d, _lib.dtype_code(query.dtype), cache.pool.data_ptr(),
            cache.pool.shape[0], self._dtype, self.physical.data_ptr(), self.width, 0,
            self.width, out.data_ptr(), hq * d, hq, cfg.kv_heads, d, cfg.page_size,
            _lib.ptr(self.attend_ws), self.attend_ws_bytes, status, stream))
        if timing is not None:
            t6 = mark(compute)
            timing += [("quest", t0, t1), ("resolve", t1, t2), ("gather", t3, t4),
                       ("attend", t5, t6)]
        st.last_use = torch.cuda.Event()
        st.last_use.record(compute)
        return out

    def last_counts(self) -> torch.Tensor:
        """[layers, B, 3] resolver counts (resident hits, hot hits, misses) of
        the most recent call of each layer."""
        return torch.stack([st.counts for st in self.layers])
