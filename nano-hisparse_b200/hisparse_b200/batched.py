"""Batched decode hot path: B requests of one layer per launch.

The reference decodes requests one at a time (engine.py:76-126). Here one
``DecodeBatch.layer`` call runs the whole per-layer hot path for B requests
with batched libhisparse launches — Quest selection, resolver, miss gather,
attention — ordered like ``RowCache.resolve`` (the gather runs on the
transfer stream after the resolver and after the previous readers of the
layer's hot rows) with one refinement: attention is split in two phases. The
first attends over the rows that need no gather (resident and hot hits, the
resolver's ready list) on the compute stream while the gather streams the
misses in; the second attends over the gathered rows after the gather, and a
merge combines both. The gather only writes hot slots that no selected row
occupies, so the first phase never reads a row being written.
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
        # Requests may have tables of different sizes (each covers its own pages):
        # the kernels read a request's tables only below ceil(length / P), so the
        # batch passes the largest capacity and every request is checked here.
        page = cache.config.page_size
        for r, t in zip(ids, tables):
            pages = -(-cache.lengths[r, layer] // page)
            own = min(int(t.source.numel()), int(t.resident.numel()),
                      int(batch.minimum[r][layer].shape[0]), int(batch.maximum[r][layer].shape[0]))
            if pages > own:
                raise ValueError(f"request {r!r} layer {layer}: {pages} pages of history exceed "
                                 f"its tables ({own} pages)")
        self.table_pages = max(int(t.source.numel()) for t in tables)
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
                 q_heads, keep_sink=True, streams=None, group=None):
        """streams: optional (compute, transfer) CUDA streams for this batch; by
        default the cache's. Batches over disjoint requests with their own
        compute streams run concurrently (micro-batch pipelining: one batch's
        gather overlaps another's selection, resolve and attention); sharing one
        transfer stream makes their gathers take the host link in turn.

        group: a process group over which the requests' KV heads are split
        (configuration 5). This rank then holds kv_heads of the cache config
        and q_heads of the queries; the page selection becomes the
        head-sharded one (partial scores, an all-gather over `group`, the
        shared top-k), identical on every rank, and resolve, gather and
        attention run over this rank's head slice."""
        self.cache, self.request_ids = cache, list(request_ids)
        if streams is None:
            self.compute, self.transfer = cache.compute, cache.transfer
        else:
            self.compute, self.transfer = streams
        self.device, self.config = cache.device, cache.config
        self.minimum, self.maximum = minimum, maximum
        self.top_pages, self.keep_sink, self.q_heads = top_pages, keep_sink, q_heads
        self.batch = len(self.request_ids)
        cfg, b, dev = cache.config, self.batch, self.device
        self.width = top_pages * cfg.page_size
        if self.width > cache.hot_config.max_union_rows:
            raise ValueError("top-k width/union exceeds the admitted max_union_rows")
        self.max_pages = max(int(minimum[r].shape[1]) for r in self.request_ids)
        self.hot_rows = cache.hot_config.hot_rows
        self.layers = [_LayerState(self, layer) for layer in range(layers)]
        lib = _lib.load()
        self.tokens = torch.empty((b, self.width), dtype=torch.int32, device=dev)
        self.token_counts = torch.empty(b, dtype=torch.int32, device=dev)
        self.physical = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.miss_host = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.miss_device = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.ready = torch.empty((b, self.width), dtype=torch.int64, device=dev)
        self.quest_ws_bytes = lib.hs_quest_workspace_bytes(b, self.max_pages)
        self.quest_ws = _lib.workspace(self.quest_ws_bytes, dev, zeroed=True)
        self.resolve_ws_bytes = lib.hs_resolve_workspace_bytes(b, self.width, self.hot_rows)
        self.resolve_ws = _lib.workspace(self.resolve_ws_bytes, dev)
        self.attend_ws_bytes = lib.hs_attend_workspace_bytes(b, q_heads, cfg.kv_heads,
                                                             cfg.head_dim, self.width)
        self.attend_ws = _lib.workspace(self.attend_ws_bytes, dev)
        self.group, self.shards = group, 1
        if group is not None:
            import torch.distributed as dist

            from .sharded import same_on_every_rank

            self.shards = dist.get_world_size(group)
            # the per-layer all-gather exchanges [batch * max_pages] partials:
            # every rank must hold the same shape
            if not same_on_every_rank(group, (b, self.max_pages, top_pages), dev):
                raise ValueError("ranks disagree on the batch size, the metadata table "
                                 "length or the page budget of a head-sharded batch")
            self.partial = torch.empty(b * self.max_pages, dtype=torch.float32, device=dev)
            self.partials = torch.empty((self.shards, b * self.max_pages), dtype=torch.float32,
                                        device=dev)
        self.status = _lib.status_word(dev)
        self._dtype = _lib.dtype_code(cfg.dtype)
        self._row_bytes = cfg.row_bytes

    def set_lengths(self, layer: int, lengths: torch.Tensor):
        """Device int32 [B] context lengths of `layer` (after an append). Each
        request's pages of history must stay within its own tables (checked on
        the host when the batch is built; a device-side length past them is
        flagged HS_DEV_PAGES_EXCEED_TABLE only against the batch's largest)."""
        self.layers[layer].lengths.copy_(lengths)

    def bind_lengths(self, lengths: torch.Tensor):
        """Makes every layer read its context lengths from `lengths` (device
        int32 [B]): in decode all layers of a request have the same length, so
        a decode loop updates one tensor per step instead of one per layer."""
        if (lengths.dtype != torch.int32 or tuple(lengths.shape) != (self.batch,)
                or lengths.device != self.device or not lengths.is_contiguous()):
            raise ValueError("lengths must be a contiguous int32 [batch] tensor on the "
                             "batch's device")
        for st in self.layers:
            st.lengths = lengths

    def layer(self, layer: int, query: torch.Tensor, out: torch.Tensor | None = None,
              counts: torch.Tensor | None = None, timing: list | None = None,
              stages=None, serial: bool = False, part: str = "all",
              positions: torch.Tensor | None = None) -> torch.Tensor:
        """Hot path of `layer` for query [B, Hq, D] (CUDA, contiguous) on the
        cache's compute stream; returns attention output [B, Hq, D].

        counts: optional int64 [B, 3] CUDA tensor receiving the resolver counts
        (default: the layer's own buffer, see last_counts). timing: optional
        list; when given, (name, start, end) CUDA-event pairs recorded on each
        launch's own stream are appended for the stages ("quest", "resolve",
        "gather", "attend_ready", "attend_gathered", "merge"; all, or only those
        in `stages`). The events are external, so they also time graph replays
        when the call is captured. serial: run the ready-row attention after
        the gather instead of beside it (each stage then runs alone, for
        per-stage timing).

        part: "all" (default), or "head" / "tail" — the layer in two pieces
        split at the exchange: "head" runs up to this rank's partial scores
        (with a group) or the whole selection (without), "tail" everything
        after, and neither runs the all-gather: the caller issues it between
        them on the stream that orders the two (DecodeGraph's segmented
        replay).

        positions: optional int32 [B, width] CUDA tensor of logical token
        positions (-1 padded, width = top_pages * page_size) to resolve in
        place of the Quest selection, which is then skipped (an externally
        chosen selection, e.g. a replayed trace)."""
        if part not in ("all", "head", "tail"):
            raise ValueError("part must be 'all', 'head' or 'tail'")
        cfg, st, compute = self.config, self.layers[layer], self.compute
        if torch.cuda.current_stream(self.device) != compute:
            raise RuntimeError("DecodeBatch.layer must run on the batch's compute stream")
        b, hq, d = query.shape
        if b != self.batch or hq != self.q_heads or d != cfg.head_dim:
            raise ValueError("query must be [batch, q_heads, head_dim]")
        if out is None:
            out = torch.empty_like(query)
        if counts is None:
            counts = st.counts
        elif counts.shape != (b, 3) or counts.dtype != torch.int64 or not counts.is_contiguous():
            raise ValueError("counts must be a contiguous int64 [batch, 3] tensor")

        def mark(stream_, *names):
            if timing is None or (stages is not None and not any(n in stages for n in names)):
                return None
            event = torch.cuda.Event(enable_timing=True, external=True)
            event.record(stream_)
            return event

        if positions is not None:
            if part != "all":
                raise ValueError("positions replace the whole selection: part must be 'all'")
            if (positions.shape != (b, self.width) or positions.dtype != torch.int32
                    or positions.device != self.device or not positions.is_contiguous()):
                raise ValueError("positions must be a contiguous int32 [batch, width] tensor "
                                 "on the batch's device")
            if st.ready is not None:
                compute.wait_event(st.ready)
            t1 = mark(compute, "resolve")
            self._rest(layer, query, out, counts, timing, stages, serial, mark, None, t1,
                       positions.data_ptr())
            st.last_use = torch.cuda.Event()
            st.last_use.record(compute)
            return out
        t0 = None
        if part != "tail":
            t0 = self._select_head(layer, query, mark)
        if part == "head":
            return out
        if part == "all":
            self.exchange()
        if self.group is not None:
            self._select_tail(layer, query)
        t1 = mark(compute, "quest", "resolve") if part == "all" else mark(compute, "resolve")
        self._rest(layer, query, out, counts, timing, stages, serial, mark, t0, t1,
                   self.tokens.data_ptr())
        st.last_use = torch.cuda.Event()
        st.last_use.record(compute)
        return out

    def exchange(self):
        """All-gather of the partial scores over the group, on the current
        stream (nothing without a group)."""
        if self.group is not None:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.partials, self.partial, group=self.group)

    def _select_head(self, layer, query, mark):
        """The selection without a group; this rank's head sums with one."""
        cfg, st, lib = self.config, self.layers[layer], _lib.load()
        b, hq, d = query.shape
        compute, stream, status = self.compute, self.compute.cuda_stream, self.status.data_ptr()
        if st.ready is not None:
            compute.wait_event(st.ready)
        t0 = mark(compute, "quest")
        if self.group is None:
            _lib.check(lib.hs_quest_select_batched(
                b, query.data_ptr(), hq * d, _lib.dtype_code(query.dtype), st.min_ptrs.data_ptr(),
                st.max_ptrs.data_ptr(), self._dtype, st.lengths.data_ptr(), hq, cfg.kv_heads, d,
                self.max_pages, cfg.page_size, self.top_pages, int(self.keep_sink),
                self.tokens.data_ptr(), self.width, self.token_counts.data_ptr(),
                _lib.ptr(self.quest_ws), self.quest_ws_bytes, status, stream))
        else:
            # this rank's head sums; the exchange and the shared top-k follow
            _lib.check(lib.hs_quest_partial_scores_batched(
                b, query.data_ptr(), hq * d, _lib.dtype_code(query.dtype), st.min_ptrs.data_ptr(),
                st.max_ptrs.data_ptr(), self._dtype, st.lengths.data_ptr(), hq, cfg.kv_heads, d,
                self.max_pages, cfg.page_size, self.partial.data_ptr(), status, stream))
        return t0

    def _select_tail(self, layer, query):
        """Every rank's head sums in shard order -> the shared top-k."""
        cfg, st, lib = self.config, self.layers[layer], _lib.load()
        b, hq = query.shape[0], query.shape[1]
        _lib.check(lib.hs_quest_select_partials(
            self.shards, self.partials.data_ptr(), b, st.lengths.data_ptr(), hq * self.shards,
            self.max_pages, cfg.page_size, self.top_pages, int(self.keep_sink),
            self.tokens.data_ptr(), self.width, self.token_counts.data_ptr(),
            _lib.ptr(self.quest_ws), self.quest_ws_bytes, self.status.data_ptr(),
            self.compute.cuda_stream))

    def _rest(self, layer, query, out, counts, timing, stages, serial, mark, t0, t1, tokens):
        """Resolve, gather, both attention phases and the merge of `layer`."""
        cache, cfg, st, lib = self.cache, self.config, self.layers[layer], _lib.load()
        b, hq, d = query.shape
        compute, transfer = self.compute, self.transfer
        stream, status = compute.cuda_stream, self.status.data_ptr()
        _lib.check(lib.hs_resolve_rows_batched(
            b, tokens, self.width, st.src_ptrs.data_ptr(), st.res_ptrs.data_ptr(),
            st.table_pages, st.hot_ptrs.data_ptr(), cache.hot_blocks, st.tag_ptrs.data_ptr(),
            st.lru_ptrs.data_ptr(), self.hot_rows, st.lengths.data_ptr(), cfg.page_size,
            self.physical.data_ptr(), self.miss_host.data_ptr(), self.miss_device.data_ptr(),
            counts.data_ptr(), self.ready.data_ptr(), _lib.ptr(self.resolve_ws),
            self.resolve_ws_bytes, status, stream))
        t2 = mark(compute, "resolve")
        resolved = torch.cuda.Event()
        resolved.record(compute)
        transfer.wait_event(resolved)
        if st.last_use is not None:
            transfer.wait_event(st.last_use)
        t3 = mark(transfer, "gather")
        _lib.check(lib.hs_gather_rows(
            cache.mapped.data_ptr(), cache.host.shape[0], cache.pool.data_ptr(),
            cache.pool.shape[0], self.miss_host.data_ptr(), self.miss_device.data_ptr(),
            b * self.width, self.width, cfg.page_size, self._row_bytes, status,
            transfer.cuda_stream))
        t4 = mark(transfer, "gather")
        st.ready = torch.cuda.Event()
        st.ready.record(transfer)
        # phase 0: rows that need no gather, concurrently with the gather
        if serial:
            compute.wait_event(st.ready)
        t5 = mark(compute, "attend_ready")
        common = (b, query.data_ptr(), hq * d, _lib.dtype_code(query.dtype), cache.pool.data_ptr(),
                  cache.pool.shape[0], self._dtype)
        _lib.check(lib.hs_attend_rows_phase(
            *common, self.ready.data_ptr(), self.width, self.width, counts.data_ptr(), 3, 0, 2, 0,
            hq, cfg.kv_heads, d, cfg.page_size, _lib.ptr(self.attend_ws), self.attend_ws_bytes,
            status, stream))
        t6 = mark(compute, "attend_ready")
        # phase 1: the gathered rows, then the merge
        compute.wait_event(st.ready)
        t7 = mark(compute, "attend_gathered")
        _lib.check(lib.hs_attend_rows_phase(
            *common, self.miss_device.data_ptr(), self.width, self.width, counts.data_ptr(), 3, 2,
            1, 1, hq, cfg.kv_heads, d, cfg.page_size, _lib.ptr(self.attend_ws),
            self.attend_ws_bytes, status, stream))
        t8 = mark(compute, "attend_gathered", "merge")
        _lib.check(lib.hs_attend_merge(
            b, 2, out.data_ptr(), hq * d, _lib.dtype_code(query.dtype), hq, cfg.kv_heads, d,
            self.width, _lib.ptr(self.attend_ws), self.attend_ws_bytes, status, stream))
        if timing is not None:
            t9 = mark(compute, "merge")
            for name, a, b_ in (("quest", t0, t1), ("resolve", t1, t2), ("gather", t3, t4),
                                ("attend_ready", t5, t6), ("attend_gathered", t7, t8),
                                ("merge", t8, t9)):
                if a is not None and b_ is not None:
                    timing.append((name, a, b_))

    def last_counts(self) -> torch.Tensor:
        """[layers, B, 3] resolver counts (resident hits, hot hits, misses) of
        the most recent call of each layer."""
        return torch.stack([st.counts for st in self.layers])


class DecodeGraph:
    """One decode step — every layer of every micro-batch — captured once as a
    CUDA graph and replayed per step, so the host issues one launch per step
    instead of ~six kernels and a dozen events per (micro-batch, layer).

    batches: DecodeBatch objects over disjoint requests, each with its own
    streams. Inputs and outputs are static buffers: ``queries[i]`` is
    [layers, B_i, Hq, D] for batch i, ``outputs[i]`` the same shape, and
    ``counts[i]`` [layers, B_i, 3] receives the resolver counts of the last
    replay. Fill ``queries`` (on the replaying stream), call ``replay()``.
    The step's stream/event ordering is that of DecodeBatch.layer; replays on
    one stream are serialised, which orders a layer's gather after the
    previous step's readers of its hot rows.
    """

    def __init__(self, batches, layers: int, timing=False, segmented=None):
        """timing: False, True (every stage) or an iterable of stage names of
        DecodeBatch.layer; the captured step then records timing events, and
        after a replay ``self.timing`` holds that replay's (name, start, end)
        pairs for every (layer, batch).

        segmented: capture each layer as two graphs split at the exchange
        (DecodeBatch.layer's "head" and "tail") and issue the batches'
        all-gathers between them at replay, so no collective is captured.
        Default: when a batch has a process group (head-sharded selection).
        A replay then costs the host two graph launches and one all-gather
        per layer."""
        self.batches, self.layers = list(batches), layers
        if segmented is None:
            segmented = any(bt.group is not None for bt in self.batches)
        self.segmented = bool(segmented)
        if self.segmented and timing:
            raise ValueError("a segmented step graph records no per-stage timing")
        for bt in self.batches:
            if bt.compute.cuda_stream == 0 or bt.transfer.cuda_stream == 0:
                raise ValueError("DecodeGraph needs batches on created streams, not the default "
                                 "stream (pass streams=(compute, transfer) to DecodeBatch)")
        b0 = self.batches[0]
        self.device = b0.device
        dt = b0.config.dtype
        self.queries = [torch.zeros((layers, bt.batch, bt.q_heads, bt.config.head_dim),
                                    dtype=dt, device=self.device) for bt in self.batches]
        self.outputs = [torch.empty_like(q) for q in self.queries]
        self.counts = [torch.zeros((layers, bt.batch, 3), dtype=torch.int64, device=self.device)
                       for bt in self.batches]
        self.timing = [] if timing else None
        self.stages = None if timing is True or not timing else frozenset(timing)
        # two eager steps settle lazy state (function attributes, workspaces)
        # before capture; the events they leave behind are dropped
        for _ in range(2):
            self._run(None)
        torch.cuda.synchronize(self.device)
        self._reset_events()
        if self.segmented:
            # thread-local capture: a process group's watchdog thread may query
            # its collectives' events while a piece is being captured
            self.graph, self.segments, pool = None, [], None
            for layer in range(layers):
                pair = []
                for part in ("head", "tail"):
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, pool=pool, capture_error_mode="thread_local"):
                        self._run_part(layer, part)
                    pool = graph.pool() if pool is None else pool
                    pair.append(graph)
                self.segments.append(tuple(pair))
        else:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._run(self.timing)
        self._reset_events()

    def _reset_events(self):
        for bt in self.batches:
            for st in bt.layers:
                st.ready = st.last_use = None

    def _run(self, timing):
        caller = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(caller)
        for bt in self.batches:
            bt.compute.wait_event(start)
        for layer in range(self.layers):
            for i, bt in enumerate(self.batches):
                with torch.cuda.stream(bt.compute):
                    bt.layer(layer, self.queries[i][layer], self.outputs[i][layer],
                             self.counts[i][layer], timing, self.stages)
        for bt in self.batches:
            done = torch.cuda.Event()
            done.record(bt.compute)
            caller.wait_event(done)

    def _run_part(self, layer, part):
        """One piece of one layer for every batch, forked from and joined back
        to the current (capturing) stream."""
        caller = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(caller)
        for bt in self.batches:
            bt.compute.wait_event(start)
        for i, bt in enumerate(self.batches):
            with torch.cuda.stream(bt.compute):
                bt.layer(layer, self.queries[i][layer], self.outputs[i][layer],
                         self.counts[i][layer], part=part)
        for bt in self.batches:
            done = torch.cuda.Event()
            done.record(bt.compute)
            caller.wait_event(done)

    def replay(self):
        """One step on the current stream."""
        if not self.segmented:
            self.graph.replay()
            return
        for head, tail in self.segments:
            head.replay()
            for bt in self.batches:  # the same order on every rank
                bt.exchange()
            tail.replay()
