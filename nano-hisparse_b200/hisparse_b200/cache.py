"""Device state of the hot path and the resolve ordering protocol.

``RowCache`` owns what the decode hot path reads and writes: the shared GPU
pool [gpu_pages, 2, P, Hkv, D], the pinned host store of the same layout
(read zero-copy by the gather), the per-(request, layer) ``LayerTables`` and
the per-request Quest metadata. ``resolve`` reproduces the stream/event
protocol of nano_hisparse/hybrid.py:412-469: the resolver runs on the compute
stream after the layer's previous gather, the gather runs on the transfer
stream after the resolver and after the previous readers of the hot rows, and
readers wait for the gather through the lease.

Placement (which pages are resident, which blocks form the hot region) is set
by the caller through ``add_layer``. The reference's residency policy —
admission credits, hot transitions, reclaim order — is host-side control with
no per-step arithmetic and stays with the reference's HybridKVCache, which can
drive libhisparse directly through ``hisparse_b200.plugin.install``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from .config import CacheConfig, HotConfig
from .row_index import LogicalTopK, resolve_rows
from .row_kernels import MappedHost, gather_rows


@dataclass
class LayerTables:
    """Per-(request, layer) device tables (hybrid.py:47-66): int32 source,
    resident, hot and tags; int64 lru permutation of the hot slots."""

    source: torch.Tensor
    resident: torch.Tensor
    hot: torch.Tensor
    tags: torch.Tensor
    lru: torch.Tensor
    blocks: list[int] = field(default_factory=list)
    ready: object = None
    last_use: object = None
    busy: bool = False


class RowLease:
    """Read lease on a layer's hot rows (hybrid.py:69-82)."""

    def __init__(self, cache: RowCache, tables: LayerTables):
        self.cache, self.tables, self.plan = cache, tables, None
        self.released, self.done = False, None
        tables.busy = True

    def _validate(self):
        if self.released:
            raise RuntimeError("lease already released")

    def wait(self):
        self._validate()
        if self.tables.ready is not None:
            self.cache.compute.wait_event(self.tables.ready)

    def release(self):
        self._validate()
        self.done = torch.cuda.Event()
        self.done.record(self.cache.compute)
        self.tables.last_use = self.done
        self.tables.busy = False
        self.released = True

    def __enter__(self):
        self.wait()
        return self

    def __exit__(self, *_):
        self.release()


class RowCache:
    def __init__(self, config: CacheConfig, hot: HotConfig, *, host=None):
        self.config, self.hot_config = config, hot
        self.device = torch.device(config.device)
        if self.device.type != "cuda":
            raise ValueError("RowCache lives on a CUDA device; there is no CPU path")
        if config.host_pages * config.page_size >= 2**31:
            raise ValueError("host row tags require int32 addresses")
        shape = (2, config.page_size, config.kv_heads, config.head_dim)
        self.pool = torch.empty((config.gpu_pages, *shape), dtype=config.dtype, device=self.device)
        self.host = host if host is not None else torch.empty(
            (config.host_pages, *shape), dtype=config.dtype, pin_memory=True)
        self.mapped = MappedHost(self.host)
        self.compute = torch.cuda.current_stream(self.device)
        self.transfer = torch.cuda.Stream(device=self.device)
        self.hot_blocks = hot.hot_blocks(config.page_size)
        self.tables: dict[tuple, LayerTables] = {}
        self.lengths: dict[tuple, int] = {}
        self.row_stats = torch.zeros(3, dtype=torch.int64, device=self.device)

    # -- placement ---------------------------------------------------------------
    def add_layer(self, request_id, layer, length, source, resident, hot_blocks):
        """Register one (request, layer): source[p] = host block of logical page
        p, resident[p] = pool block or -1, hot_blocks = the pool blocks of the
        hot region (ceil(hot_rows / P) of them). Hot contents start empty."""
        def table(values):
            return torch.as_tensor(values, dtype=torch.int32).to(self.device)

        if len(hot_blocks) != self.hot_blocks:
            raise ValueError(f"hot region needs {self.hot_blocks} blocks")
        h = self.hot_config.hot_rows
        tables = LayerTables(
            table(source), table(resident), table(hot_blocks),
            torch.full((h,), -1, dtype=torch.int32, device=self.device),
            torch.arange(h, dtype=torch.int64, device=self.device),
            blocks=[int(b) for b in hot_blocks])
        self.tables[request_id, layer] = tables
        self.lengths[request_id, layer] = int(length)
        return tables

    def set_length(self, request_id, layer, length):
        self.lengths[request_id, layer] = int(length)

    # -- hot path ----------------------------------------------------------------
    def check_stream(self):
        if torch.cuda.current_stream(self.device) != self.compute:
            raise RuntimeError("cache operations must use the construction compute stream")

    def resolve(self, request_id, layer, topk: LogicalTopK) -> RowLease:
        self.check_stream()
        topk.validate(self.device, self.hot_config.max_union_rows)
        tables = self.tables[request_id, layer]
        if tables.busy:
            raise RuntimeError("hot contents already leased by this layer")
        length = self.lengths[request_id, layer]
        if length < 1:
            raise ValueError("cannot resolve an empty history")
        lease = RowLease(self, tables)
        try:
            if tables.ready is not None:
                self.compute.wait_event(tables.ready)
            plan = resolve_rows(topk, tables.source, tables.resident, tables.hot, tables.tags,
                                tables.lru, length, self.config.page_size)
            self.row_stats.add_(plan.counts)
            resolved = torch.cuda.Event()
            resolved.record(self.compute)
            self.transfer.wait_event(resolved)
            if tables.last_use is not None:
                self.transfer.wait_event(tables.last_use)
            with torch.cuda.stream(self.transfer):
                gather_rows(self.mapped, self.pool, plan, self.config)
            tables.ready = torch.cuda.Event()
            tables.ready.record(self.transfer)
            plan.miss_host_rows.record_stream(self.transfer)
            plan.miss_device_rows.record_stream(self.transfer)
            lease.plan = plan
            return lease
        except Exception:
            lease.release()
            raise

    def attention(self, query, request_id, layer, selection, backend="auto"):
        from .attention import row_attention

        length = self.lengths[request_id, layer]
        if selection.length != length or selection.page_size != self.config.page_size:
            raise ValueError("selection has stale length or wrong page size")
        if selection.heads != query.shape[0]:
            raise ValueError("selection must have one row per query head")
        return row_attention(query, self, request_id, layer,
                             LogicalTopK.from_selection(selection, query.device), backend)

    # -- counters ----------------------------------------------------------------
    def reset_stats(self):
        self.row_stats.zero_()

    def snapshot(self):
        resident, hot, misses = self.row_stats.cpu().tolist()
        return {"row_stats": {"resident_hits": resident, "hot_hits": hot, "misses": misses,
                              "h2d_bytes": misses * 2 * self.config.row_bytes}}

    def synchronize(self):
        self.compute.synchronize()
        self.transfer.synchronize()
