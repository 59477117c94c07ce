"""KV append: new K/V rows into the pool, the pinned host mirror and the page
metadata (Quest K min/max and the mean-K summary) in one launch.

Drop-in for the tensor work of nano_hisparse/storage.py:264-330
(``HostStore.append``): per page chunk the reference copies the rows into
the pool block (:300-301), recomputes the fp32 mean of the block's valid K
rows (:305), folds the new K rows into the running min/max (:306-313) and
queues a device-to-host copy of the new rows on the transfer stream
(:316-323). Here ``hs_append_rows`` does all of it, writing the host rows
through the pinned store's device alias, so no separate copy is queued.

``append_page`` is the one-chunk form, ``append_chunks`` the batched form
(one chunk per request of a decode step) and ``host_store_append`` a
replacement for ``HostStore.append`` that keeps the reference's page
bookkeeping and ordering and runs each page chunk as one launch.
"""

from __future__ import annotations

import importlib

import torch

from . import _lib
from .row_kernels import MappedHost


def append_chunks(k, v, within, count, pool_block, pool, minimum_ptrs, maximum_ptrs,
                  summary_ptrs, config, host=None, host_block=None):
    """Append one page chunk per batch item b (all on the pool's device).

    k, v: [B, T, Hkv, D] in the KV dtype (chunk b uses rows 0..count[b]-1);
    within, count: int32 [B]; pool_block: int64 [B] (the page's pool block);
    minimum_ptrs / maximum_ptrs / summary_ptrs: int64 [B] device pointers to
    the page's [Hkv, D] bounds (KV dtype) and fp32 summary; host: MappedHost
    of the pinned store (or None) and host_block int64 [B] (-1: no mirror).
    Chunks of one call must touch distinct pages.
    """
    _lib.require_cuda(k, v, within, count, pool_block, pool, minimum_ptrs, maximum_ptrs,
                      summary_ptrs, host_block)
    if k.shape != v.shape or k.ndim != 4 or tuple(k.shape[2:]) != (config.kv_heads,
                                                                    config.head_dim):
        raise ValueError("expected matching [batch, tokens, kv_heads, head_dim] K/V")
    if k.dtype != pool.dtype or v.dtype != pool.dtype:
        raise ValueError("K/V dtype must match the cache")
    if k.stride() != v.stride() or not k.is_contiguous() or not v.is_contiguous():
        k, v = k.contiguous(), v.contiguous()
    batch = k.shape[0]
    if host_block is None:
        host_block = torch.full((batch,), -1, dtype=torch.int64, device=k.device)
    for name, t, dt in (("within", within, torch.int32), ("count", count, torch.int32),
                        ("pool_block", pool_block, torch.int64),
                        ("host_block", host_block, torch.int64),
                        ("minimum_ptrs", minimum_ptrs, torch.int64),
                        ("maximum_ptrs", maximum_ptrs, torch.int64),
                        ("summary_ptrs", summary_ptrs, torch.int64)):
        if t.dtype != dt or t.numel() != batch or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} tensor of {batch} entries")
    lib = _lib.load()
    _lib.check(lib.hs_append_rows(
        batch, k.data_ptr(), v.data_ptr(), k.stride(0), _lib.dtype_code(k.dtype),
        within.data_ptr(), count.data_ptr(), pool_block.data_ptr(), pool.data_ptr(),
        pool.shape[0], host_block.data_ptr(), None if host is None else host.data_ptr(),
        0 if host is None else host.tensor.shape[0], minimum_ptrs.data_ptr(),
        maximum_ptrs.data_ptr(), summary_ptrs.data_ptr(), config.kv_heads, config.head_dim,
        config.page_size, _lib.status_word(k.device).data_ptr(), _lib.stream_of(k.device)))


def append_page(pool, k, v, slot, within, minimum, maximum, summary, config, host=None,
                host_slot=-1):
    """One page chunk: rows within..within+len(k)-1 of pool block `slot` take
    k/v [count, Hkv, D]; minimum/maximum [Hkv, D] (KV dtype) and summary
    [Hkv, D] (fp32) are the page's metadata entries, updated in place; with a
    MappedHost `host`, host block `host_slot` receives the same rows."""
    _lib.require_cuda(pool, k, v, minimum, maximum, summary)
    count = k.shape[0]
    if count == 0:
        return
    if not (0 <= within and within + count <= config.page_size):
        raise ValueError("append chunk leaves its page")
    for name, t, dt in (("minimum", minimum, pool.dtype), ("maximum", maximum, pool.dtype),
                        ("summary", summary, torch.float32)):
        if (t.dtype != dt or tuple(t.shape) != (config.kv_heads, config.head_dim)
                or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous [kv_heads, head_dim] {dt} tensor")
    # the scalars travel in one small host->device copy: int64 slots, the first
    # two read as int32 (little endian: the value sits in the low half)
    meta = torch.tensor([within, count, slot, host_slot if host is not None else -1,
                         minimum.data_ptr(), maximum.data_ptr(), summary.data_ptr()],
                        dtype=torch.int64).to(pool.device, non_blocking=True)
    halves = meta.view(torch.int32)
    append_chunks(k.unsqueeze(0), v.unsqueeze(0), halves[0:1], halves[2:3], meta[2:3], pool,
                  meta[4:5], meta[5:6], meta[6:7], config, host, meta[3:4])


def host_store_append(store, request_id, layer, k, v, prepare_page, after_write=None):
    """``HostStore.append`` (nano_hisparse/storage.py:264-330) with each page
    chunk's tensor work in one ``hs_append_rows`` launch on the compute stream.

    The page bookkeeping, validation messages, lease handling and event
    ordering are the reference's: a chunk waits for the page's pending reads
    and host mirror (``ready``/``last_use``/``host_ready``) before it writes;
    ``page.ready`` and ``page.host_ready`` are both the launch's completion
    (the kernel writes the host rows itself).
    """
    store.check_stream()
    request = store.requests[request_id]
    cfg = store.config
    if not store.cuda:
        raise ValueError("hisparse_b200 append runs on CUDA caches only; there is no CPU path")
    if not 0 <= layer < request.layers:
        raise ValueError("invalid layer")
    expected = (cfg.kv_heads, cfg.head_dim)
    if k.ndim != 3 or k.shape != v.shape or tuple(k.shape[1:]) != expected:
        raise ValueError(f"expected matching [tokens, {expected[0]}, {expected[1]}] K/V")
    if k.device != store.pool.device or v.device != store.pool.device:
        raise ValueError("K/V must be on the cache device")
    if k.dtype != cfg.dtype or v.dtype != cfg.dtype:
        raise ValueError("K/V dtype must match the cache")
    # the reference's own exception class, so its callers' handlers still match
    capacity_error = importlib.import_module(type(store).__module__).CapacityError
    start = request.lengths[layer]
    if start + len(k) > request.max_tokens:
        raise capacity_error("request exceeds its reserved host capacity")
    if any(key[0] == request_id and key[1] == layer for key in store.pinned):
        raise RuntimeError("cannot append while this layer has active attention leases")
    if len(store.pinned) >= store.budget:
        raise capacity_error("no slot available for append")
    mapped = getattr(store, "_hs_mapped_host", None)
    if mapped is None or mapped.tensor is not store.host:
        mapped = MappedHost(store.host)
        store._hs_mapped_host = mapped
    offset = 0
    while offset < len(k):
        position = start + offset
        index, within = divmod(position, cfg.page_size)
        page = store.materialize(request_id, layer, index)
        count = min(cfg.page_size - within, len(k) - offset)
        lease = prepare_page(page)
        if lease is not None:
            lease.wait()
        for event in (page.ready, page.last_use, page.host_ready):
            store.wait(store.compute, event)
        with store.context(store.compute):
            append_page(store.pool, k[offset:offset + count].contiguous(),
                        v[offset:offset + count].contiguous(), page.slot, within,
                        request.minimum[layer, index], request.maximum[layer, index],
                        request.summaries[layer, index], cfg, mapped, page.host_slot)
        page.valid_tokens = within + count
        page.content_version += 1
        page.sealed = page.valid_tokens == cfg.page_size
        page.ready = store.event(store.compute)
        page.location = type(page.location)("resident")
        page.host_ready = page.ready
        page.host_enqueued_version = page.content_version
        store.stats["d2h_bytes"] += store.page_bytes * count // cfg.page_size
        if lease is not None:
            lease.release()
        if after_write is not None:
            after_write(page)
        offset += count
    request.lengths[layer] += len(k)
