"""Shared token selection and the Quest page selector.

Drop-in for nano_hisparse/selection.py: ``Selection`` (selection.py:11-66) keeps
the reference's fields, constructors, validation and messages;
``quest_selection`` (selection.py:69-91) keeps its signature and result, but
runs as one fused scoring + top-k + expansion pass on the GPU
(``hs_quest_select``) and returns a *device-form* Selection: the selected
tokens stay on the GPU, and ``LogicalTopK.from_selection`` consumes them
without the reference's ``.tolist()`` synchronisation and host->device copy.
Reading ``selection.positions`` materialises the per-head tuples on demand.
"""

from __future__ import annotations

from math import ceil

import torch

from . import _lib


class Selection:
    """One shared token set per query (or, for legacy callers, one per head).

    ``positions`` is a tuple with one sorted tuple of logical tokens per query
    head. A device-form selection holds the shared tokens as an int32 CUDA
    tensor padded with -1 (``device_tokens``) and fills ``positions`` lazily.
    """

    __slots__ = ("_positions", "length", "page_size", "source", "_device", "_heads")

    def __init__(self, positions, length, page_size, source, *, device_tokens=None, heads=None):
        self._positions = positions
        self.length, self.page_size, self.source = length, page_size, source
        self._device, self._heads = device_tokens, heads

    # -- reference constructors (selection.py:21-62) -----------------------------
    @classmethod
    def from_tokens(cls, rows, length, page_size, heads, source="external"):
        if length < 1 or page_size < 1 or heads < 1:
            raise ValueError("selection dimensions must be positive")
        if isinstance(rows, torch.Tensor):
            rows = rows.cpu().tolist()
        rows = list(rows)
        if rows and isinstance(rows[0], int):
            rows = [rows]
        if len(rows) == 1:
            rows = rows * heads
        if len(rows) != heads:
            raise ValueError("selection must be shared or have one row per query head")
        canonical = []
        for row in rows:
            if not isinstance(row, (list, tuple)):
                raise TypeError("selection rows must be integer sequences")
            for t in row:
                if not isinstance(t, int) or t < -1 or t >= length:
                    raise ValueError("token selection contains noncausal or invalid positions")
            values = tuple(sorted(set(row) - {-1}))
            if not values:
                raise ValueError("each query head must select at least one token")
            canonical.append(values)
        return cls(tuple(canonical), length, page_size, source)

    @classmethod
    def from_pages(cls, rows, length, page_size, heads, source="pages"):
        if isinstance(rows, torch.Tensor):
            rows = rows.cpu().tolist()
        rows = list(rows)
        if rows and isinstance(rows[0], int):
            rows = [rows]
        count = ceil(length / page_size)
        for row in rows:
            for p in row:
                if p < 0 or p >= count:
                    raise ValueError("invalid logical page")
        tokens = [
            [t for p in row for t in range(p * page_size, min((p + 1) * page_size, length))]
            for row in rows
        ]
        return cls.from_tokens(tokens, length, page_size, heads, source)

    # -- device form ------------------------------------------------------------
    @classmethod
    def from_device(cls, tokens: torch.Tensor, length, page_size, heads, source="quest"):
        """Shared selection whose sorted tokens (-1 padded) live on the GPU."""
        return cls(None, length, page_size, source, device_tokens=tokens, heads=heads)

    @property
    def device_tokens(self) -> torch.Tensor | None:
        return self._device

    @property
    def positions(self):
        if self._positions is None:
            shared = tuple(t for t in self._device.tolist() if t >= 0)
            self._positions = (shared,) * self._heads
        return self._positions

    @property
    def heads(self) -> int:
        return self._heads if self._positions is None else len(self._positions)

    @property
    def pages(self):
        return sorted({t // self.page_size for row in self.positions for t in row})

    def __eq__(self, other):
        if not isinstance(other, Selection):
            return NotImplemented
        return (self.positions, self.length, self.page_size, self.source) == (
            other.positions, other.length, other.page_size, other.source)

    def __hash__(self):
        return hash((self.positions, self.length, self.page_size, self.source))

    def __repr__(self):
        return (f"Selection(positions={self.positions!r}, length={self.length}, "
                f"page_size={self.page_size}, source={self.source!r})")


def quest_selection(query, minimum, maximum, length, page_size, top_pages, keep_sink=True):
    """Quest bounds averaged over query heads, then one shared page top-k.

    score[p] = mean_h sum_d max(q[h,d]*min[p,h/g,d], q[h,d]*max[p,h/g,d]); the
    tail page (and page 0 when keep_sink and top_pages > 1) is always kept.
    Same contract as nano_hisparse/selection.py:69-91; equal scores keep the
    lower page. query [Hq, D]; minimum/maximum [>= pages, Hkv, D] CUDA tensors.
    """
    count = ceil(length / page_size)
    if top_pages < 1 or query.shape[0] % minimum.shape[1]:
        raise ValueError("invalid page budget or GQA shape")
    heads = query.shape[0]
    if top_pages >= count:
        return Selection.from_pages(list(range(count)), length, page_size, heads, "quest")
    _lib.require_cuda(query, minimum, maximum)
    if minimum.shape != maximum.shape or minimum.dtype != maximum.dtype:
        raise ValueError("minimum and maximum metadata must match")
    if minimum.ndim != 3 or query.ndim != 2 or minimum.shape[2] != query.shape[1]:
        raise ValueError("expected query [heads, dim] and metadata [pages, kv_heads, dim]")
    if minimum.shape[0] < count:
        raise ValueError("metadata has fewer pages than the selection length")
    lib = _lib.load()
    device = query.device
    query, minimum, maximum = query.contiguous(), minimum.contiguous(), maximum.contiguous()
    width = top_pages * page_size
    tokens = torch.empty(width, dtype=torch.int32, device=device)
    counter = torch.empty(1, dtype=torch.int32, device=device)
    nbytes = lib.hs_quest_workspace_bytes(1, minimum.shape[0])
    ws = _lib.workspace(nbytes, device, zeroed=True)
    _lib.check(lib.hs_quest_select(
        query.data_ptr(), _lib.dtype_code(query.dtype), minimum.data_ptr(), maximum.data_ptr(),
        _lib.dtype_code(minimum.dtype), query.shape[0], minimum.shape[1], query.shape[1],
        minimum.shape[0], length, page_size, top_pages, int(bool(keep_sink)), tokens.data_ptr(),
        width, counter.data_ptr(), _lib.ptr(ws), nbytes, _lib.status_word(device).data_ptr(),
        _lib.stream_of(device)))
    return Selection.from_device(tokens, length, page_size, heads, "quest")
