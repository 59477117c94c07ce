"""Logical selection -> physical rows: LogicalTopK, RowPlan and the resolver.

Drop-in for nano_hisparse/row_index.py. ``resolve_rows`` keeps the reference's
signature, results and in-place update of ``tags``/``lru`` (row_index.py:62-140)
but runs as a single CUDA kernel (``hs_resolve_rows``): one CTA per request,
no host round trip, capturable in a CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .selection import Selection


@dataclass(frozen=True)
class LogicalTopK:
    """Shared [K] token positions, plus legacy per-head columns into them."""

    positions: torch.Tensor
    head_columns: torch.Tensor | None = None

    @classmethod
    def from_selection(cls, selection: Selection, device):
        """Same result as row_index.py:20-34. A device-form selection (from
        quest_selection) is used in place: no synchronisation, no copy."""
        tokens = getattr(selection, "device_tokens", None)
        if tokens is not None and tokens.device == torch.device(device):
            return cls(tokens)
        rows = selection.positions
        if all(row == rows[0] for row in rows):
            return cls(torch.tensor(rows[0], dtype=torch.int32, device=device))
        union = sorted({p for row in rows for p in row})
        column = {token: i for i, token in enumerate(union)}
        width = max(len(row) for row in rows)
        matrix = [[column[p] for p in row] + [-1] * (width - len(row)) for row in rows]
        return cls(torch.tensor(union, dtype=torch.int32, device=device),
                   torch.tensor(matrix, dtype=torch.int64, device=device))

    def validate(self, device, maximum):
        """row_index.py:36-51: same checks and messages."""
        if (
            self.positions.ndim != 1
            or self.positions.numel() < 1
            or self.positions.dtype not in (torch.int32, torch.int64)
            or self.positions.device != torch.device(device)
        ):
            raise ValueError("logical top-k must be a nonempty device integer vector")
        if self.positions.numel() > maximum:
            raise ValueError("top-k width/union exceeds the admitted max_union_rows")
        if self.head_columns is not None and (
            self.head_columns.ndim != 2
            or self.head_columns.device != torch.device(device)
            or self.head_columns.dtype != torch.int64
        ):
            raise ValueError("head columns must be a device int64 matrix")


@dataclass
class RowPlan:
    physical_rows: torch.Tensor  # shared [K] or per-head [H, K], -1 padding
    miss_host_rows: torch.Tensor  # fixed-width compact prefix; -1 after misses
    miss_device_rows: torch.Tensor
    counts: torch.Tensor  # unique resident hits, hot hits, misses


def _as(t: torch.Tensor, dtype):
    return t if (t.dtype == dtype and t.is_contiguous()) else t.to(dtype).contiguous()


def resolve_rows(topk, source_table, resident_table, hot_table, tags, lru, length, page_size):
    """Resident lookup first; every selected hot hit is protected before any
    eviction; misses take the least-recently-used unprotected slots.

    Results equal nano_hisparse/row_index.py:62-140: physical rows in input
    order (repeats and invalid inputs -> -1), the compact miss plan in sorted
    logical order, counts = [resident hits, hot hits, misses]; ``tags`` and
    ``lru`` are updated in place. Tables may be int32 or int64 CUDA tensors.
    """
    positions = topk.positions
    _lib.require_cuda(positions, source_table, resident_table, hot_table, tags, lru)
    if positions.ndim != 1 or positions.numel() < 1:
        raise ValueError("logical top-k must be a nonempty device integer vector")
    device = positions.device
    lib = _lib.load()
    pos = positions if positions.dtype in (torch.int32, torch.int64) else positions.long()
    pos = pos.contiguous()
    source = _as(source_table, torch.int32)
    resident = _as(resident_table, torch.int32)
    hot = _as(hot_table, torch.int32)
    tags_k = _as(tags, torch.int32)
    lru_k = _as(lru, torch.int64)
    if resident.numel() < source.numel():
        raise ValueError("resident table is shorter than the source table")
    k, h = pos.numel(), tags.numel()
    physical = torch.empty(k, dtype=torch.int64, device=device)
    miss_host = torch.empty(k, dtype=torch.int64, device=device)
    miss_device = torch.empty(k, dtype=torch.int64, device=device)
    counts = torch.empty(3, dtype=torch.int64, device=device)
    columns = topk.head_columns
    head_rows = None
    if columns is not None:
        columns = _as(columns, torch.int64)
        head_rows = torch.empty(columns.shape, dtype=torch.int64, device=device)
    nbytes = lib.hs_resolve_workspace_bytes(1, k, h)
    ws = _lib.workspace(nbytes, device)
    _lib.check(lib.hs_resolve_rows(
        pos.data_ptr(), _lib.HS_INT64 if pos.dtype == torch.int64 else _lib.HS_INT32, k,
        source.data_ptr(), resident.data_ptr(), source.numel(), hot.data_ptr(), hot.numel(),
        tags_k.data_ptr(), lru_k.data_ptr(), h, length, page_size, physical.data_ptr(),
        miss_host.data_ptr(), miss_device.data_ptr(), counts.data_ptr(), _lib.ptr(columns),
        columns.shape[0] if columns is not None else 0,
        columns.shape[1] if columns is not None else 0, _lib.ptr(head_rows), _lib.ptr(ws),
        nbytes, _lib.status_word(device).data_ptr(), _lib.stream_of(device)))
    if tags_k is not tags:
        tags.copy_(tags_k)
    if lru_k is not lru:
        lru.copy_(lru_k)
    return RowPlan(head_rows if columns is not None else physical, miss_host, miss_device, counts)
