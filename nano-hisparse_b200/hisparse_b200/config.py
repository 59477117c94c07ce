"""Storage dimensions and hot-buffer limits, with the reference's field names
and validation (nano_hisparse/config.py:12-30, hybrid.py:22-44), so existing
configuration objects and call sites carry over unchanged."""

from __future__ import annotations

from dataclasses import dataclass
from math import ceil

import torch

ACTIVE_TAIL_PAGES = 2  # pages at the write tail that always stay resident (hybrid.py:19)


class CapacityError(RuntimeError):
    """Admission or placement does not fit (nano_hisparse/config.py:8)."""


@dataclass(frozen=True)
class CacheConfig:
    gpu_pages: int = 16
    host_pages: int = 1024
    page_size: int = 16
    kv_heads: int = 2
    head_dim: int = 32
    device: str = "cuda"
    dtype: torch.dtype = torch.float32
    index_budget_bytes: int = 64 * 1024 * 1024

    def __post_init__(self):
        for name in ("gpu_pages", "host_pages", "page_size", "kv_heads", "head_dim"):
            if getattr(self, name) < 1:
                raise ValueError(f"{name} must be positive")
        if self.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError("KV dtype must be float32, float16 or bfloat16")
        if self.index_budget_bytes < 1:
            raise ValueError("index budget must be positive")

    @property
    def row_bytes(self) -> int:
        """Bytes of one token's K (or V) across all KV heads."""
        return self.kv_heads * self.head_dim * torch.empty((), dtype=self.dtype).element_size()


@dataclass(frozen=True)
class HotConfig:
    """max_union_rows bounds the distinct selected rows of one resolve;
    hot_rows is the per-(request, layer) hot buffer (default 2x)."""

    max_union_rows: int
    hot_rows: int | None = None
    resident_window_pages: int = 64
    transition_watermark: int | None = None

    def __post_init__(self):
        if self.max_union_rows < 1:
            raise ValueError("max_union_rows must be positive")
        if self.hot_rows is None:
            object.__setattr__(self, "hot_rows", 2 * self.max_union_rows)
        if self.hot_rows < self.max_union_rows or self.hot_rows > 32768:
            raise ValueError("hot_rows must cover max_union_rows and be <= 32768")
        if self.resident_window_pages < ACTIVE_TAIL_PAGES:
            raise ValueError("resident window must cover both active tail pages")
        if self.transition_watermark is not None and self.transition_watermark < 0:
            raise ValueError("transition watermark must be nonnegative")

    def hot_blocks(self, page_size: int) -> int:
        return ceil(self.hot_rows / page_size)

    def admission_blocks(self, page_size: int, layers: int = 1) -> int:
        return layers * (self.hot_blocks(page_size) + ACTIVE_TAIL_PAGES)
