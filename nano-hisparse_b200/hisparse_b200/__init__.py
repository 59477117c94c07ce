"""hisparse_b200 — nano-hisparse's per-step sparse-decode hot path on B200.

Operators with the reference's signatures (drop-in for the modules of the
same names in nano_hisparse):

  selection.quest_selection   Quest scoring + shared top-k + token expansion
  row_index.resolve_rows      resident/hot lookup, LRU replacement, miss plan
  row_kernels.gather_rows     pinned host -> pool miss gather (zero-copy)
  row_kernels.attend_rows     physical-row GQA decode attention
  attention.row_attention     resolve + gather + attend through a cache

plus RowCache (device state and the resolve stream/event protocol),
DecodeBatch (the same hot path for B requests per launch) and
plugin.install (routes an imported reference package through these kernels).
All compute runs in libhisparse.so (sm_100a CUDA, C ABI in include/hisparse.h).
"""

from .attention import row_attention
from .batched import DecodeBatch
from .cache import LayerTables, RowCache, RowLease
from .config import ACTIVE_TAIL_PAGES, CacheConfig, CapacityError, HotConfig
from .row_index import LogicalTopK, RowPlan, resolve_rows
from .row_kernels import MappedHost, attend_rows, gather_rows
from .selection import Selection, quest_selection

__all__ = [
    "ACTIVE_TAIL_PAGES", "CacheConfig", "CapacityError", "DecodeBatch", "HotConfig",
    "LayerTables", "LogicalTopK", "MappedHost", "RowCache", "RowLease", "RowPlan", "Selection",
    "attend_rows", "gather_rows", "quest_selection", "resolve_rows", "row_attention",
]
