"""Head-sharded Quest selection for one long request (configuration 5).

When one request is too long for one GPU, its KV heads are split over the
ranks of a process group: rank r holds KV heads [r*Hkv/W, (r+1)*Hkv/W) of
the pool, the host mirror and the Quest min/max metadata, plus the query
heads of those GQA groups. The page selection must still be ONE shared
selection (selection.py:69-91 averages over all query heads), so the ranks
exchange their partial scores once per layer:

  1. ``hs_quest_partial_scores_batched`` — this rank's per-page head sums
     (fixed fp32 order, undivided), [max_pages] fp32;
  2. an all-gather of the partials over the group (NCCL over NVLink; 64 KiB
     for 16384 pages);
  3. ``hs_quest_select_partials`` — shard-ordered sum, division by the total
     query heads, forced pages, top-k and expansion: every rank computes the
     same tokens from the same bytes.

With one rank (no group) the result equals ``quest_selection`` bit for bit.
The resolver tables are replicated per rank (the selection is shared), so
each rank then resolves, gathers and attends over its own head slice with the
ordinary operators.
"""

from __future__ import annotations

from math import ceil

import torch

from . import _lib
from .selection import Selection


def head_slice(kv_heads: int, q_heads: int, rank: int, world: int) -> tuple[slice, slice]:
    """(KV-head slice, query-head slice) owned by `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if kv_heads % world or q_heads % kv_heads:
        raise ValueError("KV heads must split evenly over the ranks, query heads over KV heads")
    kl, ql = kv_heads // world, q_heads // world
    return slice(rank * kl, (rank + 1) * kl), slice(rank * ql, (rank + 1) * ql)


def group_world(group) -> int:
    """Ranks that share one selection: the size of `group`, or 1 when no group
    is given. A process group that merely exists (e.g. a request-sharded job
    that initialised torch.distributed for its reporting) never joins an
    exchange implicitly: the caller names the group its heads are split over."""
    if group is None:
        return 1
    import torch.distributed as dist

    return dist.get_world_size(group)


def same_on_every_rank(group, values, device=None) -> bool:
    """True when every rank of `group` passed the same integers. One small
    all-reduce (MAX of each value and of its negation) on the group's backend;
    every rank gets the same answer, so all raise or none does."""
    import torch.distributed as dist

    t = torch.tensor([int(v) for v in values] + [-int(v) for v in values], dtype=torch.int64)
    if dist.get_backend(group) == "nccl":
        t = t.to(device if device is not None else torch.device("cuda",
                                                                torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    t, k = t.cpu(), len(values)
    return all(int(t[i]) == -int(t[k + i]) for i in range(k))


def _argument_problem(query, minimum, maximum, count, top_pages):
    """The ValueError message quest_selection would raise, or None."""
    if top_pages < 1 or query.shape[0] % minimum.shape[1]:
        return "invalid page budget or GQA shape"
    if top_pages >= count:
        return None
    if minimum.shape != maximum.shape or minimum.dtype != maximum.dtype:
        return "minimum and maximum metadata must match"
    if minimum.ndim != 3 or query.ndim != 2 or minimum.shape[2] != query.shape[1]:
        return "expected query [heads, dim] and metadata [pages, kv_heads, dim]"
    if minimum.shape[0] < count:
        return "metadata has fewer pages than the selection length"
    return None


def sharded_quest_selection(query, minimum, maximum, length, page_size, top_pages,
                            keep_sink=True, group=None):
    """quest_selection over heads split across the ranks of `group`.

    query [Hq_local, D], minimum/maximum [>= pages, Hkv_local, D]: this rank's
    slices (see head_slice). Returns the device-form Selection, identical on
    every rank, with `heads` = the query heads of all ranks. Without a group
    the selection is this rank's alone (no collective). Every rank must pass
    the same length, page size, budget and metadata table length: these are
    compared across the group first (the all-gather needs equal sizes on every
    rank), and a mismatch raises ValueError on every rank.
    """
    import torch.distributed as dist

    world = group_world(group)
    count = ceil(length / page_size)
    heads = query.shape[0] * world
    problem = _argument_problem(query, minimum, maximum, count, top_pages)
    if world > 1 and not same_on_every_rank(
            group, (minimum.shape[0], length, page_size, top_pages, bool(keep_sink),
                    problem is None), query.device):
        # compared before any rank can branch, so no rank waits alone in the exchange
        raise ValueError("ranks disagree on the metadata table length, the selection "
                         "length, the page size, the page budget or argument validity")
    if problem is not None:
        raise ValueError(problem)
    if top_pages >= count:
        return Selection.from_pages(list(range(count)), length, page_size, heads, "quest")
    _lib.require_cuda(query, minimum, maximum)
    lib = _lib.load()
    device = query.device
    query, minimum, maximum = query.contiguous(), minimum.contiguous(), maximum.contiguous()
    max_pages = minimum.shape[0]
    status, stream = _lib.status_word(device).data_ptr(), _lib.stream_of(device)
    # one upload: [min ptr, max ptr, length] (the batched entry points take
    # device arrays; int32 length read from the low half of the third slot)
    meta = torch.tensor([minimum.data_ptr(), maximum.data_ptr(), length],
                        dtype=torch.int64).to(device, non_blocking=True)
    lengths = meta.view(torch.int32)[4:5]
    partial = torch.empty(max_pages, dtype=torch.float32, device=device)
    _lib.check(lib.hs_quest_partial_scores_batched(
        1, query.data_ptr(), 0, _lib.dtype_code(query.dtype), meta[0:1].data_ptr(),
        meta[1:2].data_ptr(), _lib.dtype_code(minimum.dtype), lengths.data_ptr(),
        query.shape[0], minimum.shape[1], query.shape[1], max_pages, page_size,
        partial.data_ptr(), status, stream))
    if world > 1:
        partials = torch.empty((world, max_pages), dtype=torch.float32, device=device)
        dist.all_gather_into_tensor(partials, partial, group=group)
    else:
        partials = partial.view(1, max_pages)
    width = top_pages * page_size
    tokens = torch.empty(width, dtype=torch.int32, device=device)
    counter = torch.empty(1, dtype=torch.int32, device=device)
    nbytes = lib.hs_quest_workspace_bytes(1, max_pages)
    ws = _lib.workspace(nbytes, device)
    _lib.check(lib.hs_quest_select_partials(
        world, partials.data_ptr(), 1, lengths.data_ptr(), heads, max_pages, page_size,
        top_pages, int(bool(keep_sink)), tokens.data_ptr(), width, counter.data_ptr(),
        _lib.ptr(ws), nbytes, status, stream))
    return Selection.from_device(tokens, length, page_size, heads, "quest")
