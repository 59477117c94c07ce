"""TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.

Python wrapper over oracle/liboracle.so, the CPU restatement of nano-hisparse's
per-step decode hot path (see oracle/hisparse_oracle.c for the function-by-
function correspondence with the reference). Only tests/, __graft_entry__.smoke()
(as the checker) and bench.py's CPU-baseline arm import this package; the
product package nano-hisparse_b200/ never does.

Arrays are numpy; torch CPU tensors are accepted and converted. bfloat16 and
float16 data travel as raw 16-bit patterns and are widened inside the C code.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
F32, F16, BF16 = 0, 1, 2
_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int


def build():
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.or_quest_scores.argtypes = [_P, _INT, _P, _P, _INT, _INT, _INT, _INT, _I64, _P]
        _lib.or_quest_select.argtypes = [_P, _I64, _INT, _INT, _INT, _P, _I64, _P]
        _lib.or_quest_head_sums.argtypes = [_P, _INT, _P, _P, _INT, _INT, _INT, _INT, _I64, _P]
        _lib.or_resolve_rows.argtypes = [_P, _I64, _P, _P, _I64, _P, _I64, _P, _P, _I64, _I64,
                                         _INT, _P, _P, _P, _P]
        _lib.or_gather_rows.argtypes = [_P, _I64, _P, _I64, _P, _P, _I64, _INT, _I64]
        _lib.or_attend_rows.argtypes = [_P, _INT, _P, _INT, _I64, _P, _I64, _I64, _INT, _INT,
                                        _INT, _INT, _P]
        _lib.or_decode_layer_batched.argtypes = [
            _INT, _P, _INT, _P, _P, _INT, _P, _INT, _INT, _INT, _INT, _INT, _I64, _P, _P, _P,
            _I64, _P, _P, _I64, _P, _I64, _P, _I64, _P, _P, _INT]
        _lib.or_append_rows.argtypes = [_P, _P, _INT, _I64, _I64, _P, _P, _P, _P, _P, _I64,
                                        _INT]
        for name in ("or_quest_scores", "or_quest_select", "or_resolve_rows", "or_gather_rows",
                     "or_attend_rows", "or_decode_layer_batched", "or_append_rows",
                     "or_quest_head_sums"):
            getattr(_lib, name).restype = _INT
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def as_array(x, dtype=None):
    """numpy view of a numpy array or CPU torch tensor; (array, oracle dtype code)."""
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(x, torch.Tensor):
        t = x.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16), BF16
        if t.dtype == torch.float16:
            return t.view(torch.int16).numpy().view(np.uint16), F16
        x = t.numpy()
    a = np.ascontiguousarray(x if dtype is None else np.asarray(x, dtype=dtype))
    if a.dtype == np.float16:
        return a.view(np.uint16), F16
    code = F32 if a.dtype == np.float32 else None
    return a, code


def quest_scores(query, minimum, maximum, pages):
    """Per-page scores [pages] (float32) in libhisparse's fixed summation order."""
    q, qd = as_array(query)
    mn, kd = as_array(minimum)
    mx, kd2 = as_array(maximum)
    assert kd == kd2 and qd is not None and kd is not None
    hq, d = q.shape
    hkv = mn.shape[1]
    out = np.empty(pages, dtype=np.float32)
    rc = lib().or_quest_scores(_ptr(q), qd, _ptr(mn), _ptr(mx), kd, hq, hkv, d, pages, _ptr(out))
    if rc:
        raise ValueError(f"or_quest_scores failed: {rc}")
    return out


def quest_sharded_scores(query, minimum, maximum, pages, shards):
    """Scores of a head-sharded selection: shard r holds KV heads
    [r*Hkv/W, (r+1)*Hkv/W) and their query heads; its undivided head sums are
    added in shard order in float32, then divided by Hq (with shards = 1 this
    equals quest_scores bit for bit)."""
    q, qd = as_array(query)
    mn, kd = as_array(minimum)
    mx, _ = as_array(maximum)
    hq, d = q.shape
    hkv = mn.shape[1]
    if hkv % shards:
        raise ValueError("KV heads must split evenly over the shards")
    kl, ql = hkv // shards, hq // shards
    total = np.zeros(pages, dtype=np.float32)
    for r in range(shards):
        qs = np.ascontiguousarray(q[r * ql:(r + 1) * ql])
        ms = np.ascontiguousarray(mn[:pages, r * kl:(r + 1) * kl])
        xs = np.ascontiguousarray(mx[:pages, r * kl:(r + 1) * kl])
        part = np.empty(pages, dtype=np.float32)
        rc = lib().or_quest_head_sums(_ptr(qs), qd, _ptr(ms), _ptr(xs), kd, ql, kl, d, pages,
                                      _ptr(part))
        if rc:
            raise ValueError(f"or_quest_head_sums failed: {rc}")
        total = total + part
    return total / np.float32(hq)


def quest_select(scores, length, page_size, top_pages, keep_sink=True, capacity=None):
    """Forced tail/sink + top-k + expansion: (tokens padded with -1, count)."""
    sc = np.ascontiguousarray(scores, dtype=np.float32)
    capacity = capacity or top_pages * page_size
    out = np.empty(capacity, dtype=np.int32)
    count = ctypes.c_int32(0)
    rc = lib().or_quest_select(_ptr(sc), length, page_size, top_pages, int(keep_sink),
                               _ptr(out), capacity, ctypes.byref(count))
    if rc:
        raise ValueError(f"or_quest_select failed: {rc}")
    return out, count.value


def quest_tokens(query, minimum, maximum, length, page_size, top_pages, keep_sink=True):
    """Sorted token list selected by Quest (the shared selection)."""
    pages = -(-length // page_size)
    scores = quest_scores(query, minimum, maximum, pages)
    tokens, count = quest_select(scores, length, page_size, top_pages, keep_sink,
                                 max(top_pages * page_size, length))
    return tokens[:count].tolist()


def resolve_rows(positions, source, resident, hot, tags, lru, length, page_size):
    """Resolver restatement. Returns a dict with physical, miss_host, miss_device,
    counts and the updated tags/lru (inputs are not modified)."""
    pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int64))
    src = np.ascontiguousarray(np.asarray(source, dtype=np.int64))
    res = np.ascontiguousarray(np.asarray(resident, dtype=np.int64))
    hotb = np.ascontiguousarray(np.asarray(hot, dtype=np.int64))
    tg = np.array(tags, dtype=np.int64)
    lr = np.array(lru, dtype=np.int64)
    k, h = pos.size, tg.size
    phys = np.empty(k, dtype=np.int64)
    mh = np.empty(k, dtype=np.int64)
    md = np.empty(k, dtype=np.int64)
    counts = np.zeros(3, dtype=np.int64)
    rc = lib().or_resolve_rows(_ptr(pos), k, _ptr(src), _ptr(res), src.size, _ptr(hotb),
                               hotb.size, _ptr(tg), _ptr(lr), h, length, page_size, _ptr(phys),
                               _ptr(mh), _ptr(md), _ptr(counts))
    if rc:
        raise ValueError(f"or_resolve_rows failed: {rc}")
    return {"physical": phys, "miss_host": mh, "miss_device": md, "counts": counts,
            "tags": tg, "lru": lr}


def gather_rows(host, pool, miss_host, miss_device, page_size):
    """Copies planned miss rows from `host` into `pool` (numpy arrays of shape
    [blocks, 2, P, Hkv, D], any dtype) in place."""
    assert host.flags.c_contiguous and pool.flags.c_contiguous
    mh = np.ascontiguousarray(miss_host, dtype=np.int64)
    md = np.ascontiguousarray(miss_device, dtype=np.int64)
    row_bytes = host.shape[3] * host.shape[4] * host.itemsize
    rc = lib().or_gather_rows(_ptr(host), host.shape[0], _ptr(pool), pool.shape[0], _ptr(mh),
                              _ptr(md), mh.size, page_size, row_bytes)
    if rc:
        raise ValueError(f"or_gather_rows failed: {rc}")


def attend_rows(query, pool, rows, page_size):
    """fp64 attention over physical rows. rows: [K] shared or [Hq, K]."""
    q, qd = as_array(query)
    pl, kd = as_array(pool)
    r = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    hq, d = q.shape
    hkv = pl.shape[3]
    head_stride = 0 if r.ndim == 1 else r.shape[1]
    count = r.shape[-1]
    out = np.empty((hq, d), dtype=np.float64)
    rc = lib().or_attend_rows(_ptr(q), qd, _ptr(pl), kd, pl.shape[0], _ptr(r), head_stride,
                              count, hq, hkv, d, page_size, _ptr(out))
    if rc:
        raise ValueError(f"or_attend_rows failed: {rc}")
    return out


def decode_layer_batched(queries, minimums, maximums, lengths, page_size, top_pages,
                         max_pages, sources, residents, hots, tags, lrus, host, pool,
                         threads=0):
    """Whole hot path for one layer of len(queries) requests (OpenMP over
    requests). Per-request arguments are lists of arrays; tags/lrus (int64) are
    updated in place and pool is written. Returns (outputs [B][Hq, D] fp64,
    counts [B, 3])."""
    b = len(queries)
    keep = []

    def arr_ptrs(items, dtype=None):
        arrs = []
        for x in items:
            a, code = as_array(x, dtype)
            arrs.append((a, code))
        keep.extend(a for a, _ in arrs)
        ptrs = (ctypes.c_void_p * b)(*[a.ctypes.data for a, _ in arrs])
        keep.append(ptrs)
        return ptrs, arrs[0][1]

    qp, qd = arr_ptrs(queries)
    mnp, kd = arr_ptrs(minimums)
    mxp, _ = arr_ptrs(maximums)
    srcp, _ = arr_ptrs(sources, np.int64)
    resp, _ = arr_ptrs(residents, np.int64)
    hotp, _ = arr_ptrs(hots, np.int64)
    for t in list(tags) + list(lrus):
        assert t.dtype == np.int64 and t.flags.c_contiguous
    tagp = (ctypes.c_void_p * b)(*[t.ctypes.data for t in tags])
    lrup = (ctypes.c_void_p * b)(*[t.ctypes.data for t in lrus])
    hq, d = as_array(queries[0])[0].shape
    hkv = as_array(minimums[0])[0].shape[1]
    outs = [np.empty((hq, d), dtype=np.float64) for _ in range(b)]
    outp = (ctypes.c_void_p * b)(*[o.ctypes.data for o in outs])
    counts = np.zeros((b, 3), dtype=np.int64)
    lens = np.ascontiguousarray(lengths, dtype=np.int64)
    hst, _ = as_array(host)
    pl, _ = as_array(pool)
    rc = lib().or_decode_layer_batched(
        b, qp, qd, mnp, mxp, kd, _ptr(lens), hq, hkv, d, page_size, top_pages, max_pages,
        srcp, resp, hotp, hots[0].shape[0] if hasattr(hots[0], "shape") else len(hots[0]),
        tagp, lrup, tags[0].shape[0], _ptr(hst), hst.shape[0], _ptr(pl), pl.shape[0], outp,
        _ptr(counts), threads)
    if rc:
        raise ValueError(f"or_decode_layer_batched failed: {rc}")
    return outs, counts


def append_rows(k, v, within, block, host_block, minimum, maximum, summary):
    """One page chunk of HostStore.append (storage.py:296-321), on copies.

    k, v: [count, Hkv, D] torch rows; block / host_block: the page's pool block
    and host block [2, P, Hkv, D] (host_block may be None; block None makes
    the chunk host-only, which needs a host_block); minimum / maximum:
    [Hkv, D] in the KV dtype; summary: [Hkv, D] float32 (numpy arrays
    and torch tensors; 16-bit data comes back as uint16 bit patterns) — see
    as_array. Returns (block, host_block, minimum, maximum, summary)."""
    import torch

    dtype = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[k.dtype]
    arrays = [as_array(t)[0] for t in (k, v, minimum, maximum)]
    blk = None if block is None else np.ascontiguousarray(as_array(block)[0]).copy()
    host = None if host_block is None else np.ascontiguousarray(as_array(host_block)[0]).copy()
    summ = np.ascontiguousarray(summary.numpy() if hasattr(summary, "numpy") else summary,
                                dtype=np.float32).copy()
    kk, vv, mn, mx = [np.ascontiguousarray(a).copy() for a in arrays]
    elems = kk[0].size if kk.shape[0] else int(np.prod(kk.shape[1:]))
    page = blk if blk is not None else host
    rc = lib().or_append_rows(_ptr(kk), _ptr(vv), dtype, kk.shape[0], within,
                              None if blk is None else _ptr(blk),
                              None if host is None else _ptr(host), _ptr(mn), _ptr(mx),
                              _ptr(summ), elems, page.shape[1])
    if rc:
        raise ValueError(f"or_append_rows failed ({rc})")
    return blk, host, mn, mx, summ
