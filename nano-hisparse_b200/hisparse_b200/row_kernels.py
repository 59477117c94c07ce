"""Host->pool miss gather and physical-row attention.

Drop-in for nano_hisparse/row_kernels.py: ``MappedHost`` (row_kernels.py:10-32),
``gather_rows`` (row_kernels.py:58-70) and ``attend_rows`` (row_kernels.py:116-135)
keep their signatures; the Triton kernels are replaced by libhisparse's
``hs_gather_rows`` (zero-copy reads of pinned host rows, 16-byte vectors, one
warp per row) and ``hs_attend_rows`` (one CTA per GQA group and row split,
fp32 online softmax, split merge).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


class MappedHost:
    """Keeps a pinned host tensor alive and exposes its device alias.

    The pinned allocation belongs to PyTorch; nothing is registered or
    unregistered here (same rule as row_kernels.py:10-15).
    """

    def __init__(self, tensor: torch.Tensor):
        if not tensor.is_pinned():
            raise ValueError("row gather requires pinned host backing")
        lib = _lib.load()
        alias = ctypes.c_void_p()
        status = lib.hs_host_device_pointer(tensor.data_ptr(), ctypes.byref(alias))
        if status:
            raise RuntimeError(lib.hs_last_error().decode(errors="replace"))
        self.tensor, self.dtype, self.pointer = tensor, tensor.dtype, alias.value

    def data_ptr(self):
        return self.pointer


def _host_alias(host):
    if isinstance(host, MappedHost):
        return host
    if isinstance(host, torch.Tensor):
        return MappedHost(host)
    raise ValueError("host must be a MappedHost or a pinned tensor")


def gather_rows(host, pool, plan, config):
    """Copy every planned miss row (K and V planes) from host to pool.

    host: MappedHost (or pinned tensor) [host_pages, 2, P, Hkv, D]; pool: CUDA
    tensor [gpu_pages, 2, P, Hkv, D] of the same dtype; plan: RowPlan whose
    miss_host_rows / miss_device_rows are the resolver's compact prefix.
    Runs on the current stream.
    """
    mapped = _host_alias(host)
    _lib.require_cuda(pool, plan.miss_host_rows, plan.miss_device_rows)
    if mapped.tensor.dtype != pool.dtype or mapped.tensor.shape[1:] != pool.shape[1:]:
        raise ValueError("host store and pool layouts differ")
    lib = _lib.load()
    miss_host = plan.miss_host_rows.contiguous()
    miss_device = plan.miss_device_rows.contiguous()
    if miss_host.dtype != torch.int64 or miss_device.dtype != torch.int64:
        miss_host, miss_device = miss_host.long(), miss_device.long()
    n = miss_host.numel()
    row_bytes = config.kv_heads * config.head_dim * pool.element_size()
    _lib.check(lib.hs_gather_rows(
        mapped.data_ptr(), mapped.tensor.shape[0], pool.data_ptr(), pool.shape[0],
        miss_host.data_ptr(), miss_device.data_ptr(), n, n, config.page_size, row_bytes,
        _lib.status_word(pool.device).data_ptr(), _lib.stream_of(pool.device)))


def attend_rows(query, pool, rows, config):
    """Decode attention of query [Hq, D] over physical rows of the pool.

    rows: int64 [Hq, K] (a stride-0 expansion of a shared [K] vector is read
    once per GQA group) or [K]; -1 entries are masked; a head with no valid row
    gets zeros. Output has the query's dtype.
    """
    _lib.require_cuda(query, pool, rows)
    if rows.ndim == 1:
        rows = rows[None, :].expand(query.shape[0], -1)
    query = query.contiguous()
    output = torch.empty_like(query)
    attend_into(output, query, pool, rows, config)
    return output


def attend_into(output, query, pool, rows, config, batch=1):
    """attend_rows for `batch` queries [B, Hq, D] with rows [B, Hq, K] (or
    [Hq, K] for batch 1), writing into `output`."""
    lib = _lib.load()
    if rows.dtype != torch.int64:
        rows = rows.long()
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    head_stride = rows.stride(-2)
    batch_stride = rows.stride(0) if rows.ndim == 3 else 0
    count = rows.shape[-1]
    q_heads, head_dim = query.shape[-2], query.shape[-1]
    if head_dim != config.head_dim or q_heads % config.kv_heads:
        raise ValueError("query GQA/device mismatch")
    if count < 1:
        output.zero_()
        return output
    nbytes = lib.hs_attend_workspace_bytes(batch, q_heads, config.kv_heads, head_dim, count)
    ws = _lib.workspace(nbytes, query.device)
    _lib.check(lib.hs_attend_rows(
        batch, query.data_ptr(), q_heads * head_dim, _lib.dtype_code(query.dtype),
        pool.data_ptr(), pool.shape[0], _lib.dtype_code(pool.dtype), rows.data_ptr(),
        batch_stride, head_stride, count, output.data_ptr(), q_heads * head_dim, q_heads,
        config.kv_heads, head_dim, config.page_size, _lib.ptr(ws), nbytes,
        _lib.status_word(query.device).data_ptr(), _lib.stream_of(query.device)))
    return output
