"""hs_attend_rows_static (attention with the library's fixed device scratch,
no caller workspace) against hs_attend_rows with a caller workspace.

Collected last on purpose: the static entry point must give the same results
whether it is the first libhisparse call of the process or follows the rest of
the suite."""

import ctypes

import pytest
import torch

from helpers import TOL
from hisparse_b200 import _lib

DEV = "cuda:0"
STATIC_SCRATCH_BYTES = 16 << 20


def _static(lib, query, pool, rows, out, kv_heads, page_size, batch=1, batch_stride=0):
    q_heads, head_dim = query.shape[-2], query.shape[-1]
    return lib.hs_attend_rows_static(
        batch, query.data_ptr(), q_heads * head_dim, _lib.dtype_code(query.dtype),
        pool.data_ptr(), pool.shape[0], _lib.dtype_code(pool.dtype), rows.data_ptr(),
        batch_stride, rows.stride(-2), rows.shape[-1], out.data_ptr(), q_heads * head_dim,
        q_heads, kv_heads, head_dim, page_size, _lib.status_word(query.device).data_ptr(),
        _lib.stream_of(query.device))


def _with_workspace(lib, query, pool, rows, out, kv_heads, page_size, batch=1, batch_stride=0):
    q_heads, head_dim = query.shape[-2], query.shape[-1]
    nbytes = lib.hs_attend_workspace_bytes(batch, q_heads, kv_heads, head_dim, rows.shape[-1])
    ws = torch.empty(nbytes, dtype=torch.uint8, device=query.device)
    rc = lib.hs_attend_rows(
        batch, query.data_ptr(), q_heads * head_dim, _lib.dtype_code(query.dtype),
        pool.data_ptr(), pool.shape[0], _lib.dtype_code(pool.dtype), rows.data_ptr(),
        batch_stride, rows.stride(-2), rows.shape[-1], out.data_ptr(), q_heads * head_dim,
        q_heads, kv_heads, head_dim, page_size, ws.data_ptr(), nbytes,
        _lib.status_word(query.device).data_ptr(), _lib.stream_of(query.device))
    torch.cuda.synchronize()
    return rc


def test_static_scratch_rejects_oversized_calls():
    """A call needing more than the fixed scratch fails on the host with
    HS_ERR_WORKSPACE before touching any pointer (no GPU needed)."""
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)
    need = lib.hs_attend_workspace_bytes(64, 64, 8, 256, 1 << 20)
    assert need > STATIC_SCRATCH_BYTES
    rc = lib.hs_attend_rows_static(64, dummy, 64 * 256, _lib.HS_BFLOAT16, dummy, 1,
                                   _lib.HS_BFLOAT16, dummy, 0, 0, 1 << 20, dummy, 64 * 256,
                                   64, 8, 256, 16, None, None)
    assert rc == _lib.HS_ERR_WORKSPACE
    message = lib.hs_last_error().decode()
    assert "static scratch" in message and str(STATIC_SCRATCH_BYTES) in message


CASES = [
    # (name, batch, q_heads, kv_heads, head_dim, count, page_size, dtype, per_head_rows)
    ("bf16 shared rows, tensor-core path", 1, 32, 8, 128, 3000, 16, torch.bfloat16, False),
    ("bf16 batch of 4, shared rows", 4, 32, 8, 128, 700, 16, torch.bfloat16, False),
    ("fp16 per-head rows", 1, 8, 2, 64, 257, 8, torch.float16, True),
    ("fp32 shared rows, one row", 1, 4, 4, 32, 1, 4, torch.float32, False),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_static_scratch_matches_workspace_entry_point(case):
    name, batch, hq, hkv, d, count, page, dtype, per_head = case
    lib = _lib.load()
    gen = torch.Generator().manual_seed(7)
    blocks = (count + page - 1) // page + 3
    pool = torch.randn(blocks, 2, page, hkv, d, generator=gen).to(dtype).to(DEV)
    query = torch.randn(batch, hq, d, generator=gen).to(dtype).to(DEV)
    rows_total = blocks * page
    rows = torch.randint(-1, rows_total, (batch, hq if per_head else 1, count), generator=gen)
    rows[..., 0] = torch.clamp(rows[..., 0], min=0)  # at least one valid row per head
    rows = rows.to(DEV)
    if not per_head:
        rows = rows.expand(batch, hq, count)  # shared selection: head stride 0
    batch_stride = rows.stride(0) if batch > 1 else 0
    assert lib.hs_attend_workspace_bytes(batch, hq, hkv, d, count) <= STATIC_SCRATCH_BYTES

    expected = torch.empty_like(query)
    assert _with_workspace(lib, query, pool, rows, expected, hkv, page, batch,
                           batch_stride) == 0, lib.hs_last_error()
    for call in range(2):  # two calls in a row share the same scratch array
        out = torch.full_like(query, float("nan"))
        torch.cuda.synchronize()
        allocated = torch.cuda.memory_allocated(DEV)
        free_before = torch.cuda.mem_get_info(DEV)[0]
        rc = _static(lib, query, pool, rows, out, hkv, page, batch, batch_stride)
        assert rc == 0, lib.hs_last_error()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated(DEV) == allocated
        if call == 1:  # after the first call's set-up nothing changes device memory
            assert torch.cuda.mem_get_info(DEV)[0] == free_before
        torch.testing.assert_close(out.float(), expected.float(), **TOL[dtype],
                                   msg=f"{name}, call {call}")
    assert not _lib.device_flags(DEV)
