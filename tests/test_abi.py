"""The C ABI library loads, exports every symbol include/hisparse.h declares,
and rejects invalid arguments on the host (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from hisparse_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "hisparse.h"


def declared():
    return re.findall(r"^HS_API\s+[\w\s\*]*?\b(hs_\w+)\s*\(", HEADER.read_text(), flags=re.M)


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) == 19
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib._SIGNATURES)


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.hs_version() == _lib.ABI_VERSION
    assert lib.hs_status_string(0) == b"ok"
    assert lib.hs_status_string(_lib.HS_ERR_WORKSPACE) == b"workspace too small"


def test_host_side_validation_needs_no_device():
    lib = _lib.load()
    status = lib.hs_quest_select(1, _lib.HS_FLOAT32, 1, 1, _lib.HS_FLOAT32, 4, 2, 8, 10, 37, 4,
                                 0, 1, 1, 64, 1, 1, 64, None, None)
    assert status == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_last_error() == b"invalid page budget or GQA shape"
    status = lib.hs_resolve_rows(1, _lib.HS_INT32, 0, 1, 1, 4, 1, 1, 1, 1, 4, 16, 4, 1, 1, 1, 1,
                                 None, 0, 0, None, None, 0, None, None)
    assert status == _lib.HS_ERR_INVALID_ARGUMENT
    status = lib.hs_gather_rows(None, 1, 1, 1, 1, 1, 4, 4, 4, 64, None, None)
    assert status == _lib.HS_ERR_INVALID_ARGUMENT
    status = lib.hs_attend_rows(1, 1, 32, _lib.HS_FLOAT32, 1, 4, _lib.HS_FLOAT32, 1, 4, 0, 4, 1,
                                32, 6, 4, 8, 4, None, 0, None, None)
    assert status == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_last_error() == b"query GQA/device mismatch"
    status = lib.hs_quest_select(1, 7, 1, 1, _lib.HS_FLOAT32, 4, 2, 8, 10, 37, 4, 2, 1, 1, 64, 1,
                                 1, 64, None, None)
    assert status == _lib.HS_ERR_WORKSPACE or status == _lib.HS_ERR_INVALID_ARGUMENT
    status = lib.hs_quest_select(1, _lib.HS_FLOAT32, 1, 1, _lib.HS_FLOAT32, 4, 2, 300, 10, 37, 4,
                                 2, 1, 1, 64, 1, 1, 64, None, None)
    assert status == _lib.HS_ERR_UNSUPPORTED


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.hs_quest_workspace_bytes(2, 100) == 2 * 100 * 4 + 2 * 4  # scores + counters
    assert lib.hs_resolve_workspace_bytes(1, 2048, 4096) == 0  # fits shared memory
    assert lib.hs_resolve_workspace_bytes(2, 32768, 32768) > 2 * 1024 * 1024
    assert lib.hs_attend_workspace_bytes(16, 32, 8, 128, 2048) > 0


def test_host_alias_rejects_unpinned_memory():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(64)
    alias = ctypes.c_void_p()
    status = lib.hs_host_device_pointer(ctypes.addressof(buf), ctypes.byref(alias))
    assert status == _lib.HS_ERR_NOT_MAPPED


def test_operators_refuse_cpu_tensors():
    """There is no CPU fallback on the product path."""
    from hisparse_b200 import LogicalTopK, quest_selection, resolve_rows

    with pytest.raises(ValueError, match="CUDA"):
        quest_selection(torch.randn(4, 8), torch.zeros(10, 2, 8), torch.zeros(10, 2, 8), 37, 4, 2)
    t = torch.zeros(4, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        resolve_rows(LogicalTopK(t), t, t, t, t, t.long(), 16, 4)


def test_host_side_validation_of_append_and_sharded_selection():
    """Argument errors of the append and head-sharded selection entry points
    are reported on the host, before any device work."""
    lib = _lib.load()
    d = 256  # a dummy non-null pointer value: never dereferenced on these paths
    # append: negative batch, bad head shape, unknown dtype, null pointers
    assert lib.hs_append_rows(-1, d, d, 0, _lib.HS_BFLOAT16, d, d, d, d, 1, d, d, 1, d, d, d,
                              8, 128, 16, None, None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_append_rows(1, d, d, 0, _lib.HS_BFLOAT16, d, d, d, d, 1, d, d, 1, d, d, d,
                              0, 128, 16, None, None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_append_rows(1, None, d, 0, _lib.HS_BFLOAT16, d, d, d, d, 1, d, d, 1, d, d, d,
                              8, 128, 16, None, None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert b"null" in lib.hs_last_error()
    assert lib.hs_append_rows(0, None, None, 0, _lib.HS_BFLOAT16, None, None, None, None, 0,
                              None, None, 0, None, None, None, 8, 128, 16, None,
                              None) == _lib.HS_OK  # an empty batch is a no-op
    # sharded selection: no shards, a too small output, a missing workspace
    assert lib.hs_quest_select_partials(0, d, 1, d, 28, 16384, 64, 128, 1, d, 8192, d, d,
                                        1 << 20, None, None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_quest_select_partials(2, d, 1, d, 28, 16384, 64, 128, 1, d, 100, d, d,
                                        1 << 20, None, None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert b"out_capacity" in lib.hs_last_error()
    assert lib.hs_quest_select_partials(2, d, 1, d, 28, 16384, 64, 128, 1, d, 8192, d, None, 0,
                                        None, None) == _lib.HS_ERR_WORKSPACE
    assert lib.hs_quest_partial_scores_batched(1, d, 0, _lib.HS_BFLOAT16, d, d, _lib.HS_BFLOAT16,
                                               d, 14, 2, 128, 16384, 64, None, None,
                                               None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_quest_partial_scores_batched(1, d, 0, _lib.HS_BFLOAT16, d, d, _lib.HS_BFLOAT16,
                                               d, 14, 4, 128, 16384, 64, d, None,
                                               None) == _lib.HS_ERR_INVALID_ARGUMENT
    assert lib.hs_last_error() == b"invalid page budget or GQA shape"


def test_sharded_head_slices():
    from hisparse_b200.sharded import head_slice

    assert head_slice(4, 28, 1, 2) == (slice(2, 4), slice(14, 28))
    assert [head_slice(8, 32, r, 4)[0] for r in range(4)] == [slice(0, 2), slice(2, 4),
                                                              slice(4, 6), slice(6, 8)]
    with pytest.raises(ValueError):
        head_slice(4, 28, 0, 3)
    with pytest.raises(ValueError):
        head_slice(4, 28, 2, 2)
