"""Quest selection kernel vs the reference's recorded selections and the oracle."""

import math

import numpy as np
import pytest
import torch

import oracle
from helpers import quest_sets_agree
from hisparse_b200 import LogicalTopK, Selection, _lib, quest_selection
from hisparse_b200.selection import quest_selection as qs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _tokens(sel):
    return list(sel.positions[0])


def test_reference_fixtures(golden):
    identical = 0
    for case in golden("quest_cases"):
        q, mn, mx = (case[k].to(DEV) for k in ("query", "minimum", "maximum"))
        for sink in (0, 1):
            key = f"tokens_{sink}"
            if key not in case:
                continue
            sel = quest_selection(q, mn, mx, case["length"], case["page_size"],
                                  case["top_pages"], keep_sink=bool(sink))
            got = _tokens(sel)
            # bit-exact against the oracle (same fixed fp32 summation order)
            assert got == oracle.quest_tokens(case["query"], case["minimum"], case["maximum"],
                                              case["length"], case["page_size"],
                                              case["top_pages"], bool(sink)), case["name"]
            ok, detail = quest_sets_agree(case[key], got, case["query"], case["minimum"],
                                          case["maximum"], case["length"], case["page_size"],
                                          case["top_pages"], bool(sink))
            assert ok, f"{case['name']}: {detail}"
            identical += detail == "identical"
    assert identical >= 50
    assert not _lib.device_flags(DEV)


def _metadata(gen, pages, hkv, d, dtype, spare=0):
    keys = torch.randn(pages, 16, hkv, d, generator=gen).to(dtype)
    return keys.float().amin(1).to(dtype), keys.float().amax(1).to(dtype)


@pytest.mark.parametrize("hq,hkv,d,p,length,top,dtype", [
    (32, 8, 128, 16, 32768, 128, torch.bfloat16),   # configuration 2
    (32, 8, 128, 16, 131072, 256, torch.bfloat16),  # configuration 3, page 16
    (32, 8, 128, 64, 131072, 64, torch.bfloat16),   # configuration 3, page 64
    (28, 4, 128, 64, 1048576, 128, torch.bfloat16),  # configuration 5
    (8, 2, 32, 16, 150, 4, torch.float32),          # configuration 1
    (6, 2, 24, 7, 1000, 9, torch.float16),
    (40, 8, 96, 5, 3001, 17, torch.float32),         # more than 32 query heads, C = 3
    (4, 4, 256, 3, 100, 2, torch.bfloat16),          # head_dim 256
])
def test_full_size_against_oracle(hq, hkv, d, p, length, top, dtype):
    gen = torch.Generator().manual_seed(hq * 1000 + length)
    pages = math.ceil(length / p)
    mn, mx = _metadata(gen, pages + 5, hkv, d, dtype)
    q = torch.randn(hq, d, generator=gen).to(dtype)
    for sink in (True, False):
        sel = quest_selection(q.to(DEV), mn.to(DEV), mx.to(DEV), length, p, top, sink)
        assert sel.device_tokens is not None
        assert _tokens(sel) == oracle.quest_tokens(q, mn, mx, length, p, top, sink)
    assert not _lib.device_flags(DEV)


def test_device_form_feeds_the_resolver_without_sync():
    gen = torch.Generator().manual_seed(1)
    mn, mx = _metadata(gen, 64, 2, 32, torch.bfloat16)
    q = torch.randn(8, 32, generator=gen).to(torch.bfloat16)
    sel = qs(q.to(DEV), mn.to(DEV), mx.to(DEV), 1000, 16, 6)
    topk = LogicalTopK.from_selection(sel, torch.device(DEV))
    assert topk.positions.data_ptr() == sel.device_tokens.data_ptr()
    assert topk.positions.numel() == 6 * 16
    expected = oracle.quest_tokens(q, mn, mx, 1000, 16, 6)
    assert topk.positions.tolist() == expected + [-1] * (96 - len(expected))
    assert sel.positions == (tuple(expected),) * 8
    assert sel == Selection.from_tokens(expected, 1000, 16, 8, "quest")


def test_all_pages_when_budget_covers_history():
    q = torch.randn(4, 8, device=DEV)
    mn = torch.zeros(10, 2, 8, device=DEV)
    sel = quest_selection(q, mn, mn, 37, 4, 10)
    assert sel.positions[0] == tuple(range(37))


def test_invalid_arguments_raise():
    q = torch.randn(6, 8, device=DEV)
    mn = torch.zeros(10, 4, 8, device=DEV)
    with pytest.raises(ValueError, match="invalid page budget or GQA shape"):
        quest_selection(q, mn, mn, 37, 4, 2)
    with pytest.raises(ValueError, match="invalid page budget or GQA shape"):
        quest_selection(q[:4], mn, mn, 37, 4, 0)
    with pytest.raises(ValueError):
        quest_selection(q[:4], mn[:5], mn[:5], 37, 4, 2)


def test_batched_matches_single():
    gen = torch.Generator().manual_seed(8)
    b, hq, hkv, d, p, top = 5, 32, 8, 128, 16, 16
    lengths = [4096, 1000, 17, 4000, 2049]
    mins, maxs, qs_ = [], [], []
    for length in lengths:
        mn, mx = _metadata(gen, 300, hkv, d, torch.bfloat16)
        mins.append(mn.to(DEV))
        maxs.append(mx.to(DEV))
    query = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16).to(DEV)
    lib = _lib.load()
    width = top * p
    tokens = torch.empty(b, width, dtype=torch.int32, device=DEV)
    counts = torch.empty(b, dtype=torch.int32, device=DEV)
    mptr = torch.tensor([t.data_ptr() for t in mins], dtype=torch.int64, device=DEV)
    xptr = torch.tensor([t.data_ptr() for t in maxs], dtype=torch.int64, device=DEV)
    lens = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    nbytes = lib.hs_quest_workspace_bytes(b, 300)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    _lib.check(lib.hs_quest_select_batched(
        b, query.data_ptr(), hq * d, _lib.HS_BFLOAT16, mptr.data_ptr(), xptr.data_ptr(),
        _lib.HS_BFLOAT16, lens.data_ptr(), hq, hkv, d, 300, p, top, 1, tokens.data_ptr(), width,
        counts.data_ptr(), ws.data_ptr(), nbytes, 0, torch.cuda.current_stream().cuda_stream))
    for i, length in enumerate(lengths):
        single = qs(query[i], mins[i], maxs[i], length, p, top)
        expected = list(single.positions[0])
        assert counts[i].item() == len(expected)
        row = tokens[i].tolist()
        assert row[:len(expected)] == expected and set(row[len(expected):]) <= {-1}
