"""Quest selection kernel vs the reference's recorded selections and the oracle."""

import math

import numpy as np
import pytest
import torch

import oracle
from helpers import full_quest_inputs, near_tie_report, pages_to_tokens
from hisparse_b200 import LogicalTopK, Selection, _lib, quest_selection
from hisparse_b200.selection import quest_selection as qs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _tokens(sel):
    return list(sel.positions[0])


def test_reference_fixtures(golden):
    checked = 0
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
            # and token for token the reference's selection
            assert got == list(case[key]), f"{case['name']} sink={sink}: " + near_tie_report(
                case[key], got, case["query"], case["minimum"], case["maximum"],
                case["length"], case["page_size"], case["top_pages"], bool(sink))
            checked += 1
    assert checked == 62
    assert not _lib.device_flags(DEV)


def _full_cases(golden):
    """Full-size reference cases grouped by shape, inputs regenerated from
    their seeds (digest-checked)."""
    groups = {}
    for case in golden("quest_full_cases"):
        q, mn, mx, digest = full_quest_inputs(case["q_heads"], case["kv_heads"],
                                              case["head_dim"], case["page_size"],
                                              case["max_pages"], case["seed"])
        assert digest == case["digest"], f"{case['name']}: input generator changed"
        key = (case["q_heads"], case["kv_heads"], case["head_dim"], case["page_size"],
               case["max_pages"], case["top_pages"])
        groups.setdefault(key, []).append((case, q, mn, mx))
    return groups


def test_full_size_selections_equal_the_reference(golden):
    """The kernels' selections at the sizes the bench runs equal the
    reference's, page for page: the single-request entry point and the
    batched one (all seeds of a shape in one launch; configuration 5's 16,389
    pages take the partial-score + cluster-select path), sink on and off."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for (hq, hkv, d, p, max_pages, top), cases in _full_cases(golden).items():
        dq = torch.stack([q for _, q, _, _ in cases]).to(DEV)
        dmins = [mn.to(DEV) for _, _, mn, _ in cases]
        dmaxs = [mx.to(DEV) for _, _, _, mx in cases]
        b, width = len(cases), top * p
        mptr = torch.tensor([t.data_ptr() for t in dmins], dtype=torch.int64, device=DEV)
        xptr = torch.tensor([t.data_ptr() for t in dmaxs], dtype=torch.int64, device=DEV)
        lens = torch.tensor([c["length"] for c, *_ in cases], dtype=torch.int32, device=DEV)
        tokens = torch.empty(b, width, dtype=torch.int32, device=DEV)
        counts = torch.empty(b, dtype=torch.int32, device=DEV)
        nbytes = lib.hs_quest_workspace_bytes(b, max_pages)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
        for sink in (1, 0):
            _lib.check(lib.hs_quest_select_batched(
                b, dq.data_ptr(), hq * d, _lib.HS_BFLOAT16, mptr.data_ptr(), xptr.data_ptr(),
                _lib.HS_BFLOAT16, lens.data_ptr(), hq, hkv, d, max_pages, p, top, sink,
                tokens.data_ptr(), width, counts.data_ptr(), ws.data_ptr(), nbytes, 0, stream))
            batched = tokens.cpu().tolist()
            for i, (case, q, mn, mx) in enumerate(cases):
                want = pages_to_tokens(case[f"pages_{sink}"], case["length"], p)
                single = _tokens(quest_selection(dq[i], dmins[i], dmaxs[i], case["length"], p,
                                                 top, keep_sink=bool(sink)))
                for form, got in (("single", single),
                                  ("batched", batched[i][:int(counts[i])])):
                    assert got == want, f"{case['name']} sink={sink} {form}: " + \
                        near_tie_report(want, got, q, mn, mx, case["length"], p, top,
                                        bool(sink))
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
    (8, 2, 32, 16, 80000, 20, torch.float32),        # long table, register path (fp32)
    (12, 4, 96, 16, 70001, 33, torch.float16),       # long table, register path (C = 3)
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


def _select_partials(partials, lengths, q_heads, page_size, top, sink):
    """hs_quest_select_partials on device partials [shards, batch, max_pages]."""
    lib = _lib.load()
    shards, batch, max_pages = partials.shape
    width = top * page_size
    tokens = torch.empty(batch, width, dtype=torch.int32, device=DEV)
    counts = torch.empty(batch, dtype=torch.int32, device=DEV)
    lens = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    nbytes = lib.hs_quest_workspace_bytes(batch, max_pages)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    _lib.check(lib.hs_quest_select_partials(
        shards, partials.data_ptr(), batch, lens.data_ptr(), q_heads, max_pages, page_size, top,
        int(sink), tokens.data_ptr(), width, counts.data_ptr(), ws.data_ptr(), nbytes, 0,
        torch.cuda.current_stream().cuda_stream))
    return tokens.cpu().numpy(), counts.cpu().numpy()


@pytest.mark.parametrize("top", [1, 2, 3, 128])
@pytest.mark.parametrize("sink", [True, False])
def test_long_table_selection_edges(top, sink):
    """Tables of >= 4096 pages rank over a thread-block cluster per request:
    chunk edges (5000 pages over 8 CTAs), a tail just past the budget, budgets
    that hold only the forced pages, all-pages requests, empty requests, ties,
    NaN and infinities — token for token the oracle's selection."""
    gen = torch.Generator().manual_seed(top * 2 + sink)
    shards, q_heads, p, max_pages = 2, 28, 16, 5000
    lengths = [max_pages * p, 4999 * p - 3, 17, (top + 1) * p - 5, 70000, 0, 3000 * p]
    partials = torch.randn(shards, len(lengths), max_pages, generator=gen) * 50 + 900
    partials[:, 3] = torch.randint(0, 3, (shards, max_pages), generator=gen).float()  # ties
    partials[:, 4, ::97] = float("nan")
    partials[0, 4, 5::101] = float("inf")
    partials[1, 4, 7::103] = float("-inf")
    partials[:, 6] = torch.randn(shards, max_pages, generator=gen)  # mixed signs, -0 below
    partials[:, 6, 11::50] = -0.0
    tokens, counts = _select_partials(partials.to(DEV), lengths, q_heads, p, top, sink)
    part = partials.numpy()
    for i, length in enumerate(lengths):
        if length == 0:
            assert counts[i] == 0 and set(tokens[i].tolist()) == {-1}
            continue
        total = np.zeros(max_pages, dtype=np.float32)
        for r in range(shards):
            total = (total + part[r, i]).astype(np.float32)
        scores = (total / np.float32(q_heads)).astype(np.float32)
        n = -(-length // p)
        want, count = oracle.quest_select(scores[:n], length, p, top, sink, top * p)
        assert counts[i] == count, (i, length)
        assert tokens[i].tolist() == want.tolist(), (i, length)
    assert not _lib.device_flags(DEV)


def test_long_table_batched_matches_oracle():
    """hs_quest_select_batched with a long table and few requests scores in
    partial mode and ranks over a cluster: same tokens as the oracle."""
    gen = torch.Generator().manual_seed(21)
    hq, hkv, d, p, top, max_pages = 28, 4, 128, 64, 128, 4200
    lengths = [max_pages * p, 1000, 3000 * p + 5]
    mins, maxs = [], []
    query = torch.randn(len(lengths), hq, d, generator=gen).to(torch.bfloat16)
    for _ in lengths:
        mn, mx = _metadata(gen, max_pages, hkv, d, torch.bfloat16)
        mins.append(mn)
        maxs.append(mx)
    lib = _lib.load()
    b, width = len(lengths), top * p
    dmins = [t.to(DEV) for t in mins]
    dmaxs = [t.to(DEV) for t in maxs]
    dq = query.to(DEV)
    tokens = torch.empty(b, width, dtype=torch.int32, device=DEV)
    counts = torch.empty(b, dtype=torch.int32, device=DEV)
    mptr = torch.tensor([t.data_ptr() for t in dmins], dtype=torch.int64, device=DEV)
    xptr = torch.tensor([t.data_ptr() for t in dmaxs], dtype=torch.int64, device=DEV)
    lens = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    nbytes = lib.hs_quest_workspace_bytes(b, max_pages)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    for sink in (True, False):
        _lib.check(lib.hs_quest_select_batched(
            b, dq.data_ptr(), hq * d, _lib.HS_BFLOAT16, mptr.data_ptr(), xptr.data_ptr(),
            _lib.HS_BFLOAT16, lens.data_ptr(), hq, hkv, d, max_pages, p, top, int(sink),
            tokens.data_ptr(), width, counts.data_ptr(), ws.data_ptr(), nbytes, 0,
            torch.cuda.current_stream().cuda_stream))
        for i, length in enumerate(lengths):
            want = oracle.quest_tokens(query[i], mins[i], maxs[i], length, p, top, sink)
            assert counts[i].item() == len(want)
            row = tokens[i].tolist()
            assert row[:len(want)] == want and set(row[len(want):]) <= {-1}
    assert not _lib.device_flags(DEV)
