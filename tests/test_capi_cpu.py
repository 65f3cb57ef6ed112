"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and the host planner covers every (row, head, token) once."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from aspire_b200 import _capi
from aspire_b200.workloads import make_layout

HEADER = Path(__file__).resolve().parent.parent / "include" / "aspire_b200.h"
ITEM_FIELDS = ["row", "kv_head", "q_start", "q_len", "kv_page_base", "kv_len", "tok_begin", "tok_end",
               "pq_begin", "pq_end", "chunk", "n_chunks", "partial_base", "merge_id", "kind", "cols"]


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"ASPIRE_API\s+[\w\s\*]+?\b(aspire_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(built_library):
    declared = header_functions()
    assert declared, "no ASPIRE_API declarations found"
    for name in declared:
        assert hasattr(built_library, name), name
    assert set(declared) == set(_capi.exported_symbols())
    assert built_library.aspire_abi_version() == _capi.EXPECTED_ABI_VERSION == 5
    assert built_library.aspire_status_offset() == 256


def _plan(lib, qo, kvp, kvl, hq, hkv, num_sms=8, float_ws=1 << 30, causal=1):
    qo = np.ascontiguousarray(qo, dtype=np.int32)
    kvp = np.ascontiguousarray(kvp, dtype=np.int32)
    kvl = np.ascontiguousarray(kvl, dtype=np.int32)
    buf = np.zeros(1 << 22, dtype=np.uint8)
    info = _capi.AspirePlanInfo()
    p = lambda a: a.ctypes.data_as(_capi.c_int32_p)  # noqa: E731
    rc = lib.aspire_plan_host_only(p(qo), p(kvp), p(kvl), len(kvl), hq, hkv, 128, 16, causal, num_sms,
                                   buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes, float_ws, ctypes.byref(info))
    return rc, info, buf


def _decode(buf, info):
    w = buf.view(np.int32)
    off_items = w[5]
    items = w[off_items: off_items + info.num_items * 16].reshape(-1, 16)
    return w, [dict(zip(ITEM_FIELDS, map(int, r))) for r in items]


def _check_coverage(lay, info, buf):
    """Every (row, KV head, packed query) sees keys [0, kv_len) exactly once
    over its items; merge descriptors, list order and CTA indptrs agree."""
    w, items = _decode(buf, info)
    assert w[0] == 0x41535042
    assert int(w[17]) == info.chunk_tokens  # the plan's common chunk length
    group = lay.num_qo_heads // lay.num_kv_heads
    cover = {}
    for it in items:
        for pq in range(it["pq_begin"], it["pq_end"]):
            key = (it["row"], it["kv_head"], pq)
            cover.setdefault(key, []).append((it["tok_begin"], it["tok_end"]))
        assert 0 <= it["chunk"] < it["n_chunks"]
        assert (it["merge_id"] >= 0) == (it["n_chunks"] > 1)
        if it["merge_id"] >= 0:
            md = w[w[6] + 8 * it["merge_id"]: w[6] + 8 * it["merge_id"] + 8]
            assert md[2] == it["pq_end"] - it["pq_begin"] and md[5] == it["n_chunks"]
            assert md[4] == it["partial_base"] and md[3] == it["kv_head"]
    for b in range(lay.batch):
        nq = int(lay.q_lens[b]) * group
        for h in range(lay.num_kv_heads):
            for pq in range(nq):
                ranges = sorted(cover[(b, h, pq)])
                assert ranges[0][0] == 0 and ranges[-1][1] == int(lay.kv_lens[b])
                for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                    assert a1 == b0
    # tcgen05 decode items follow the CUDA-core items, then the prefill items;
    # each list longest first (claimed in that order at run time); the claim
    # counters start at zero.
    assert w[4] == info.num_items_gather and w[14] == 0 and w[16] == 0
    assert w[15] == info.num_items_gather + info.num_items_tc
    assert w[1] == w[15] + info.num_items_prefill
    for lo, hi in ((w[4], w[15]), (w[15], w[1])):
        cost = [it["tok_end"] - it["tok_begin"] for it in items[lo:hi]]
        assert all(a >= b for a, b in zip(cost, cost[1:]))
    # CTA indptrs partition the CUDA-core item list.
    g_ctas = w[2]
    g_indptr = w[w[3]: w[3] + g_ctas + 1]
    assert g_indptr[0] == 0 and np.all(np.diff(g_indptr) >= 0)
    assert g_indptr[-1] == info.num_items_gather
    return items


@pytest.mark.parametrize("draft_fraction", [0.0, 0.5, 1.0])
def test_plan_covers_every_token_once(built_library, draft_fraction):
    lay = make_layout(batch=12, ctx=3000, num_qo_heads=32, num_kv_heads=8, draft_fraction=draft_fraction,
                      budget_pages=40, seed=3)
    rc, info, buf = _plan(built_library, lay.qo_indptr, lay.kv_indptr, lay.kv_lens, 32, 8)
    assert rc == 0, built_library.aspire_last_error()
    _check_coverage(lay, info, buf)


@pytest.mark.parametrize("batch,ctx,draft_fraction,hq,hkv", [(1, 2000, 0.0, 32, 8), (2, 1500, 0.5, 16, 8),
                                                              (4, 900, 1.0, 32, 8), (3, 5000, 0.5, 8, 1)])
def test_small_plans_cover_every_token_once(built_library, batch, ctx, draft_fraction, hq, hkv):
    """Small batches on 148 SMs, the plans the small-plan and item-width rules
    shape: 256-token chunks where the split plan keeps at most a quarter of
    the SMs busy, long verify items padded to one width."""
    lay = make_layout(batch=batch, ctx=ctx, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=draft_fraction,
                      budget_pages=16, seed=batch)
    rc, info, buf = _plan(built_library, lay.qo_indptr, lay.kv_indptr, lay.kv_lens, hq, hkv, num_sms=148)
    assert rc == 0, built_library.aspire_last_error()
    items = _check_coverage(lay, info, buf)
    _check_item_columns(items, info, 148)
    # Spans per (row, query tile of 48 packed rows), as the planner groups them:
    # the tile with query 0 sees every key, a later one keys up to its last query.
    group, spans = hq // hkv, []
    for ql, kl in zip(lay.q_lens.tolist(), lay.kv_lens.tolist()):
        tile = 48 // group * group
        for p0 in range(0, ql * group, tile):
            p1 = min(ql * group, p0 + tile)
            spans.append(kl if p0 < group else min(kl, kl - ql + (p1 - 1) // group + 1))
    assert info.chunk_tokens == _expected_chunk(spans, hkv, 148)


def test_plan_balances_ctas(built_library):
    lay = make_layout(batch=64, ctx=32768, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5,
                      budget_pages=128, seed=0)
    rc, info, buf = _plan(built_library, lay.qo_indptr, lay.kv_indptr, lay.kv_lens, 32, 8, num_sms=148)
    assert rc == 0, built_library.aspire_last_error()
    w, items = _decode(buf, info)
    loads = {}
    for i, it in enumerate(items):
        loads.setdefault(it["kind"], []).append(it["tok_end"] - it["tok_begin"])
    assert info.partial_rows * 129 * 4 == info.float_bytes
    assert info.float_bytes < 128 * 1024 * 1024


def _expected_chunk(spans, hkv, num_sms):
    """The planner's chunk rule, restated: about four items per SM when the
    groups' spans are within 2x of each other, else about two; but every
    group whole (chunk = longest span rounded up to 128, at least 512) when
    the whole-group makespan estimate is no worse than the split one (in
    tenths of a 128-token tile: an item boundary 2.3 tiles, the merge 2.5);
    few long groups cut into one piece per SM; and 256-token chunks for a
    split plan at 512 that keeps at most a quarter of the SMs busy."""
    total = sum(max(s, 1) for s in spans) * hkv
    cdiv = lambda a, b: -(-a // b)  # noqa: E731

    def chunk_for(per_cta):
        target = num_sms * per_cta
        c = max(cdiv(total, target), 512)
        return cdiv(c, 128) * 128

    similar = 2 * min(spans) >= max(spans)
    chunk = chunk_for(4 if similar else 2)
    if not similar:
        # Long groups (span > max / 2) cut into k = SMs / n_long pieces each,
        # when the short groups (tiles + 2.3 per group) fit the spare SMs.
        mx = max(spans)
        n_long = sum(2 * s > mx for s in spans) * hkv
        short = sum(cdiv(s, 128) * 10 + 23 for s in spans if 2 * s <= mx) * hkv
        k = num_sms // n_long if n_long else 0
        if k >= 1:
            c = max(512, cdiv(cdiv(mx, k), 128) * 128)
            spare = num_sms - n_long * cdiv(mx, c)
            if spare >= 0 and short <= spare * (c // 128 * 10 + 23):
                chunk = c
    n_groups = len(spans) * hkv
    n_items = sum(cdiv(s, chunk) if s > 0 else 1 for s in spans) * hkv
    whole = cdiv(n_groups, num_sms) * (cdiv(max(spans), 128) * 10 + 23)
    split = (max(cdiv(total * 10, 128 * num_sms), chunk // 128 * 10) + cdiv(n_items, num_sms) * 23
             + (25 if n_items > n_groups else 0))
    if whole <= split:
        return max(512, cdiv(max(spans), 128) * 128)
    # A split plan at the 512 minimum on at most a quarter of the SMs: 256.
    return 256 if chunk == 512 and n_items > n_groups and 4 * n_items <= num_sms else chunk


def _check_item_columns(items, info, num_sms):
    """Product columns of the tcgen05 decode items (WorkItem.cols): when the
    decode list has at most two items per SM, every item of a long group
    (span above half the longest) takes the widest long group's width
    (packed rows rounded up to 16), other items 0 (their own width); with
    more items, all 0."""
    tc = [it for it in items if it["kind"] == 1]
    assert all(it["cols"] == 0 for it in items if it["kind"] != 1)
    if not tc:
        return
    r16 = lambda n: -(-n // 16) * 16  # noqa: E731
    span = {}
    for it in tc:
        key = (it["row"], it["kv_head"], it["pq_begin"])
        span[key] = max(span.get(key, 0), it["tok_end"])
    longest = max(span.values())
    long_of = lambda it: 2 * span[(it["row"], it["kv_head"], it["pq_begin"])] > longest  # noqa: E731
    if len(tc) <= 2 * num_sms:
        width = max(r16(it["pq_end"] - it["pq_begin"]) for it in tc if long_of(it))
        for it in tc:
            assert it["cols"] == (width if long_of(it) else 0), it
    else:
        assert all(it["cols"] == 0 for it in tc)


@pytest.mark.parametrize("case", ["mixed", "mixed_tp4", "mixed_tp8", "full_context", "prefill_spread", "draft_b1",
                                  "draft_b4", "draft_b16", "draft_b32"])
def test_plan_chunk_rule(built_library, case):
    """Decode batches (long verify rows beside short draft rows) get about two
    items per SM; whole-context rows of equal length, four; the spread-out
    query tiles of a causal prefill chunk stay whole at two per SM.  When the
    long groups are fewer than the SMs (the TP-4 and TP-8 head shares of the
    decode batch), each is cut into SMs / long groups pieces.  Medium
    draft-only batches keep every group whole (one item each, no merge): 16
    rows over 64 pages at 32 / 8 heads, 32 rows over 136 pages at 16 / 8; one
    row over 64 pages is still split, into 256-token chunks (its 8 groups
    use 32 SMs), four rows into 512-token chunks."""
    num_sms = 148
    if case.startswith("draft_"):
        B, pages, hq, hkv = {"draft_b1": (1, 64, 32, 8), "draft_b4": (4, 64, 32, 8), "draft_b16": (16, 64, 32, 8),
                             "draft_b32": (32, 136, 16, 8)}[case]
        kvl = np.full(B, pages * 16, np.int32)
        qo = np.arange(B + 1, dtype=np.int32)
        kvp = (np.arange(B + 1) * pages).astype(np.int32)
        rc, info, _ = _plan(built_library, qo, kvp, kvl, hq, hkv, num_sms=num_sms)
        assert rc == 0, built_library.aspire_last_error()
        assert info.chunk_tokens == _expected_chunk([pages * 16] * B, hkv, num_sms)
        if case == "draft_b1":  # 16 items at 512 tokens on 148 SMs: cut at 256
            assert info.chunk_tokens == 256 and info.num_merge == B * hkv
        elif case == "draft_b4":  # 64 items at 512 tokens: more than a quarter of the SMs
            assert info.chunk_tokens == 512 and info.num_merge == B * hkv
        else:
            assert info.chunk_tokens == pages * 16
            assert info.num_merge == 0 and info.num_items_tc == B * hkv
        return
    hq, hkv = 32, 8
    if case.startswith("mixed"):
        # The bench's batch at TP 1 and at the TP-4 / TP-8 head shares (2 and 1
        # KV heads): at the shares the verify groups are cut into one piece per SM.
        hq, hkv = {"mixed": (32, 8), "mixed_tp4": (8, 2), "mixed_tp8": (4, 1)}[case]
        lay = make_layout(batch=64, ctx=32768, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.5,
                          budget_pages=128, seed=0)
        qo, kvp, kvl = lay.qo_indptr, lay.kv_indptr, lay.kv_lens
        spans = [int(k) for k in kvl]
    elif case == "full_context":
        kvl = np.full(64, 32773, np.int32)
        qo = np.arange(65, dtype=np.int32)
        kvp = np.concatenate([[0], np.cumsum((kvl + 15) // 16)]).astype(np.int32)
        spans = [int(k) for k in kvl]
    else:  # one 8192-token prefill chunk: 128 query tiles of 64 positions (group 4), each
        # stopping at its causal span except the tile holding query 0 (all keys)
        kvl = np.array([8192], np.int32)
        qo = np.array([0, 8192], np.int32)
        kvp = np.array([0, 512], np.int32)
        spans = [8192] + [64 * (t + 1) for t in range(1, 128)]
    rc, info, buf = _plan(built_library, qo, kvp, kvl, hq, hkv, num_sms=num_sms)
    assert rc == 0, built_library.aspire_last_error()
    assert info.chunk_tokens == _expected_chunk(spans, hkv, num_sms)
    _, items = _decode(buf, info)
    _check_item_columns(items, info, num_sms)
    if case == "mixed":
        assert info.num_items_tc == 768  # verify rows in two chunks, draft rows whole
    if case in ("mixed_tp4", "mixed_tp8"):
        assert info.chunk_tokens == {"mixed_tp4": 16384, "mixed_tp8": 8192}[case]
        # verify rows of 3-9 queries x 4 heads: all 48 columns
        assert {it["cols"] for it in items if it["kind"] == 1 and it["q_len"] > 1} == {48}
    if case == "mixed":
        assert all(it["cols"] == 0 for it in items)
    if case == "prefill_spread":
        assert info.num_merge == 0 and info.num_items_prefill == 128 * 8


def test_plan_rejects_bad_input(built_library):
    rc, _, _ = _plan(built_library, [0, 1], [0, 1], [17], 32, 8)  # 17 tokens need 2 pages
    assert rc == _capi.ASPIRE_ERR_INVALID
    assert b"exceeds its page list" in built_library.aspire_last_error()
    rc, _, _ = _plan(built_library, [0, 1], [0, 1], [5], 30, 8)  # heads not a multiple
    assert rc == _capi.ASPIRE_ERR_INVALID
    # 8 groups of 64k tokens on 148 SMs split into chunks, whose partials need float workspace.
    rc, _, _ = _plan(built_library, [0, 1], [0, 4096], [65536], 32, 8, num_sms=148, float_ws=16)
    assert rc == _capi.ASPIRE_ERR_CAPACITY


def test_plan_handles_empty_and_padding_rows(built_library):
    # row 0 empty (q_len 0), row 1 kv_len 0 with queries (bucket padding), row 2 normal.
    rc, info, buf = _plan(built_library, [0, 0, 3, 4], [0, 0, 0, 2], [0, 0, 20], 16, 8)
    assert rc == 0, built_library.aspire_last_error()
    _, items = _decode(buf, info)
    rows = {it["row"] for it in items}
    assert rows == {1, 2}
    assert all(it["tok_begin"] == it["tok_end"] == 0 for it in items if it["row"] == 1)


@pytest.mark.parametrize("q_len,group", [(600, 4), (130, 1), (45, 3), (17, 8)])
def test_plan_clips_causal_tiles_to_their_span(built_library, q_len, group):
    """A prefill row (q_len queries over as many keys): prefill items of two
    halves of (128 // group) query positions each; item i > 0 covers keys up
    to its last query's; the item holding query 0 keeps all keys (the dump
    records its raw logits everywhere)."""
    kvh = 2
    pages = (q_len + 15) // 16
    rc, info, buf = _plan(built_library, [0, q_len], [0, pages], [q_len], kvh * group, kvh, num_sms=148)
    assert rc == 0, built_library.aspire_last_error()
    w, items = _decode(buf, info)
    nq = q_len * group
    item_rows = 2 * (128 // group) * group
    assert info.num_items_tc == 0 and info.num_items_prefill == len(items) and w[15] == 0
    span = {}
    for it in items:
        assert it["kind"] == 2 and it["pq_begin"] % item_rows == 0
        assert it["pq_end"] == min(it["pq_begin"] + item_rows, nq)
        key = (it["kv_head"], it["pq_begin"])
        span[key] = max(span.get(key, 0), it["tok_end"])
        assert it["tok_begin"] <= it["tok_end"]
    assert len(span) == kvh * ((nq + item_rows - 1) // item_rows)
    for (h, pq0), end in span.items():
        q_last = (min(pq0 + item_rows, nq) - 1) // group
        assert end == (q_len if pq0 == 0 else q_last + 1), (h, pq0, end)


def test_plan_keeps_every_query0_tile_whole(built_library, monkeypatch):
    """With the group wider than the CUDA-core tile (4 packed rows), query 0's
    heads span several tiles; all of them keep every key for the dump."""
    monkeypatch.setenv("ASPIRE_B200_DISABLE_TC", "1")  # every row on 4-row CUDA-core tiles
    rc, info, buf = _plan(built_library, [0, 20], [0, 63], [1000], 64, 8)  # group 8
    assert rc == 0, built_library.aspire_last_error()
    _, items = _decode(buf, info)
    assert info.num_items_gather == len(items)
    assert {it["pq_begin"] for it in items if it["pq_begin"] < 8} == {0, 4}
    for it in items:
        if it["pq_begin"] < 8:
            assert max(i["tok_end"] for i in items
                       if i["pq_begin"] == it["pq_begin"] and i["kv_head"] == it["kv_head"]) == 1000


def _attn_args(**over):
    """Attention args with plausible, 16-byte aligned (but never dereferenced)
    addresses; the cases below are rejected before any CUDA call."""
    a = _capi.AspireAttnArgs()
    a.q, a.kv_cache, a.out, a.kv_indices = 0x10000, 0x20000, 0x30000, 0x40000
    a.q_stride_n, a.q_stride_h, a.o_stride_n, a.o_stride_h = 32 * 128, 128, 32 * 128, 128
    a.num_pages_total, a.q_rows = 100, 12
    a.num_qo_heads, a.num_kv_heads, a.head_dim, a.page_size = 32, 8, 128, 16
    for k, v in over.items():
        setattr(a, k, v)
    return a


def _plan_info(**over):
    info = _capi.AspirePlanInfo()
    info.num_qo_heads, info.num_kv_heads, info.tc_enabled = 32, 8, 1
    for k, v in over.items():
        setattr(info, k, v)
    return info


@pytest.mark.parametrize("case,args,plan,msg", [
    ("dump_kind", dict(dump=0x50000, dump_num_heads=32, dump_kv_stride=1024, dump_kind=7), {}, b"dump_kind"),
    ("dump_dtype", dict(dump=0x50000, dump_num_heads=32, dump_kv_stride=1024, dump_dtype=3), {}, b"dump_dtype"),
    ("dump_f32_align", dict(dump=0x50002, dump_num_heads=32, dump_kv_stride=1024, dump_dtype=1), {},
     b"not aligned to its element type"),
    ("append_half", dict(k_new=0x60000), {}, b"needs k_new and v_new"),
    ("append_device_plan", dict(k_new=0x60000, v_new=0x70000), dict(on_device=1), b"fused append"),
    ("append_prefill", dict(k_new=0x60000, v_new=0x70000), dict(num_items_prefill=3), b"fused append"),
    ("append_gather", dict(k_new=0x60000, v_new=0x70000), dict(num_items_gather=3), b"fused append"),
    ("append_stride", dict(k_new=0x60000, v_new=0x70000, k_new_stride_n=1028, k_new_stride_h=128,
                           v_new_stride_n=1024, v_new_stride_h=128), {}, b"multiples of 8"),
    ("append_align", dict(k_new=0x60008, v_new=0x70000), {}, b"16-byte aligned"),
])
def test_attention_rejects_bad_dump_and_append_args(built_library, case, args, plan, msg):
    a = _attn_args(**args)
    info = _plan_info(**plan)
    rc = built_library.aspire_mixed_attention(ctypes.byref(a), ctypes.byref(info), None)
    assert rc == _capi.ASPIRE_ERR_INVALID, (case, rc)
    assert msg in built_library.aspire_last_error(), built_library.aspire_last_error()
