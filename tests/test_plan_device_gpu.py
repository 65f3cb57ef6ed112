"""The device planner (aspire_plan_device): the same work list as the host
planner, identical attention outputs, and re-planning inside a replayed CUDA
graph from device arrays that change between replays."""

import ctypes

import numpy as np
import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.attention import HolisticAttentionWrapper, first_last_dump_jit_args
from aspire_b200.workloads import fill_tensors, full_context_layout, last_page_lens, make_layout
from gpu_helpers import MAX_ABS, MEAN_ABS, assert_attention_close, oracle_attention

pytestmark = pytest.mark.gpu

ITEM = ["row", "kv_head", "q_start", "q_len", "kv_page_base", "kv_len", "tok_begin", "tok_end", "pq_begin",
        "pq_end", "chunk", "n_chunks", "partial_base", "merge_id", "kind", "cols"]


def _decode(words):
    w = np.asarray(words, dtype=np.int32)
    n = int(w[1])
    items = w[w[5]:w[5] + 16 * n].reshape(-1, 16)
    merges = w[w[6]:w[6] + 8 * int(w[7])].reshape(-1, 8)
    return w, items, merges


def _canon(w, items, merges):
    """Order-free view: items keyed by their geometry with their merge group's
    descriptor instead of the merge index."""
    out = []
    for it in items:
        d = dict(zip(ITEM, map(int, it)))
        m = tuple(int(x) for x in merges[d["merge_id"]][:6]) if d["merge_id"] >= 0 else None
        if m is not None:
            assert m[4] == d["partial_base"] and m[5] == d["n_chunks"]
        out.append((d["row"], d["kv_head"], d["q_start"], d["q_len"], d["kv_page_base"], d["kv_len"],
                    d["tok_begin"], d["tok_end"], d["pq_begin"], d["pq_end"], d["chunk"], d["n_chunks"], d["kind"],
                    None if m is None else (m[0], m[1], m[2], m[3], m[5])))
    return sorted(out, key=lambda x: tuple(-1 if v is None else (hash(v) if isinstance(v, tuple) else v) for v in x))


def _host_plan(lay, num_sms):
    lib = _capi.load_library()
    buf = np.zeros(1 << 22, dtype=np.uint8)
    info = _capi.AspirePlanInfo()
    i32 = lambda a: np.ascontiguousarray(a, dtype=np.int32)  # noqa: E731
    qo, kvp, kvl = i32(lay.qo_indptr), i32(lay.kv_indptr), i32(lay.kv_lens)
    p = lambda a: a.ctypes.data_as(_capi.c_int32_p)  # noqa: E731
    rc = lib.aspire_plan_host_only(p(qo), p(kvp), p(kvl), lay.batch, lay.num_qo_heads, lay.num_kv_heads, 128, 16, 1,
                                   num_sms, buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes, 1 << 30,
                                   ctypes.byref(info))
    assert rc == 0, lib.aspire_last_error()
    return buf.view(np.int32)


def _prefill_layout(hq, hkv):
    """Prefill chunks: long queries over a cached prefix (several query tiles
    per row, each clipped to its causal span)."""
    q_lens = [600, 77, 1300, 1, 40]
    kv_lens = [600, 2077, 1400, 500, 40]
    lay = make_layout(batch=len(q_lens), ctx=2100, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.0,
                      budget_pages=8, seed=44)
    lay.q_lens = np.array(q_lens, np.int32)
    lay.kv_lens = np.array(kv_lens, np.int32)
    lay.qo_indptr = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    pages = [(k + 15) // 16 for k in kv_lens]
    lay.kv_indptr = np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)
    lay.kv_indices = np.concatenate([lay.block_table[r, :pages[r]] for r in range(len(q_lens))]).astype(np.int32)
    return lay


@pytest.mark.parametrize("hq,hkv,draft_fraction", [(32, 8, 0.5), (16, 8, 0.0), (32, 4, 1.0), (40, 8, 0.5),
                                                   (32, 8, "prefill"), (40, 8, "prefill")])
def test_device_plan_matches_host_plan(cuda_device, hq, hkv, draft_fraction):
    dev = cuda_device
    if draft_fraction == "prefill":
        lay = _prefill_layout(hq, hkv)
    else:
        lay = make_layout(batch=23, ctx=9000, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=draft_fraction,
                          budget_pages=48, seed=41)
    num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    w.plan_device(t(lay.qo_indptr), t(lay.kv_indptr), t(last_page_lens(lay)), hq, hkv, 128, 16,
                  paged_kv_indices=t(lay.kv_indices), causal=True)
    torch.cuda.synchronize()
    dev_words = w._int_workspace[256:].view(torch.int32).cpu().numpy()
    assert dev_words[0] == 0x41535042
    host_words = _host_plan(lay, num_sms)
    dw, ditems, dmerges = _decode(dev_words)
    hw, hitems, hmerges = _decode(host_words)
    assert len(ditems) == len(hitems) and len(dmerges) == len(hmerges)
    assert _canon(dw, ditems, dmerges) == _canon(hw, hitems, hmerges)
    # Each list (decode items, then prefill items from word 15 on) longest
    # first, and the claim counters armed.
    lens = (ditems[:, 7] - ditems[:, 6] + 127) // 128
    for lo, hi in ((0, dw[15]), (dw[15], len(ditems))):
        assert np.all(lens[lo:hi - 1] >= lens[lo + 1:hi])
    assert dw[14] == 0 and dw[16] == 0 and dw[4] == 0
    assert w.device_status() == 0


def test_device_plan_gives_identical_attention(cuda_device):
    dev = cuda_device
    lay = make_layout(batch=12, ctx=5000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=40,
                      seed=42)
    q, kv = fill_tensors(lay, device=dev, seed=43)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    idx = t(lay.kv_indices)
    host = HolisticAttentionWrapper(torch.empty(1, device=dev))
    host.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                   idx, 32, 8, 128, 16, causal=True)
    o1, l1 = host.run(q, kv, return_lse=True)
    devw = HolisticAttentionWrapper(torch.empty(1, device=dev))
    devw.plan_device(t(lay.qo_indptr), t(lay.kv_indptr), t(last_page_lens(lay)), 32, 8, 128, 16,
                     paged_kv_indices=idx, causal=True)
    o2, l2 = devw.run(q, kv, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(o2, l2, ref_out, ref_lse)


def test_device_plan_replans_inside_a_graph(cuda_device):
    """Plan + run captured once; each replay plans from the current contents of
    the device arrays (different lengths and page lists every time)."""
    dev = cuda_device
    batch, hq, hkv, ppr = 10, 32, 8, 200
    layouts = [make_layout(batch=batch, ctx=ctx, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.5,
                           budget_pages=24, pages_per_row=ppr, seed=50 + i) for i, ctx in enumerate((1500, 3000, 700))]
    _, kv = fill_tensors(layouts[1], device=dev, seed=51)
    max_q = max(int(l.qo_indptr[-1]) for l in layouts)
    max_pages = max(len(l.kv_indices) for l in layouts)
    g = torch.Generator(device=dev)
    g.manual_seed(52)
    q = torch.randn(max_q, hq, 128, generator=g, device=dev).to(torch.bfloat16)
    qo = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
    kvp = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
    lpl = torch.zeros(batch, dtype=torch.int32, device=dev)
    idx = torch.zeros(max_pages, dtype=torch.int32, device=dev)
    out = torch.zeros(max_q, hq, 128, dtype=torch.bfloat16, device=dev)
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))

    def load(lay):
        qo.copy_(torch.from_numpy(lay.qo_indptr.astype(np.int32)))
        kvp.copy_(torch.from_numpy(lay.kv_indptr.astype(np.int32)))
        lpl.copy_(torch.from_numpy(last_page_lens(lay)))
        idx[:len(lay.kv_indices)].copy_(torch.from_numpy(lay.kv_indices.astype(np.int32)))

    def step():
        w.plan_device(qo, kvp, lpl, hq, hkv, 128, 16, paged_kv_indices=idx, causal=True)
        w.run(q, kv, out=out)

    load(layouts[0])
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for lay in layouts:
        load(lay)
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        ref = HolisticAttentionWrapper(torch.empty(1, device=dev))
        ref.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr),
                      torch.from_numpy(lay.kv_lens), idx, hq, hkv, 128, 16, causal=True)
        n = int(lay.qo_indptr[-1])
        expect = ref.run(q[:n], kv)
        torch.cuda.synchronize()
        assert torch.equal(out[:n], expect)
        o_ref, _, _ = oracle_attention(lay, q[:n], kv)
        err = (out[:n].float().cpu() - o_ref).abs()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS
    del graph


def test_device_plan_reports_bad_rows(cuda_device):
    dev = cuda_device
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w.clear_device_status()
    t = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)  # noqa: E731
    # Row 0 claims 40 tokens on 2 pages (last page length 24 > 16 is impossible).
    w.plan_device(t([0, 1]), t([0, 2]), t([24]), 32, 8, 128, 16, paged_kv_indices=t([0, 1]), causal=True)
    q = torch.randn(1, 32, 128, device=dev).to(torch.bfloat16)
    kv = torch.zeros(4, 2, 16, 8, 128, dtype=torch.bfloat16, device=dev)
    out = torch.full((1, 32, 128), 7.0, dtype=torch.bfloat16, device=dev)
    w.run(q, kv, out=out)
    torch.cuda.synchronize()
    assert w.device_status() & _capi.STATUS_BAD_PLAN
    assert bool((out == 7.0).all())  # the program skipped the invalid plan
