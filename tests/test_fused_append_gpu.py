"""The fused KV append: ``run(..., append=(k_new, v_new))`` writes each row's
new tokens into the cache inside the attention launch, before the row's keys
are read.  It must leave the cache bit-identical to the separate append
(``append_kv`` with the same qo_indptr and page source, the reference's
mylib::update_kv_padded, aspire/attention/kv_ops.py:127-187) followed by the
attention, with bit-identical outputs and LSE, and agree with the oracle.

Cases: a mixed draft/verify batch through a flat page list and through the
page tables (draft rows' new token lands in the last page of their draft
table), the refresh program with its dump, a row whose new tokens straddle a
split-KV chunk boundary (two items each write their part), CUDA-graph
replay, and the plans it refuses (prefill rows, device-side plans)."""

import numpy as np
import pytest
import torch

from aspire_b200.attention import HolisticAttentionWrapper, first_last_dump_jit_args
from aspire_b200.kv_ops import append_kv
from aspire_b200.workloads import fill_tensors, full_context_layout, last_page_lens, make_layout, rows_layout
from gpu_helpers import assert_attention_close, oracle_attention

pytestmark = pytest.mark.gpu


def _i32(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)


def _tables(lay, dev):
    counts = np.diff(lay.kv_indptr)
    draft = np.zeros((lay.batch, max(1, int(counts.max()))), np.int32)
    for b in range(lay.batch):
        if lay.modes[b] == 0:
            draft[b, :counts[b]] = lay.kv_indices[lay.kv_indptr[b]:lay.kv_indptr[b + 1]]
    return _i32(lay.modes, dev), _i32(draft, dev), _i32(lay.block_table, dev)


def _new_tokens(lay, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    T = int(lay.qo_indptr[-1])
    k = torch.randn(T, lay.num_kv_heads, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(T, lay.num_kv_heads, 128, generator=g, device=dev).to(torch.bfloat16)
    return k, v


def _both_ways(lay, q, kv0, k_new, v_new, dev, *, tables=False, dump_stride=0):
    """(cache, out, lse, dump) after separate append + attention, and after
    the fused launch, from the same starting cache."""
    res = []
    for fused in (False, True):
        kv = kv0.clone()
        jit = first_last_dump_jit_args() if dump_stride else None
        w = HolisticAttentionWrapper(torch.empty(1, device=dev), jit_args=jit)
        page_tables = None
        indices = _i32(lay.kv_indices, dev)
        if tables:
            page_tables = _tables(lay, dev)
            w.set_page_tables(*page_tables)
        w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                    None if tables else indices, lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)
        args = []
        dump = None
        if dump_stride:
            dump = torch.full((lay.batch * lay.num_qo_heads * 2 * dump_stride,), float("-inf"),
                              dtype=torch.float16, device=dev)
            args = [dump, lay.num_qo_heads, dump_stride]
        if fused:
            out, lse = w.run(q, kv, *args, return_lse=True, append=(k_new, v_new))
        else:
            append_kv(k_new, v_new, _i32(lay.qo_indptr, dev), kv, None if tables else indices,
                      _i32(lay.kv_indptr, dev), _i32(last_page_lens(lay), dev), 16, page_tables=page_tables)
            out, lse = w.run(q, kv, *args, return_lse=True)
        torch.cuda.synchronize()
        assert w.device_status() == 0
        res.append((kv, out, lse, dump))
    return res


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (8, 1)])
@pytest.mark.parametrize("tables", [False, True], ids=["page_list", "page_tables"])
def test_fused_append_matches_separate_append(cuda_device, tables, hq, hkv):
    dev = cuda_device
    lay = make_layout(batch=12, ctx=3000, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.5, budget_pages=40,
                      seed=61 + hq + hkv, block_table="random")
    q, kv0 = fill_tensors(lay, device=dev, seed=62)
    k_new, v_new = _new_tokens(lay, dev, 63)
    (kv_a, out_a, lse_a, _), (kv_b, out_b, lse_b, _) = _both_ways(lay, q, kv0, k_new, v_new, dev, tables=tables)
    assert not torch.equal(kv_a, kv0), "the append wrote nothing"
    assert torch.equal(kv_a, kv_b) and torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv_a)
    assert_attention_close(out_b, lse_b, ref_out, ref_lse)


def test_fused_append_refresh_program_with_dump(cuda_device):
    dev = cuda_device
    lay = make_layout(batch=6, ctx=2000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=24,
                      seed=64, block_table="random")
    full = full_context_layout(lay)
    q, kv0 = fill_tensors(full, device=dev, seed=65)
    k_new, v_new = _new_tokens(full, dev, 66)
    stride = lay.pages_per_row * 16
    (kv_a, out_a, lse_a, d_a), (kv_b, out_b, lse_b, d_b) = _both_ways(full, q, kv0, k_new, v_new, dev,
                                                                      dump_stride=stride)
    assert torch.equal(kv_a, kv_b) and torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert torch.equal(d_a, d_b)


def test_fused_append_across_a_chunk_boundary(cuda_device):
    """One verify row of 1028 keys and 9 queries: the plan splits its keys in
    512-token chunks, so its new tokens (1019..1027) span two items."""
    dev = cuda_device
    lay = rows_layout([9, 1, 5], [1028, 700, 1024 + 3], 32, 8, seed=67)
    q, kv0 = fill_tensors(lay, device=dev, seed=68)
    k_new, v_new = _new_tokens(lay, dev, 69)
    (kv_a, out_a, lse_a, _), (kv_b, out_b, lse_b, _) = _both_ways(lay, q, kv0, k_new, v_new, dev)
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                _i32(lay.kv_indices, dev), 32, 8, 128, 16, causal=True)
    assert w.plan_info.chunk_tokens <= 1024 and w.plan_info.num_merge > 0, "the row must be split"
    assert torch.equal(kv_a, kv_b) and torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)


def test_fused_append_graph_replay(cuda_device):
    """Captured once, replayed: the same cache and outputs as the eager fused
    launch (the append is part of the graph's attention node)."""
    dev = cuda_device
    lay = make_layout(batch=8, ctx=2500, num_qo_heads=16, num_kv_heads=8, draft_fraction=0.5, budget_pages=32,
                      seed=70)
    q, kv0 = fill_tensors(lay, device=dev, seed=71)
    k_new, v_new = _new_tokens(lay, dev, 72)
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w.set_page_tables(*_tables(lay, dev))
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                None, 16, 8, 128, 16, causal=True)
    kv_e = kv0.clone()
    out_e = w.run(q, kv_e, append=(k_new, v_new))
    kv_g = kv0.clone()
    out_g = torch.empty_like(q)
    w.run(q, kv_g, out=out_g, append=(k_new, v_new))
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        w.run(q, kv_g, out=out_g, append=(k_new, v_new))
    kv_g.copy_(kv0)
    out_g.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(kv_g, kv_e) and torch.equal(out_g, out_e)
    del graph


def test_fused_append_refuses_other_plans(cuda_device):
    """Prefill rows read each other's new tokens across items, and a device
    plan is not known to the host: both must append separately."""
    dev = cuda_device
    lay = rows_layout([300, 1], [1000, 500], 32, 8, seed=73)
    q, kv = fill_tensors(lay, device=dev, seed=74)
    k_new, v_new = _new_tokens(lay, dev, 75)
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                _i32(lay.kv_indices, dev), 32, 8, 128, 16, causal=True)
    assert w.plan_info.num_items_prefill > 0
    with pytest.raises((ValueError, RuntimeError), match="fused append"):
        w.run(q, kv, append=(k_new, v_new))
    lay2 = make_layout(batch=4, ctx=1000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=16,
                       seed=76)
    q2, kv2 = fill_tensors(lay2, device=dev, seed=77)
    k2, v2 = _new_tokens(lay2, dev, 78)
    w2 = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w2.plan_device(_i32(lay2.qo_indptr, dev), _i32(lay2.kv_indptr, dev), _i32(last_page_lens(lay2), dev), 32, 8,
                   128, 16, paged_kv_indices=_i32(lay2.kv_indices, dev), causal=True)
    with pytest.raises((ValueError, RuntimeError), match="fused append"):
        w2.run(q2, kv2, append=(k2, v2))
