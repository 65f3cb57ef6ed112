"""Page-table mode: the attention and the append read each row's pages from
the draft table / block table by mode flag (build_unified_indices absorbed,
the reference's aspire/models/sparse_draft_runner.py:126-153).  Results must
be bit-identical to the flat page-list mode on the same pages, and agree with
the oracle (attention within the bf16 tolerance, append bit-exact)."""

import numpy as np
import pytest
import torch

from aspire_b200.attention import HolisticAttentionWrapper, dump_jit_args, first_last_dump_jit_args
from aspire_b200.kv_ops import append_kv
from aspire_b200.workloads import fill_tensors, full_context_layout, last_page_lens, make_layout
from gpu_helpers import assert_attention_close, assert_dump_close, oracle_attention
from oracle import kv_append as oracle_append

pytestmark = pytest.mark.gpu


def _tables(lay, dev, table_cols=None):
    """Mode flags, a draft table holding each draft row's page list (padded
    with garbage past the count) and the block table, as the engine keeps them."""
    counts = np.diff(lay.kv_indptr)
    cols = table_cols or int(counts.max())
    rng = np.random.default_rng(7)
    draft = rng.integers(0, lay.num_pages_total, size=(lay.batch, cols)).astype(np.int32)
    for b in range(lay.batch):
        if lay.modes[b] == 0:
            draft[b, :counts[b]] = lay.kv_indices[lay.kv_indptr[b]:lay.kv_indptr[b + 1]]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    # The block table gets padding columns too, so its row stride differs from its width.
    bt = np.full((lay.batch, lay.block_table.shape[1] + 5), -1, np.int32)
    bt[:, :lay.block_table.shape[1]] = lay.block_table
    return t(lay.modes), t(draft), t(bt)[:, :lay.block_table.shape[1]]


def _plan(w, lay, dev, indices):
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                indices, lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 8)])
def test_attention_page_tables_match_flat_list(cuda_device, hq, hkv):
    dev = cuda_device
    lay = make_layout(batch=9, ctx=3000, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.5, budget_pages=40,
                      seed=11, block_table="random")
    q, kv = fill_tensors(lay, device=dev, seed=12)
    flat = HolisticAttentionWrapper(torch.empty(1, device=dev))
    _plan(flat, lay, dev, torch.from_numpy(lay.kv_indices).to(dev))
    out_flat, lse_flat = flat.run(q, kv, return_lse=True)
    tab = HolisticAttentionWrapper(torch.empty(1, device=dev))
    tab.set_page_tables(*_tables(lay, dev))
    _plan(tab, lay, dev, None)
    out_tab, lse_tab = tab.run(q, kv, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(out_flat, out_tab)
    assert torch.equal(lse_flat, lse_tab)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out_tab, lse_tab, ref_out, ref_lse)


def test_refresh_dump_page_tables_match_flat_list(cuda_device):
    dev = cuda_device
    lay = make_layout(batch=6, ctx=2000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=24,
                      seed=13, block_table="random")
    full = full_context_layout(lay)
    q, kv = fill_tensors(full, device=dev, seed=14)
    stride = lay.pages_per_row * 16
    outs = []
    for use_tables in (False, True):
        w = HolisticAttentionWrapper(torch.empty(1, device=dev), jit_args=first_last_dump_jit_args())
        if use_tables:
            _, draft, bt = _tables(full, dev)
            w.set_page_tables(torch.ones(full.batch, dtype=torch.int32, device=dev), draft, bt)
            _plan(w, full, dev, None)
        else:
            _plan(w, full, dev, torch.from_numpy(full.kv_indices).to(dev))
        dump = torch.full((full.batch * 32 * 2 * stride,), float("-inf"), dtype=torch.float16, device=dev)
        out, lse = w.run(q, kv, dump, 32, stride, return_lse=True)
        outs.append((out, lse, dump))
    torch.cuda.synchronize()
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    ref_out, ref_lse, ref_dump = oracle_attention(full, q, kv, dump_stride=stride)
    assert_attention_close(outs[1][0], outs[1][1], ref_out, ref_lse)
    assert_dump_close(outs[1][2], ref_dump, full, stride)


def test_last_token_flagged_dump_device_plan_tables_graph(cuda_device):
    """The last-token dump with per-row mode flags into an fp32 buffer (the
    base backend's variant), planned on the device inside a CUDA graph with
    the pages read from the tables: bit-identical to the host-planned
    flat-list launch, rows flagged off untouched, and the oracle's dump."""
    dev = cuda_device
    lay = make_layout(batch=6, ctx=2000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=24,
                      seed=41, block_table="random")
    full = full_context_layout(lay)
    q, kv = fill_tensors(full, device=dev, seed=42)
    stride = lay.pages_per_row * 16
    H = full.num_qo_heads
    flags = torch.tensor([1, 0, 1, 1, 0, 1], dtype=torch.int32, device=dev)
    jit = dump_jit_args("last_token", use_mode_flags=True, dump_buffer_dtype=torch.float32)
    new_dump = lambda: torch.full((full.batch * H * stride,), float("-inf"), dtype=torch.float32, device=dev)  # noqa: E731

    w1 = HolisticAttentionWrapper(torch.empty(1, device=dev), jit_args=jit)
    _plan(w1, full, dev, torch.from_numpy(full.kv_indices).to(dev))
    d1 = new_dump()
    out1, lse1 = w1.run(q, kv, d1, flags, H, stride, return_lse=True)

    w2 = HolisticAttentionWrapper(torch.empty(1, device=dev), jit_args=jit)
    _, draft, bt = _tables(full, dev)
    w2.set_page_tables(torch.ones(full.batch, dtype=torch.int32, device=dev), draft, bt)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    qo, kvp, lpl = t(full.qo_indptr), t(full.kv_indptr), t(last_page_lens(full))
    d2 = new_dump()
    out2 = torch.empty_like(q)
    lse2 = torch.empty(q.shape[0], H, dtype=torch.float32, device=dev)

    def step():
        w2.plan_device(qo, kvp, lpl, H, full.num_kv_heads, 128, 16, causal=True)
        w2.run(q, kv, d2, flags, H, stride, out=out2, lse=lse2)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    d2.fill_(float("-inf"))
    out2.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert w2.device_status() == 0
    assert torch.equal(d1, d2) and torch.equal(out1, out2) and torch.equal(lse1, lse2)
    ref_out, ref_lse, ref_dump = oracle_attention(full, q, kv, dump_stride=stride, dump_kind="last_token",
                                                  dump_dtype=torch.float32, dump_flags=flags.cpu())
    assert_attention_close(out2, lse2, ref_out, ref_lse)
    assert_dump_close(d2, ref_dump, full, stride, dump_kind="last_token", dump_flags=flags.cpu())
    del graph


def test_append_page_tables_match_flat_list(cuda_device):
    dev = cuda_device
    lay = make_layout(batch=10, ctx=700, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=12,
                      seed=15, block_table="random")
    _, kv0 = fill_tensors(lay, device=dev, seed=16)
    T = int(lay.qo_indptr[-1])
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    k = torch.randn(T + 3, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(T + 3, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    indptr, lpl = t(lay.kv_indptr), t(last_page_lens(lay))
    app = t(lay.qo_indptr)
    flat = kv0.clone()
    append_kv(k, v, app, flat, t(lay.kv_indices), indptr, lpl, 16)
    tab = kv0.clone()
    append_kv(k, v, app, tab, None, indptr, lpl, 16, page_tables=_tables(lay, dev))
    torch.cuda.synchronize()
    assert torch.equal(flat, tab)
    assert not torch.equal(flat, kv0)
    ref = kv0.cpu()
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
    oracle_append.update_kv_padded(k.cpu(), v.cpu(), i32(lay.qo_indptr), ref, i32(lay.kv_indices),
                                   i32(lay.kv_indptr), i32(last_page_lens(lay)))
    assert torch.equal(tab.cpu(), ref)


def test_page_tables_require_a_page_source(cuda_device):
    w = HolisticAttentionWrapper(torch.empty(1, device=cuda_device))
    with pytest.raises(ValueError):
        w.plan_host(torch.tensor([0, 1]), torch.tensor([0, 1]), torch.tensor([5]), None, 32, 8, 128, 16)


def test_prefill_rows_page_tables_match_flat_list(cuda_device):
    """Prefill rows (the prefill phase's producers) read the block table the
    same way: a prefill chunk after a prefix, a short prefill row and a draft
    row in one batch."""
    from aspire_b200.workloads import MixedLayout
    dev = cuda_device
    rng = np.random.default_rng(21)
    q_lens, kv_lens, modes = [300, 40, 1], [800, 40, 500], [1, 1, 0]
    B = len(q_lens)
    pages = [(k + 15) // 16 for k in kv_lens]
    ppr = max(pages) + 3
    bt = rng.permutation(B * ppr).reshape(B, ppr).astype(np.int32)
    kv_indptr = np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)
    kv_indices = np.concatenate([bt[r, :pages[r]] for r in range(B)]).astype(np.int32)
    qo = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    lay = MixedLayout(num_qo_heads=32, num_kv_heads=8, modes=np.array(modes), q_lens=np.array(q_lens, np.int32),
                      kv_lens=np.array(kv_lens, np.int32), qo_indptr=qo, kv_indptr=kv_indptr, kv_indices=kv_indices,
                      block_table=bt, ctx_lens=np.array(kv_lens, np.int32), pages_per_row=ppr,
                      num_pages_total=B * ppr)
    q, kv = fill_tensors(lay, device=dev, seed=22)
    flat = HolisticAttentionWrapper(torch.empty(1, device=dev))
    _plan(flat, lay, dev, torch.from_numpy(lay.kv_indices).to(dev))
    assert flat.plan_info.num_items_prefill > 0 or not flat.plan_info.tc_enabled
    out_flat, lse_flat = flat.run(q, kv, return_lse=True)
    tab = HolisticAttentionWrapper(torch.empty(1, device=dev))
    tab.set_page_tables(*_tables(lay, dev))
    _plan(tab, lay, dev, None)
    out_tab, lse_tab = tab.run(q, kv, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(out_flat, out_tab)
    assert torch.equal(lse_flat, lse_tab)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out_tab, lse_tab, ref_out, ref_lse)
