"""Parity at the benchmark's own workload, at every tensor-parallel head share.

bench.py times one decode step of the hot path on the reference's config-3
shapes (Qwen3-8B heads, B=64, 32k context, half draft rows with 128 selected
pages, half verify rows with q_len U{3..9}), with the kernels reading pages
straight from the draft / block tables.  This test builds that same HotPath
(bench.build_workload + bench.HotPath, the bench's CFG) for the head share of
rank 0 at TP 1, 2, 4 and 8 ((32, 8), (16, 4), (8, 2) and (4, 1) query / KV
heads, split as aspire/tp.py:35-51 splits them), with the engine's arange
block tables and with scattered (random) ones, replays the captured step
graph once and checks, for a sample of 8 rows (4 draft, 4 verify), against
the fp32 oracle:

* layer 0 (a mixed layer: sparse draft rows, causal verify rows);
* the refresh layer (every row over its full context): output, LSE and the
  first/last logit dump;
* the page selection the step wrote into the draft table: scores within
  2e-5 relative of the oracle's (computed from the kernel's dump and LSE),
  and the whole table bit-exact against the oracle's top-k of the kernel's
  own scores.

Each layer's new K/V tokens land in the same cache slots, so the cache as a
layer saw it is the final cache with that layer's tokens written back by the
oracle's append.  At TP 8 the mixed plan's split-KV chunks are short enough
(<= 4096 tokens) for the kernel's one-column-width mode, which is asserted.
"""

import numpy as np
import pytest
import torch

import bench
from aspire_b200.workloads import MixedLayout, last_page_lens
from gpu_helpers import assert_attention_close, assert_dump_close
from oracle import attention as oracle_attn
from oracle import kv_append as oracle_append
from oracle import page_selector as oracle_sel

pytestmark = pytest.mark.gpu

SCORE_RTOL = 2e-5
CASES = [(1, "arange"), (1, "random"), (2, "arange"), (4, "arange"), (8, "arange"), (8, "random")]


def _sample_rows(lay, n_each=4):
    draft = np.flatnonzero(lay.modes == 0)
    verify = np.flatnonzero(lay.modes == 1)
    pick = lambda rows: rows[np.linspace(0, len(rows) - 1, n_each).round().astype(int)]  # noqa: E731
    return sorted(set(pick(draft).tolist()) | set(pick(verify).tolist()))


def _sub_layout(lay, full, rows):
    """The sampled rows as a layout over a small cache holding only their pages
    (every page of the row's full context), with the page ids remapped."""
    pages = np.concatenate([full.kv_indices[full.kv_indptr[r]:full.kv_indptr[r + 1]] for r in rows])
    uniq = np.unique(pages)
    remap = {int(p): i for i, p in enumerate(uniq)}

    def sub(src):
        idx = [np.array([remap[int(p)] for p in src.kv_indices[src.kv_indptr[r]:src.kv_indptr[r + 1]]], np.int32)
               for r in rows]
        q_lens = src.q_lens[rows].astype(np.int32)
        kv_indptr = np.concatenate([[0], np.cumsum([len(i) for i in idx])]).astype(np.int32)
        return MixedLayout(num_qo_heads=src.num_qo_heads, num_kv_heads=src.num_kv_heads, modes=src.modes[rows],
                           q_lens=q_lens, kv_lens=src.kv_lens[rows].astype(np.int32),
                           qo_indptr=np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32),
                           kv_indptr=kv_indptr, kv_indices=np.concatenate(idx).astype(np.int32),
                           block_table=src.block_table[rows], ctx_lens=src.ctx_lens[rows],
                           pages_per_row=src.pages_per_row, num_pages_total=len(uniq))
    return sub(lay), sub(full), torch.from_numpy(uniq.astype(np.int64))


def _token_rows(lay, rows):
    return np.concatenate([np.arange(lay.qo_indptr[r], lay.qo_indptr[r + 1]) for r in rows])


def _cache_for_layer(kv_sub, src_sub, hp, layer, tok):
    """The sampled rows' cache as `layer` saw it: its new tokens written back."""
    kv = kv_sub.clone()
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
    oracle_append.update_kv_padded(hp.k_new[layer][tok].cpu(), hp.v_new[layer][tok].cpu(), i32(src_sub.qo_indptr),
                                   kv, i32(src_sub.kv_indices), i32(src_sub.kv_indptr),
                                   i32(last_page_lens(src_sub)))
    return kv


@pytest.mark.parametrize("world,table", CASES)
def test_bench_step_matches_oracle(cuda_device, world, table):
    dev = cuda_device
    saved = dict(bench.CFG)
    bench.CFG["block_table"] = table
    try:
        lay, full, lpl_m, lpl_f = bench.build_workload(dev, 0, world)
        hp = bench.HotPath(dev, lay, full, lpl_m, lpl_f)
        hp.plan()
        hp.capture()
        hp.graph.replay()
        torch.cuda.synchronize()
        if world == 8:
            # 128 verify groups on 148 SMs: each cut in one 8192-token piece per SM
            assert hp.mixed.plan_info.chunk_tokens == 8192, hp.mixed.plan_info.chunk_tokens
        assert hp.mixed.device_status() == 0 and hp.refresh.device_status() == 0

        rows = _sample_rows(lay)
        lay_s, full_s, pages = _sub_layout(lay, full, rows)
        kv_s = hp.kv[pages.to(dev)].cpu()
        tok = _token_rows(lay, rows)
        hq = lay.num_qo_heads

        # Layer 0: mixed attention.
        kv0 = _cache_for_layer(kv_s, lay_s, hp, 0, tok)
        q0 = hp.q[0][tok].float().cpu()
        ref_out, _ = oracle_attn.paged_attention(q0, kv0, lay_s.qo_indptr, lay_s.kv_indptr, lay_s.kv_indices,
                                                 lay_s.kv_lens, causal=True)
        err = (hp.out[0][tok].float().cpu() - ref_out).abs()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (world, table, err.max().item())

        # Refresh layer: full attention, LSE and the first/last dump.
        L = bench.CFG["refresh_layer"]
        kvr = _cache_for_layer(kv_s, full_s, hp, L, tok)
        stride = hp.kv_stride
        ref_dump = torch.full((len(rows) * hq * 2 * stride,), float("-inf"), dtype=torch.float16)
        ref_out, ref_lse = oracle_attn.paged_attention(hp.q[L][tok].float().cpu(), kvr, full_s.qo_indptr,
                                                       full_s.kv_indptr, full_s.kv_indices, full_s.kv_lens,
                                                       causal=True, dump=ref_dump, dump_num_heads=hq,
                                                       dump_kv_stride=stride)
        assert_attention_close(hp.out[L][tok], hp.lse[tok], ref_out, ref_lse)
        dump_rows = hp.dump.view(lay.batch, hq, 2, stride)[torch.tensor(rows, device=dev)].cpu().reshape(-1)
        assert_dump_close(dump_rows, ref_dump, full_s, stride)

        # Selection: the kernel's scores against the oracle's on the same dump
        # and LSE, and the step's table against the oracle's top-k of those scores.
        scores = torch.empty(lay.batch, lay.pages_per_row, dtype=torch.float32, device=dev)
        table_chk = torch.zeros_like(hp.draft_table)
        counts_chk = torch.zeros_like(hp.draft_counts)
        hp.selector.select_into(table_chk, counts_chk, hp.dump, hp.lse, hp.num_pages, hp.block_table,
                                hp.qo_indptr, scores_out=scores)
        torch.cuda.synchronize()
        assert torch.equal(table_chk, hp.draft_table) and torch.equal(counts_chk, hp.draft_counts)
        lse_cpu = hp.lse.cpu()
        qo = torch.from_numpy(lay.qo_indptr.astype(np.int64))
        r_t = torch.tensor(rows)
        ref_scores = oracle_sel.first_last_scores(dump_rows.view(len(rows), hq, 2, stride), lse_cpu[qo[r_t]],
                                                  lse_cpu[qo[r_t + 1] - 1], lay.pages_per_row, 16)
        got = scores.cpu()[r_t]
        fin = torch.isfinite(ref_scores)
        assert torch.equal(torch.isfinite(got), fin)
        rel = (got[fin] - ref_scores[fin]).abs() / ref_scores[fin].abs().clamp(min=1e-6)
        assert rel.max().item() <= SCORE_RTOL, rel.max().item()
        sel, valid = oracle_sel.finalize_scores(scores.cpu(), hp.num_pages.cpu(), hp.block_table.cpu(), hp.k_sel,
                                                bench.CFG["L"], None, hp.k_sel)
        assert torch.equal(hp.draft_table.cpu(), sel) and torch.equal(hp.draft_counts.cpu(), valid)
    finally:
        bench.CFG.clear()
        bench.CFG.update(saved)
