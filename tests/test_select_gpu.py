"""GPU parity of the fused page scoring + radix top-k (aspire_select_pages)."""

import pytest
import torch

from aspire_b200.page_selector import PageSelector, PageSelectorFirstLastAvg
from oracle import page_selector as oracle_sel

pytestmark = pytest.mark.gpu

CASES = ["cfg1", "pct", "budget"]
SCORE_RTOL = 2e-5


def _selector(p, dev):
    return PageSelectorFirstLastAvg(max_batch_size=p["B"], pages_per_slot=p["pps"], subset_cache_size=p["k"],
                                    L=p["L"], n_heads=p["H"], page_size=16, max_seq_length=p["max_seq_len"],
                                    device=dev, bsz=p["B"], dec_len=9, head_dim=128, kv_stride=p["kv_stride"],
                                    draft_percent=p["draft_percent"], min_draft_pages=p["min_draft_pages"])


def _assert_scores_close(got, ref):
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got), fin)
    assert torch.equal(got[~fin], ref[~fin])
    err = (got[fin] - ref[fin]).abs() / ref[fin].abs().clamp(min=1e-6)
    assert err.max().item() <= SCORE_RTOL, err.max().item()


@pytest.mark.parametrize("case", CASES)
def test_fused_select_matches_reference(cuda_device, golden_dir, case):
    g = torch.load(golden_dir / f"page_selector_{case}.pt", weights_only=False)
    p = g["params"]
    dev = cuda_device
    sel = _selector(p, dev)
    scores = torch.empty(p["B"], p["pps"], dtype=torch.float32, device=dev)
    selected, valid = sel.select(g["dump"].to(dev), g["lse"].to(dev), g["num_pages"].to(dev),
                                 g["block_table"].to(dev), g["qo_indptr"].to(dev), scores_out=scores)
    torch.cuda.synchronize()
    _assert_scores_close(scores.cpu(), g["scores_raw"])
    # Bit-exact given identical fp32 scores: the oracle's top-k on the kernel's own scores.
    o_sel, o_valid = oracle_sel.finalize_scores(scores.cpu(), g["num_pages"], g["block_table"], p["k"], p["L"],
                                                p["draft_percent"], p["min_draft_pages"])
    assert torch.equal(valid.cpu(), o_valid)
    assert torch.equal(selected.cpu(), o_sel)
    # And the reference's own tables on these (tie-free) fixtures.
    assert torch.equal(valid.cpu(), g["valid"])
    assert torch.equal(selected.cpu(), g["selected"])


def test_topk_ties_lower_index_first(cuda_device, golden_dir):
    g = torch.load(golden_dir / "page_selector_ties.pt", weights_only=False)
    p = g["params"]
    sel = PageSelectorFirstLastAvg(max_batch_size=p["B"], pages_per_slot=p["pps"], subset_cache_size=p["k"],
                                   L=p["L"], n_heads=2, page_size=16, max_seq_length=p["pps"] * 16,
                                   device=cuda_device, bsz=p["B"], dec_len=1)
    got_sel, got_valid = sel.finalize_scores(g["scores_raw"].to(cuda_device), g["num_pages"].to(cuda_device),
                                             g["block_table"].to(cuda_device))
    o_sel, o_valid = oracle_sel.finalize_scores(g["scores_raw"], g["num_pages"], g["block_table"], p["k"], p["L"])
    assert torch.equal(got_valid.cpu(), o_valid)
    assert torch.equal(got_sel.cpu(), o_sel)


@pytest.mark.parametrize("pps,k,L", [(64, 8, 2), (2080, 128, 8), (5136, 256, 8), (300, 300, 0)])
def test_topk_random_scores_with_ties(cuda_device, pps, k, L):
    gen = torch.Generator().manual_seed(pps + k)
    B = 7
    scores = torch.randint(0, 50, (B, pps), generator=gen).float() * 0.25
    scores[0] = 1.0  # all tied
    scores[1, ::3] = float("inf")
    num_pages = torch.randint(1, pps + 1, (B,), generator=gen).to(torch.int32)
    num_pages[2] = pps
    num_pages[3] = 1
    block_table = torch.stack([torch.randperm(10 * pps, generator=gen)[:pps] for _ in range(B)]).to(torch.int32)
    for dp, mdp in ((None, None), (7.0, 32), (None, 5), (None, 2 * k)):
        sel = PageSelectorFirstLastAvg(max_batch_size=B, pages_per_slot=pps, subset_cache_size=k, L=L, n_heads=2,
                                       page_size=16, max_seq_length=pps * 16, device=cuda_device, bsz=B, dec_len=1,
                                       draft_percent=dp, min_draft_pages=mdp)
        got_sel, got_valid = sel.finalize_scores(scores.to(cuda_device), num_pages.to(cuda_device),
                                                 block_table.to(cuda_device))
        o_sel, o_valid = oracle_sel.finalize_scores(scores, num_pages, block_table, k, L, dp, mdp)
        assert torch.equal(got_valid.cpu(), o_valid)
        assert torch.equal(got_sel.cpu(), o_sel)


def test_select_into_writes_table_in_place(cuda_device, golden_dir):
    g = torch.load(golden_dir / "page_selector_cfg1.pt", weights_only=False)
    p = g["params"]
    dev = cuda_device
    sel = _selector(p, dev)
    width = p["k"] + 5
    table = torch.full((p["B"] + 2, width), 777, dtype=torch.int32, device=dev)
    counts = torch.full((p["B"] + 2,), -1, dtype=torch.int32, device=dev)
    sel.select_into(table, counts, g["dump"].to(dev), g["lse"].to(dev), g["num_pages"].to(dev),
                    g["block_table"].to(dev), g["qo_indptr"].to(dev))
    ref_table = torch.full((p["B"] + 2, width), 777, dtype=torch.int32)
    ref_counts = torch.full((p["B"] + 2,), -1, dtype=torch.int32)
    oracle_sel.store_draft_rows(ref_table, ref_counts, g["selected"], g["valid"])
    torch.cuda.synchronize()
    assert torch.equal(table.cpu(), ref_table)
    assert torch.equal(counts.cpu(), ref_counts)


def test_select_subset_rows(cuda_device, golden_dir):
    g = torch.load(golden_dir / "page_selector_cfg1.pt", weights_only=False)
    p = g["params"]
    dev = cuda_device
    sel = _selector(p, dev)
    ids = torch.tensor([2, 0], device=dev)
    got_sel, got_valid = sel.select_subset(ids, g["dump"].to(dev), g["lse"].to(dev), g["num_pages"].to(dev),
                                           g["block_table"].to(dev), g["qo_indptr"].to(dev))
    assert torch.equal(got_sel.cpu(), g["selected"][[2, 0]])
    assert torch.equal(got_valid.cpu(), g["valid"][[2, 0]])


@pytest.mark.parametrize("case", ["budget", "pct", "floor"])
def test_seed_recent_matches_reference_golden(cuda_device, golden_dir, case):
    """Recent-page seeding through the selection kernel (page-index scores,
    page-order rows) against the reference's _build_recent_draft_rows."""
    c = torch.load(golden_dir / "recent_rows.pt", weights_only=False)[case]
    p = c["params"]
    sel = PageSelectorFirstLastAvg(max_batch_size=p["B"], pages_per_slot=p["pps"], subset_cache_size=p["k"],
                                   L=p["L"], n_heads=2, page_size=16, max_seq_length=p["pps"] * 16,
                                   device=cuda_device, bsz=p["B"], dec_len=1, draft_percent=p["draft_percent"],
                                   min_draft_pages=p["min_draft_pages"])
    rows, valid = sel.seed_recent(c["num_pages"].to(cuda_device), c["block_table"].to(cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(valid.cpu(), c["valid"])
    assert torch.equal(rows.cpu(), c["rows"])


LAST_CASES = ["cfg1", "f32"]


def _last_selector(p, dev):
    return PageSelector(max_batch_size=p["B"], pages_per_slot=p["pps"], subset_cache_size=p["k"], L=p["L"],
                        n_heads=p["H"], page_size=16, max_seq_length=p["max_seq_len"], device=dev, bsz=p["B"],
                        dec_len=9, head_dim=128, kv_stride=p["kv_stride"], draft_percent=p["draft_percent"],
                        min_draft_pages=p["min_draft_pages"])


@pytest.mark.parametrize("case", LAST_CASES)
def test_last_token_select_matches_reference(cuda_device, golden_dir, case):
    """The base PageSelector (last-token dump, fp16 and fp32 buffers) against
    the reference's own PageSelector.select on the same inputs: page scores
    within SCORE_RTOL, tables equal, and the oracle's top-k of the kernel's
    scores bit-exact; select_subset picks the same rows."""
    g = torch.load(golden_dir / f"page_selector_last_{case}.pt", weights_only=False)
    p = g["params"]
    dev = cuda_device
    sel = _last_selector(p, dev)
    scores = torch.empty(p["B"], p["pps"], dtype=torch.float32, device=dev)
    selected, valid = sel.select(g["dump"].to(dev), g["lse"].to(dev), g["num_pages"].to(dev),
                                 g["block_table"].to(dev), g["qo_indptr"].to(dev), scores_out=scores)
    torch.cuda.synchronize()
    _assert_scores_close(scores.cpu(), g["scores_raw"])
    o_sel, o_valid = oracle_sel.finalize_scores(scores.cpu(), g["num_pages"], g["block_table"], p["k"], p["L"],
                                                p["draft_percent"], p["min_draft_pages"])
    assert torch.equal(valid.cpu(), o_valid) and torch.equal(selected.cpu(), o_sel)
    assert torch.equal(valid.cpu(), g["valid"]) and torch.equal(selected.cpu(), g["selected"])
    ids = torch.tensor([p["B"] - 1, 0], dtype=torch.long)
    s_sel, s_valid = sel.select_subset(ids.to(dev), g["dump"].to(dev), g["lse"].to(dev), g["num_pages"].to(dev),
                                       g["block_table"].to(dev), g["qo_indptr"].to(dev))
    assert torch.equal(s_sel.cpu(), g["selected"][ids]) and torch.equal(s_valid.cpu(), g["valid"][ids])


def test_compact_first_last_entry_points(cuda_device, golden_dir):
    """select_from_compact_first_last / select_layers_from_compact_first_last
    (explicit [B, H, 2, max_seq_len] logit views and first/last LSE) give the
    tables of select() on the same dump."""
    g = torch.load(golden_dir / "page_selector_pct.pt", weights_only=False)
    p = g["params"]
    dev = cuda_device
    sel = _selector(p, dev)
    dump = g["dump"].to(dev)
    lse = g["lse"].to(dev)
    qo = g["qo_indptr"].long()
    max_q = lse.shape[0] - 1
    first = lse[qo[:p["B"]].clamp(0, max_q).to(dev)]
    last = lse[(qo[1:p["B"] + 1] - 1).clamp(0, max_q).to(dev)]
    logits = dump.view(p["B"], p["H"], 2, p["kv_stride"])[..., :p["max_seq_len"]]
    a_sel, a_valid = sel.select_from_compact_first_last(logits, first, last, g["num_pages"].to(dev),
                                                        g["block_table"].to(dev))
    assert torch.equal(a_sel.cpu(), g["selected"]) and torch.equal(a_valid.cpu(), g["valid"])
    layers = torch.stack([dump.view(p["B"], p["H"], 2, p["kv_stride"])] * 2)
    l_sel, l_valid = sel.select_layers_from_compact_first_last(layers, torch.stack([first] * 2),
                                                               torch.stack([last] * 2), g["num_pages"].to(dev),
                                                               g["block_table"].to(dev))
    assert l_sel.shape == (2, p["B"], p["k"])
    assert torch.equal(l_sel[0].cpu(), g["selected"]) and torch.equal(l_sel[1].cpu(), g["selected"])
    assert torch.equal(l_valid.cpu(), g["valid"])
