"""GPU parity of the draft-page spill insert (aspire_draft_page_spill)
against the reference's _handle_draft_page_spill on its spill mask (golden
fixture) and the CPU oracle on random batches, inside a CUDA graph too."""

import numpy as np
import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.kv_ops import draft_page_spill
from oracle import draft_spill as oracle_spill

pytestmark = pytest.mark.gpu


def test_spill_matches_reference_golden(cuda_device, golden_dir):
    g = torch.load(golden_dir / "draft_spill.pt", weights_only=False)
    dev = cuda_device
    draft, counts = g["draft_before"].to(dev), g["counts_before"].to(dev)
    draft_page_spill(g["mode_flags"].to(dev), g["dec_lens"].to(dev), g["draft_cachelens"].to(dev), draft, counts,
                     g["block_table"].to(dev))
    torch.cuda.synchronize()
    assert torch.equal(draft.cpu(), g["draft_after"])
    assert torch.equal(counts.cpu(), g["counts_after"])


def _random_batch(rng, B, width, pps):
    mode = (rng.random(B) < 0.7).astype(np.int32) ^ 1           # ~70 % draft rows (mode 0)
    dec = np.where(rng.random(B) < 0.1, 0, np.where(mode == 0, 1, rng.integers(2, 10, B))).astype(np.int32)
    dcl = (rng.integers(0, pps - 1, B) * 16 + rng.choice([1, 1, 2, 9, 16], B)).astype(np.int32)
    counts = rng.integers(0, width + 1, B).astype(np.int32)
    block = np.stack([rng.permutation(pps) + r * pps for r in range(B)]).astype(np.int32)
    draft = rng.integers(0, B * pps, (B, width)).astype(np.int32)
    # Some tables already end at the page of the newest token.
    for b in np.flatnonzero(rng.random(B) < 0.2):
        if counts[b] > 0:
            draft[b, counts[b] - 1] = block[b, max((int(dcl[b]) + 15) // 16 - 1, 0)]
    return mode, dec, dcl, counts, block, draft


@pytest.mark.parametrize("B,width", [(1, 4), (37, 8), (300, 130)])
def test_spill_matches_oracle_random(cuda_device, B, width):
    dev = cuda_device
    rng = np.random.default_rng(B)
    pps = 64
    mode, dec, dcl, counts, block, draft = _random_batch(rng, B, width, pps)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    # A wider allocation for the draft table, so its row stride differs from its width.
    draft_full = torch.full((B, width + 3), -7, dtype=torch.int32, device=dev)
    draft_full[:, :width] = t(draft)
    draft_dev, counts_dev = draft_full[:, :width], t(counts)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    draft_page_spill(t(mode), t(dec), t(dcl), draft_dev, counts_dev, t(block), status=status.view(torch.int32))
    torch.cuda.synchronize()
    ref_draft, ref_counts = torch.from_numpy(draft.copy()), torch.from_numpy(counts.copy())
    oracle_spill.draft_page_spill(torch.from_numpy(mode), torch.from_numpy(dec), torch.from_numpy(dcl), ref_draft,
                                  ref_counts, torch.from_numpy(block))
    assert torch.equal(draft_dev.cpu(), ref_draft) and torch.equal(counts_dev.cpu(), ref_counts)
    assert bool((draft_full[:, width:] == -7).all())
    assert int(status.item()) == 0


def test_spill_in_a_graph_and_bad_rows(cuda_device):
    """Captured once, replayed over changing lengths; a page index past the
    block table's columns is reported, not read."""
    dev = cuda_device
    B, width, pps = 16, 8, 10
    rng = np.random.default_rng(5)
    mode, dec, dcl, counts, block, draft = _random_batch(rng, B, width, pps)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    m, d, l_, c, bt, dr = t(mode), t(dec), t(dcl), t(counts), t(block), t(draft)
    draft_page_spill(m, d, l_, dr, c, bt)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        draft_page_spill(m, d, l_, dr, c, bt)
    for seed in (6, 7):
        mode, dec, dcl, counts, block, draft = _random_batch(np.random.default_rng(seed), B, width, pps)
        for dst, src in ((m, mode), (d, dec), (l_, dcl), (c, counts), (bt, block), (dr, draft)):
            dst.copy_(t(src))
        graph.replay()
        torch.cuda.synchronize()
        ref_draft, ref_counts = torch.from_numpy(draft.copy()), torch.from_numpy(counts.copy())
        oracle_spill.draft_page_spill(torch.from_numpy(mode), torch.from_numpy(dec), torch.from_numpy(dcl),
                                      ref_draft, ref_counts, torch.from_numpy(block))
        assert torch.equal(dr.cpu(), ref_draft) and torch.equal(c.cpu(), ref_counts)
    del graph
    # A draft row whose new page lies past the table's columns.
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    one = lambda v: torch.tensor([v], dtype=torch.int32, device=dev)  # noqa: E731
    tab = torch.zeros(1, 4, dtype=torch.int32, device=dev)
    cnt = one(1)
    draft_page_spill(one(0), one(1), one(16 * 5 + 1), tab, cnt, torch.zeros(1, 3, dtype=torch.int32, device=dev),
                     status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _capi.STATUS_BAD_ROW
    assert int(cnt.item()) == 1 and bool((tab == 0).all())
