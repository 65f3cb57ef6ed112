"""Pins the CPU oracle against fixtures produced by the reference's own code."""

import math

import numpy as np

import pytest
import torch

from oracle import kv_append as oracle_append
from oracle import unified_indices as oracle_indices
from oracle import page_selector as oracle_sel

CASES = ["cfg1", "pct", "budget"]


def _load(golden_dir, name):
    return torch.load(golden_dir / name, weights_only=False)


@pytest.mark.parametrize("case", CASES)
def test_selector_scores_match_reference(golden_dir, case):
    g = _load(golden_dir, f"page_selector_{case}.pt")
    p = g["params"]
    _, _, scores = oracle_sel.select(
        g["dump"], g["lse"], g["num_pages"], g["block_table"], g["qo_indptr"], batch=p["B"], n_heads=p["H"],
        kv_stride=p["kv_stride"], max_seq_len=p["max_seq_len"], pages_per_slot=p["pps"], k=p["k"], L=p["L"],
        draft_percent=p["draft_percent"], min_draft_pages=p["min_draft_pages"], return_scores=True)
    # Same torch CPU operations in the same order: bit-identical.
    assert torch.equal(scores, g["scores_raw"])


@pytest.mark.parametrize("case", CASES)
def test_selector_tables_match_reference(golden_dir, case):
    g = _load(golden_dir, f"page_selector_{case}.pt")
    p = g["params"]
    selected, valid = oracle_sel.select(
        g["dump"], g["lse"], g["num_pages"], g["block_table"], g["qo_indptr"], batch=p["B"], n_heads=p["H"],
        kv_stride=p["kv_stride"], max_seq_len=p["max_seq_len"], pages_per_slot=p["pps"], k=p["k"], L=p["L"],
        draft_percent=p["draft_percent"], min_draft_pages=p["min_draft_pages"])
    assert torch.equal(valid, g["valid"])
    assert torch.equal(selected, g["selected"])


LAST_CASES = ["cfg1", "f32"]


@pytest.mark.parametrize("case", LAST_CASES)
def test_last_token_selector_matches_reference(golden_dir, case):
    """The base PageSelector on a last-token dump (fp16 and fp32 buffers):
    the oracle's page scores are bit-identical and its tables equal."""
    g = _load(golden_dir, f"page_selector_last_{case}.pt")
    p = g["params"]
    selected, valid, scores = oracle_sel.select_last_token(
        g["dump"], g["lse"], g["num_pages"], g["block_table"], g["qo_indptr"], batch=p["B"], n_heads=p["H"],
        kv_stride=p["kv_stride"], max_seq_len=p["max_seq_len"], pages_per_slot=p["pps"], k=p["k"], L=p["L"],
        draft_percent=p["draft_percent"], min_draft_pages=p["min_draft_pages"], return_scores=True)
    assert torch.equal(scores, g["scores_raw"])
    assert torch.equal(valid, g["valid"])
    assert torch.equal(selected, g["selected"])
    if case == "f32":
        assert g["dump"].dtype == torch.float32


def _boundary_tied(scores_row, num_pages, L, valid):
    s = scores_row.clone()
    j = torch.arange(s.shape[0])
    s[(j >= max(num_pages - L, 0)) & (j < num_pages)] = float("inf")
    s[j >= num_pages] = float("-inf")
    srt = torch.sort(s, descending=True).values
    return valid < s.shape[0] and bool(srt[valid - 1] == srt[valid])


def test_golden_cases_have_untied_boundaries(golden_dir):
    """The fixtures exercise selection where the reference's result is tie-free."""
    for case in CASES + ["last_" + c for c in LAST_CASES]:
        g = _load(golden_dir, f"page_selector_{case}.pt")
        p = g["params"]
        for b in range(p["B"]):
            assert not _boundary_tied(g["scores_raw"][b], int(g["num_pages"][b]), p["L"], int(g["valid"][b])), (case, b)


def test_selector_finalize_with_ties(golden_dir):
    """On tied scores the reference's torch.topk picks an arbitrary subset of the tied
    pages; the oracle fixes the rule to lower page index first.  Both must agree on
    every page scored above the boundary and on how many tied pages are taken."""
    g = _load(golden_dir, "page_selector_ties.pt")
    p = g["params"]
    selected, valid = oracle_sel.finalize_scores(g["scores_raw"], g["num_pages"], g["block_table"], p["k"], p["L"])
    assert torch.equal(valid, g["valid"])
    for b in range(p["B"]):
        n, npg = int(valid[b]), int(g["num_pages"][b])
        s = g["scores_raw"][b].clone()
        j = torch.arange(s.shape[0])
        s[(j >= max(npg - p["L"], 0)) & (j < npg)] = float("inf")
        s[j >= npg] = float("-inf")
        bt = g["block_table"][b]
        page_of = {int(bt[i]): i for i in range(bt.shape[0])}
        mine = [page_of[int(x)] for x in selected[b, :n]]
        ref = [page_of[int(x)] for x in g["selected"][b, :n]]
        boundary = min(float(s[i]) for i in ref)
        assert min(float(s[i]) for i in mine) == boundary
        assert {i for i in mine if s[i] > boundary} == {i for i in ref if s[i] > boundary}
        tied = [i for i in range(s.shape[0]) if float(s[i]) == boundary]
        n_tied = sum(1 for i in ref if float(s[i]) == boundary)
        assert sorted(i for i in mine if float(s[i]) == boundary) == tied[:n_tied]


def test_valid_counts_match_engine_formula():
    num_pages = torch.arange(0, 3000, 7, dtype=torch.int32)
    v = oracle_sel.valid_counts(num_pages, k=73, L=8, draft_percent=7.0, min_draft_pages=32)
    # Independent restatement with Python floats rounded to fp32 per operation.
    import numpy as np
    prod = (num_pages.numpy().astype(np.float32) * np.float32(7.0)) / np.float32(100.0)
    target = np.ceil(prod).astype(np.int64)
    lo = np.minimum(num_pages.numpy(), 32)
    hi = np.minimum(num_pages.numpy(), 73)
    assert np.array_equal(v.numpy(), np.clip(target, lo, hi))


def test_append_matches_reference_triton_kernel(golden_dir):
    g = _load(golden_dir, "kv_append.pt")
    bidx, pos = oracle_append.positions(g["append_indptr"], g["page_indptr"], g["last_page_len"], g["k"].shape[0])
    valid_rows = pos >= 0
    assert torch.equal(pos.to(torch.int32), g["positions"])
    assert torch.equal(bidx[valid_rows].to(torch.int32), g["batch_indices"][valid_rows])
    cache = g["cache_before"].clone()
    oracle_append.update_kv_padded(g["k"], g["v"], g["append_indptr"], cache, g["page_indices"],
                                   g["page_indptr"], g["last_page_len"])
    assert torch.equal(cache, g["cache_after"])


def test_fp16_scalar_multiply_rounds_through_fp32():
    """The selector's fp16 * python-float multiply equals fp16(fp32(x) * fp32(c)) for every fp16 x."""
    x = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.float16)
    c = (1.0 / math.sqrt(128)) * math.log2(math.e)
    ref = x * c
    mine = (x.float() * torch.tensor(c, dtype=torch.float32)).half()
    same = (ref.view(torch.int16) == mine.view(torch.int16)) | (torch.isnan(ref) & torch.isnan(mine))
    assert bool(same.all())


FI_CASES = ["cfg1", "qwen8b_mixed", "qwen8b_full", "qwen8b_q9"]


@pytest.mark.parametrize("case", FI_CASES)
def test_attention_oracle_matches_flashinfer(golden_dir, case):
    """The fp32 attention oracle against FlashInfer's persistent attention (the
    reference's kernel family), run on the same seeded inputs by
    tests/golden/make_flashinfer_golden.py: pins the causal alignment, the
    base-2 LSE and the GQA mapping."""
    from aspire_b200.workloads import MixedLayout, fill_tensors
    from oracle import attention as oracle_attn

    g = _load(golden_dir, "flashinfer_attention.pt")["cases"][case]
    lay = MixedLayout(**g["layout"])
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse = oracle_attn.paged_attention(q.float(), kv, lay.qo_indptr, lay.kv_indptr, lay.kv_indices,
                                           lay.kv_lens)
    err = (out - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    assert (lse - g["lse"]).abs().max().item() <= 2e-3


@pytest.mark.parametrize("case", ["prefill_g4", "prefill_g1"])
def test_attention_oracle_matches_flashinfer_prefill(golden_dir, case):
    """The oracle against FlashInfer's BatchPrefillWithPagedKVCacheWrapper (the
    library the reference runs its prefill chunks through), on seeded prefill
    chunks (tests/golden/make_flashinfer_golden.py --prefill)."""
    from aspire_b200.workloads import MixedLayout, fill_tensors
    from oracle import attention as oracle_attn

    g = _load(golden_dir, "flashinfer_prefill.pt")["cases"][case]
    lay = MixedLayout(**g["layout"])
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse = oracle_attn.paged_attention(q.float(), kv, lay.qo_indptr, lay.kv_indptr, lay.kv_indices,
                                           lay.kv_lens)
    err = (out - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    assert (lse - g["lse"]).abs().max().item() <= 2e-3


def test_unified_indices_oracle_matches_reference_golden(golden_dir):
    """The restatement of build_unified_indices reproduces the reference's
    output (Triton interpreter) bit for bit, untouched entries included."""
    g = _load(golden_dir, "unified_indices.pt")
    indices = g["indices_before"].numpy().copy()
    indptr = g["indptr_before"].numpy().copy()
    oracle_indices.build_unified_indices(g["mode_flags"].numpy(), g["draft_indices"].numpy(),
                                         g["verify_indices"].numpy(), g["draft_num_pages"].numpy(),
                                         g["verify_num_pages"].numpy(), indices, indptr)
    np.testing.assert_array_equal(indptr, g["indptr"].numpy())
    np.testing.assert_array_equal(indices, g["indices"].numpy())


def test_prologue_oracle_matches_flashinfer_rope_golden(golden_dir):
    """The prologue restatement against the reference's math run on the GPU
    (its RMSNorm module and FlashInfer's interleaved RoPE): the norm and the
    permutation agree bit for bit; the rotation agrees to the error of
    FlashInfer's fast sincosf / powf intrinsics, which the float64 oracle
    does not share (largest at the 32k+ positions of the qwen3_8b case)."""
    import sys
    sys.path.insert(0, str(golden_dir))
    import make_rope_golden as mg
    from oracle import prologue as op

    g = torch.load(golden_dir / "rope_prologue.pt", weights_only=False)
    for name, c in g["cases"].items():
        p = c["params"]
        q, k, v, qw, kw, indptr, offsets = mg.case_inputs(p["seed"], p["T"], p["hq"], p["hkv"], p["rows"],
                                                          p["pos_base"])
        if p["norm"]:
            qn = op.permute_for_rope(op.rms_norm(q, qw, p["eps"]))
            kn = op.permute_for_rope(op.rms_norm(k, kw, p["eps"]))
        else:
            qn, kn = q, k
        assert torch.equal(qn, c["q_normed"]) and torch.equal(kn, c["k_normed"]), name
        for x, ref in ((qn, c["q_rot"]), (kn, c["k_rot"])):
            got = op.rope_interleaved(x, indptr.tolist(), offsets.tolist(), p["theta"], p["scale"], p["llama31"])
            d = (got.float() - ref.float()).abs()
            assert d.max().item() <= 0.04, (name, d.max().item())
            assert d.mean().item() <= 5e-4, (name, d.mean().item())
            # Tokens outside the rows are not rotated.
            tail = int(indptr[-1])
            assert torch.equal(got[tail:], x[tail:]) and torch.equal(ref[tail:], x[tail:])


def test_recent_rows_oracle_matches_reference_golden(golden_dir):
    """Recent-page seeding restated against the reference's own
    _build_recent_draft_rows (budget, draft_percent and floor variants)."""
    g = _load(golden_dir, "recent_rows.pt")
    for name, c in g.items():
        p = c["params"]
        rows, valid = oracle_sel.recent_rows(c["num_pages"], c["block_table"], p["k"], p["L"], p["draft_percent"],
                                             p["min_draft_pages"])
        assert torch.equal(valid, c["valid"]), name
        assert torch.equal(rows, c["rows"]), name


def test_draft_spill_oracle_matches_reference_golden(golden_dir):
    """Draft-page spill restated against the reference's own
    _handle_draft_page_spill / _handle_draft_page_spill_ids."""
    from oracle import draft_spill as oracle_spill

    g = _load(golden_dir, "draft_spill.pt")
    draft, counts = g["draft_before"].clone(), g["counts_before"].clone()
    oracle_spill.draft_page_spill(g["mode_flags"], g["dec_lens"], g["draft_cachelens"], draft, counts,
                                  g["block_table"])
    assert torch.equal(draft, g["draft_after"])
    assert torch.equal(counts, g["counts_after"])
    assert not torch.equal(counts, g["counts_before"])  # the fixture has rows that spill


def dump_positions_close(got, ref, lay):
    """fp16 dumps agree within one fp16 rounding step (plus a small absolute
    slack for the fp32 accumulation order) at every position the first/last
    transform defines: slot 0 of every row and slot 1 of rows with more than
    one query, keys [0, kv_len)."""
    for b in range(lay.batch):
        L = int(lay.kv_lens[b])
        for s in [0] + ([1] if int(lay.q_lens[b]) > 1 else []):
            a, e = got[b, :, s, :L].float(), ref[b, :, s, :L].float()
            tol = e.abs() * 2.0 ** -10 + 2.0 ** -14 + 2e-3
            assert bool(torch.isfinite(e).all()), (b, s)
            assert bool(((a - e).abs() <= tol).all()), (b, s, float((a - e).abs().max()))


@pytest.mark.parametrize("case", ["cfg1_full", "qwen8b_full"])
def test_dump_oracle_matches_flashinfer_variant(golden_dir, case):
    """The oracle's first/last dump against the reference's dump transform run
    inside FlashInfer (a custom FA2 attention variant, fixture from
    tests/golden/make_flashinfer_golden.py --dump): pins that the dump holds
    the raw q.k before scaling and masking, fp16-rounded, slot 0 for query 0
    and slot 1 for the last query."""
    from aspire_b200.workloads import MixedLayout, fill_tensors
    from oracle import attention as oracle_attn

    g = _load(golden_dir, "flashinfer_dump.pt")["cases"][case]
    lay = MixedLayout(**g["layout"])
    S = g["kv_stride"]
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    dump = torch.full((lay.batch * lay.num_qo_heads * 2 * S,), float("-inf"), dtype=torch.float16)
    out, lse = oracle_attn.paged_attention(q.float(), kv, lay.qo_indptr, lay.kv_indptr, lay.kv_indices,
                                           lay.kv_lens, dump=dump, dump_num_heads=lay.num_qo_heads,
                                           dump_kv_stride=S)
    dump_positions_close(dump.view(lay.batch, lay.num_qo_heads, 2, S), g["dump"], lay)
    err = (out - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    assert (lse - g["lse"]).abs().max().item() <= 2e-3


def last_dump_positions_close(got, ref, lay, flags):
    """Last-token dumps [B, H, stride] agree within one fp16 step at keys
    [0, kv_len) of every row whose flag is set (all rows without flags);
    rows flagged off hold only the -inf fill in both."""
    for b in range(lay.batch):
        if flags is not None and int(flags[b]) == 0:
            assert bool(torch.isinf(ref[b]).all()) and bool(torch.isinf(got[b]).all()), b
            continue
        L = int(lay.kv_lens[b])
        a, e = got[b, :, :L].float(), ref[b, :, :L].float()
        tol = e.abs() * 2.0 ** -10 + 2.0 ** -14 + 2e-3
        assert bool(torch.isfinite(e).all()), b
        assert bool(((a - e).abs() <= tol).all()), (b, float((a - e).abs().max()))


LAST_DUMP_CASES = ["f32_flags/cfg1_full", "f32_flags/qwen8b_full", "f16/cfg1_full", "f16/qwen8b_full"]


@pytest.mark.parametrize("case", LAST_DUMP_CASES)
def test_last_dump_oracle_matches_flashinfer_variant(golden_dir, case):
    """The oracle's last-token dump (with the mode-flag guard and an fp32
    buffer) against the reference's last_token transform run inside
    FlashInfer (fixture from tests/golden/make_flashinfer_golden.py
    --dump-last): the raw q.k of each row's last query, fp16-rounded, at
    dump[b, h, kv_idx]; rows whose flag is 0 untouched."""
    from aspire_b200.workloads import MixedLayout, fill_tensors
    from oracle import attention as oracle_attn

    g = _load(golden_dir, "flashinfer_dump_last.pt")["cases"][case]
    lay = MixedLayout(**g["layout"])
    S = g["kv_stride"]
    dtype = g["dump"].dtype
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    dump = torch.full((lay.batch * lay.num_qo_heads * S,), float("-inf"), dtype=dtype)
    out, lse = oracle_attn.paged_attention(q.float(), kv, lay.qo_indptr, lay.kv_indptr, lay.kv_indices,
                                           lay.kv_lens, dump=dump, dump_num_heads=lay.num_qo_heads,
                                           dump_kv_stride=S, dump_kind="last_token", dump_flags=g["flags"])
    assert dtype == (torch.float32 if case.startswith("f32") else torch.float16)
    last_dump_positions_close(dump.view(lay.batch, lay.num_qo_heads, S), g["dump"], lay, g["flags"])
    err = (out - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    assert (lse - g["lse"]).abs().max().item() <= 2e-3


@pytest.mark.parametrize("case", ["f16_first_last", "f32_last_token"])
def test_dump_state_oracle_matches_reference(golden_dir, case):
    """The restatement of LMBackendBase._clear_variant_slot_state reproduces
    the reference's own method (run on CPU by tests/golden/make_golden.py)."""
    from oracle import dump_state as oracle_dump

    g = _load(golden_dir, "dump_state.pt")[case]
    p = g["params"]
    dump, lse, flags = (g["before"][k].clone() for k in ("dump", "lse", "mode_flags"))
    oracle_dump.clear_variant_slot_state(dump, lse, g["before"]["qo_indptr"], flags, g["slot_ids"],
                                         num_heads=p["H"], dump_slots=p["slots"], kv_stride=p["kv_stride"])
    assert torch.equal(dump, g["after"]["dump"])
    assert torch.equal(lse, g["after"]["lse"])
    assert torch.equal(flags, g["after"]["mode_flags"])
