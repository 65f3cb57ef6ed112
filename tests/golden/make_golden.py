"""Generates the golden fixtures of tests/golden/ from the reference's own code.

Run where the reference tree is checked out, with $ASPIRE_REFERENCE naming
its root:

    ASPIRE_REFERENCE=<path to the ASPIRE checkout> python tests/golden/make_golden.py [group ...]

* page_selector_*.pt : inputs and outputs of the reference's
  aspire.backends.page_selector.PageSelectorFirstLastAvg.select (imported
  unchanged from the reference tree, run on CPU), including its page-score
  buffer before the +/-inf forcing; tie cases run its _finalize_scores.
  page_selector_last_*.pt: the same for the base PageSelector.select on a
  last-token dump (fp16 and fp32 buffers).
* recent_rows.pt : the reference's LMBackendBase._build_recent_draft_rows
  (recent-page seeding of the draft table) on CPU.
* dump_state.pt : the reference's LMBackendBase._clear_variant_slot_state
  (dump-state reset of cleared slots) on CPU.
* unified_indices.pt : the reference's build_unified_indices
  (aspire/models/sparse_draft_runner.py, with its Triton _copy_indices_kernel)
  under the Triton CPU interpreter.
* kv_append.pt : the reference's Triton kernels
  (aspire.attention.kv_ops._append_paged_kv_cache_padded_kernel and
  FlashInfer's get_batch_indices_positions_kernel) executed by Triton's CPU
  interpreter (TRITON_INTERPRET=1) on a padded mixed batch.

The fixtures are small (about 4 MB together) and committed; tests never
read the reference tree.
"""

from __future__ import annotations

import math
import os
import subprocess
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("ASPIRE_REFERENCE", ""))


def _ref_selector_cls():
    sys.path.insert(0, str(REF))
    from aspire.backends.page_selector import PageSelectorFirstLastAvg  # noqa: E402

    return PageSelectorFirstLastAvg


def _make_dump(gen, B, H, kv_stride, lens, stale_slot1_rows):
    """fp16 dump [B*H*2*kv_stride] with -inf fill beyond each row's length."""
    d = torch.full((B, H, 2, kv_stride), float("-inf"), dtype=torch.float16)
    for b in range(B):
        L = int(lens[b])
        vals = (torch.randn(H, 2, L, generator=gen) * 11.3).to(torch.float16)
        d[b, :, :, :L] = vals
        if b in stale_slot1_rows:
            # slot 1 holds older logits over a shorter prefix (q_len == 1 rows)
            d[b, :, 1, L // 2:] = float("-inf")
    return d.reshape(-1)


def selector_case(name, *, B, H, max_seq_len, kv_stride, top_k_pages, L, draft_percent, seed,
                  q_lens, lens, stale_rows=(), lse_neg_inf_rows=()):
    cls = _ref_selector_cls()
    gen = torch.Generator().manual_seed(seed)
    page = 16
    pps = (max_seq_len + page - 1) // page
    if draft_percent is not None:
        k = max(top_k_pages, math.ceil(pps * draft_percent / 100))
    else:
        k = top_k_pages
    sel = cls(max_batch_size=B, pages_per_slot=pps, subset_cache_size=k, L=L, n_heads=H, page_size=page,
              max_seq_length=max_seq_len, device="cpu", bsz=B, dec_len=9, head_dim=128,
              kv_stride=kv_stride, draft_percent=draft_percent, min_draft_pages=top_k_pages)
    dump = _make_dump(gen, B, H, kv_stride, lens, set(stale_rows))
    qo = torch.zeros(B + 1, dtype=torch.int32)
    qo[1:] = torch.cumsum(torch.tensor(q_lens, dtype=torch.int32), 0)
    T = int(qo[-1]) + 3
    # LSE of a random logit row is around log2(len) + a few; keep it realistic.
    lse = (torch.randn(T, H, generator=gen) * 2.0 + 12.0).float()
    dview = dump.view(B, H, 2, kv_stride)
    for b in lse_neg_inf_rows:
        # A first query that saw no keys: -inf LSE and -inf logits, so the
        # normalised logit is NaN and the selector maps it to -inf.
        lse[int(qo[b])] = float("-inf")
        dview[b, :, 0, :] = float("-inf")
    num_pages = torch.tensor([(int(x) + page - 1) // page for x in lens], dtype=torch.int32)
    block_table = torch.stack([b * pps + torch.randperm(pps, generator=gen) for b in range(B)]).to(torch.int32)

    captured = {}
    orig = sel._finalize_scores

    def capture(scores, num_pages_, block_table_):
        captured["scores_raw"] = scores.clone()
        return orig(scores, num_pages_, block_table_)

    sel._finalize_scores = capture
    selected, valid = sel.select(dump, lse, num_pages, block_table, qo)
    out = {
        "params": dict(B=B, H=H, max_seq_len=max_seq_len, kv_stride=kv_stride, pps=pps, k=k, L=L,
                       draft_percent=draft_percent, min_draft_pages=top_k_pages, page_size=page),
        "dump": dump, "lse": lse, "num_pages": num_pages, "block_table": block_table, "qo_indptr": qo,
        "scores_raw": captured["scores_raw"], "selected": selected.clone(), "valid": valid.clone(),
    }
    torch.save(out, HERE / f"page_selector_{name}.pt")
    print(f"page_selector_{name}: k={k} valid={valid.tolist()}")


def last_token_case(name, *, B, H, max_seq_len, kv_stride, top_k_pages, L, draft_percent, seed, q_lens, lens,
                    dump_dtype=torch.float16, lse_neg_inf_rows=()):
    """The base PageSelector (last-token dump [B, H, kv_stride])."""
    sys.path.insert(0, str(REF))
    from aspire.backends.page_selector import PageSelector  # noqa: E402

    gen = torch.Generator().manual_seed(seed)
    page = 16
    pps = (max_seq_len + page - 1) // page
    k = max(top_k_pages, math.ceil(pps * draft_percent / 100)) if draft_percent is not None else top_k_pages
    sel = PageSelector(max_batch_size=B, pages_per_slot=pps, subset_cache_size=k, L=L, n_heads=H, page_size=page,
                       max_seq_length=max_seq_len, device="cpu", bsz=B, dec_len=9, head_dim=128,
                       kv_stride=kv_stride, draft_percent=draft_percent, min_draft_pages=top_k_pages)
    d = torch.full((B, H, kv_stride), float("-inf"), dtype=dump_dtype)
    for b in range(B):
        n = int(lens[b])
        # fp16-representable logits in either buffer, as the dump kernels write them
        d[b, :, :n] = (torch.randn(H, n, generator=gen) * 11.3).to(torch.float16).to(dump_dtype)
    qo = torch.zeros(B + 1, dtype=torch.int32)
    qo[1:] = torch.cumsum(torch.tensor(q_lens, dtype=torch.int32), 0)
    T = int(qo[-1]) + 3
    lse = (torch.randn(T, H, generator=gen) * 2.0 + 12.0).float()
    for b in lse_neg_inf_rows:
        # A last query that saw no keys: -inf LSE and -inf logits -> NaN -> -inf.
        lse[int(qo[b + 1]) - 1] = float("-inf")
        d[b] = float("-inf")
    dump = d.reshape(-1)
    num_pages = torch.tensor([(int(x) + page - 1) // page for x in lens], dtype=torch.int32)
    block_table = torch.stack([b * pps + torch.randperm(pps, generator=gen) for b in range(B)]).to(torch.int32)
    captured = {}
    orig = sel._finalize_scores

    def capture(scores, num_pages_, block_table_):
        captured["scores_raw"] = scores.clone()
        return orig(scores, num_pages_, block_table_)

    sel._finalize_scores = capture
    selected, valid = sel.select(dump, lse, num_pages, block_table, qo)
    out = {
        "params": dict(B=B, H=H, max_seq_len=max_seq_len, kv_stride=kv_stride, pps=pps, k=k, L=L,
                       draft_percent=draft_percent, min_draft_pages=top_k_pages, page_size=page),
        "dump": dump, "lse": lse, "num_pages": num_pages, "block_table": block_table, "qo_indptr": qo,
        "scores_raw": captured["scores_raw"], "selected": selected.clone(), "valid": valid.clone(),
    }
    torch.save(out, HERE / f"page_selector_last_{name}.pt")
    print(f"page_selector_last_{name}: k={k} valid={valid.tolist()}")


def tie_case():
    """_finalize_scores on scores with exact ties (finite and +inf)."""
    cls = _ref_selector_cls()
    B, pps, k, L = 4, 48, 12, 3
    sel = cls(max_batch_size=B, pages_per_slot=pps, subset_cache_size=k, L=L, n_heads=2, page_size=16,
              max_seq_length=pps * 16, device="cpu", bsz=B, dec_len=1, head_dim=128,
              draft_percent=None, min_draft_pages=None)
    gen = torch.Generator().manual_seed(7)
    scores = torch.randint(0, 6, (B, pps), generator=gen).float()  # many exact ties
    scores[1, 10:20] = 3.0
    num_pages = torch.tensor([48, 30, 5, 13], dtype=torch.int32)
    block_table = torch.stack([torch.randperm(1000, generator=gen)[:pps] for _ in range(B)]).to(torch.int32)
    raw = scores.clone()
    selected, valid = sel._finalize_scores(scores, num_pages, block_table)
    torch.save({"params": dict(B=B, pps=pps, k=k, L=L), "scores_raw": raw, "num_pages": num_pages,
                "block_table": block_table, "selected": selected.clone(), "valid": valid.clone()},
               HERE / "page_selector_ties.pt")
    print("page_selector_ties: valid", valid.tolist())


_APPEND_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from aspire.attention import kv_ops
import flashinfer.triton.page as fpage
torch.manual_seed(3)
H, D, page = 2, 128, 16
# rows: draft (1 token through its sparse table), verify (5 tokens), verify
# starting a fresh page, an empty row, then the bucket padding row.
append_indptr = torch.tensor([0, 1, 6, 9, 9, 12], dtype=torch.int32)
T = 12
page_indptr = torch.tensor([0, 3, 6, 8, 8, 8], dtype=torch.int32)
page_indices = torch.tensor([7, 2, 11, 0, 4, 9, 13, 5], dtype=torch.int32)
last = torch.tensor([9, 12, 3, 0, 0], dtype=torch.int32)
P = 16
k = torch.randn(T, H, D)
v = torch.randn(T, H, D)
cache = torch.randn(P, 2, page, H, D)
cache0 = cache.clone()
seq_lens = torch.clamp(page_indptr[1:] - page_indptr[:-1] - 1, min=0) * page + last
bi = torch.zeros(T, dtype=torch.int32)
pos = torch.full((T,), -1, dtype=torch.int32)
fpage.get_batch_indices_positions_kernel[(seq_lens.shape[0],)](append_indptr, seq_lens, bi, pos, num_stages=2)
kv_ops._append_paged_kv_cache_padded_kernel[(T, H)](
    k, v, bi, pos, cache, page_indices, page_indptr, last,
    k.stride(0), k.stride(1), v.stride(0), v.stride(1),
    cache.stride(0), cache.stride(1), cache.stride(2), cache.stride(3), HEAD_DIM=D, PAGE_SIZE=page)
torch.save({"k": k, "v": v, "append_indptr": append_indptr, "page_indices": page_indices,
            "page_indptr": page_indptr, "last_page_len": last, "cache_before": cache0,
            "cache_after": cache, "batch_indices": bi, "positions": pos}, sys.argv[2])
print("kv_append positions", pos.tolist())
"""


def append_case():
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, "-c", _APPEND_SCRIPT, str(REF), str(HERE / "kv_append.pt")], check=True,
                   env=env)


_INDICES_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from aspire.models.sparse_draft_runner import build_unified_indices
g = torch.Generator().manual_seed(11)
# draft rows, verify rows, an empty row of each kind, and a verify row longer
# than one 128-wide Triton block; the output buffers are oversized and
# pre-filled so untouched entries are visible.
mode = torch.tensor([0, 1, 0, 1, 1, 0, 1, 0], dtype=torch.int32)
dn = torch.tensor([5, 0, 40, 3, 0, 0, 131, 17], dtype=torch.int32)
vn = torch.tensor([9, 300, 2, 3, 0, 12, 131, 4], dtype=torch.int32)
B = mode.shape[0]
draft = torch.randint(0, 5000, (B, 40), generator=g, dtype=torch.int32)
verify = torch.randint(0, 5000, (B, 300), generator=g, dtype=torch.int32)
indices = torch.full((700,), -7, dtype=torch.int32)
indptr = torch.full((B + 2,), -9, dtype=torch.int32)
build_unified_indices(mode, draft, verify, dn, vn, indices, indptr)
torch.save({"mode_flags": mode, "draft_indices": draft, "verify_indices": verify, "draft_num_pages": dn,
            "verify_num_pages": vn, "indices_before": torch.full((700,), -7, dtype=torch.int32),
            "indptr_before": torch.full((B + 2,), -9, dtype=torch.int32), "indices": indices,
            "indptr": indptr}, sys.argv[2])
print("unified_indices indptr", indptr.tolist())
"""


def indices_case():
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, "-c", _INDICES_SCRIPT, str(REF), str(HERE / "unified_indices.pt")],
                   check=True, env=env)


def recent_case():
    """Recent-page seeding: the reference's LMBackendBase._build_recent_draft_rows
    (imported unchanged) on a scattered block table; the bound instance carries
    the attributes the method reads, with _get_num_pages the documented
    ceil(seq_len / page_size) (aspire/models/mixed_runner.py:114-120)."""
    import types

    sys.path.insert(0, str(REF))
    from aspire.backends.base import LMBackendBase  # noqa: E402

    sel_cls = _ref_selector_cls()
    out = {}
    for name, (k, L, pct, mdp) in {"budget": (16, 4, None, None), "pct": (32, 8, 7.0, None),
                                    "floor": (32, 8, None, 12)}.items():
        B, pps, page = 9, 64, 16
        g = torch.Generator().manual_seed(len(name) * 7)
        cachelens = torch.tensor([0, 1, 16, 17, 100, 400, 1000, 1024, 555], dtype=torch.int64)
        # The engine's tables are wider than the longest row (the method gathers
        # k columns from the first recent page), so give the table that headroom.
        width = pps + k
        block_table = torch.stack([torch.randperm(width, generator=g) + r * width for r in range(B)]).to(torch.int32)
        selector = sel_cls(max_batch_size=B, pages_per_slot=pps, subset_cache_size=k, L=L, n_heads=2, page_size=page,
                           max_seq_length=pps * page, device="cpu", bsz=B, dec_len=1, draft_percent=pct,
                           min_draft_pages=mdp)
        fake = types.SimpleNamespace(device=torch.device("cpu"), cachelens=cachelens, page_selector=selector,
                                     max_draft_pages=k, target_block_table=block_table,
                                     _get_num_pages=lambda s: (s + page - 1) // page)
        slots = torch.arange(B)
        rows, valid = LMBackendBase._build_recent_draft_rows(fake, slots)
        out[name] = {"params": dict(k=k, L=L, draft_percent=pct, min_draft_pages=mdp, pps=pps, B=B),
                     "num_pages": ((cachelens + page - 1) // page).to(torch.int32), "block_table": block_table,
                     "rows": rows.to(torch.int32), "valid": valid.to(torch.int32)}
        print("recent", name, valid.tolist())
    torch.save(out, HERE / "recent_rows.pt")


def dump_state_case():
    """Dump-state reset of cleared slots: the reference's
    LMBackendBase._clear_variant_slot_state (imported unchanged) on a bound
    stand-in carrying the attributes it reads, for an fp16 first/last dump and
    an fp32 last-token dump; the buffers before and after are saved."""
    import types

    sys.path.insert(0, str(REF))
    from aspire.backends.base import LMBackendBase  # noqa: E402

    out = {}
    for name, (dtype, slots, H, stride) in {"f16_first_last": (torch.float16, 2, 16, 1040),
                                            "f32_last_token": (torch.float32, 1, 4, 2053)}.items():
        B = 6
        g = torch.Generator().manual_seed(slots * 13)
        dump = (torch.randn(B * H * slots * stride, generator=g) * 9).to(dtype)
        q_lens = torch.randint(1, 10, (B,), generator=g)
        qo = torch.zeros(B + 1, dtype=torch.int32)
        qo[1:] = torch.cumsum(q_lens, 0).to(torch.int32)
        lse = torch.randn(int(qo[-1]) + 3, H, generator=g).float()
        flags = torch.zeros(B, dtype=torch.int32)
        before = {"dump": dump.clone(), "lse": lse.clone(), "mode_flags": flags.clone(), "qo_indptr": qo.clone()}
        fake = types.SimpleNamespace(
            attention_weights_buffer=dump, batch_size=B,
            model=types.SimpleNamespace(config=types.SimpleNamespace(n_head=H)),
            _dump_query_slots=lambda slots=slots: slots, _kv_stride_alloc=stride,
            attention_weights_buffer_neg_inf=torch.tensor(float("-inf"), dtype=dtype),
            unified_full_qo_indptr=qo, _lse_buffer=lse, _dump_mode_flags=flags)
        slot_ids = torch.tensor([1, 4, 5])
        LMBackendBase._clear_variant_slot_state(fake, slot_ids)
        out[name] = {"params": dict(B=B, H=H, slots=slots, kv_stride=stride), "slot_ids": slot_ids.to(torch.int32),
                     "before": before, "after": {"dump": dump, "lse": lse, "mode_flags": flags}}
        print("dump_state", name, int(torch.isinf(dump).sum()))
    torch.save(out, HERE / "dump_state.pt")


def spill_case():
    """Draft-page spill insert: the reference's LMBackendBase._handle_draft_page_spill
    (aspire/backends/base.py:718-742, imported unchanged) applied to the spill
    mask that prepare_forward_inputs computes (:1222-1236, whose statements
    are evaluated here on the fixture's tensors), and its host-identified
    variant _handle_draft_page_spill_ids (:744-759) on the rows of that mask
    that have a free column; both must give the same tables.  Rows cover: a
    token opening a new page (spill), the table already ending at that page,
    a full table, no crossing, verify and finished rows, an empty row."""
    import types

    sys.path.insert(0, str(REF))
    from aspire.backends.base import LMBackendBase  # noqa: E402

    page, width, pps = 16, 6, 20
    g = torch.Generator().manual_seed(99)
    B = 12
    block_table = torch.stack([torch.randperm(pps, generator=g) + r * pps for r in range(B)]).to(torch.int32)
    # mode 0 = draft; dec_lens 0 = finished
    mode = torch.tensor([0, 0, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1], dtype=torch.int32)
    dec = torch.tensor([1, 1, 1, 1, 0, 1, 5, 1, 1, 1, 1, 3], dtype=torch.int32)
    dcl = torch.tensor([33, 17, 49, 20, 33, 1, 33, 0, 65, 16, 97, 48], dtype=torch.int32)
    counts = torch.tensor([3, 2, 6, 2, 3, 0, 4, 0, 4, 1, 5, 2], dtype=torch.int32)
    draft = torch.randint(0, B * pps, (B, width), generator=g, dtype=torch.int32)
    # Row 1: the table already ends at the new page (no insert).
    draft[1, 1] = block_table[1, 1]
    # Row 5 (empty table, first token): column 0 holds another page.
    draft[5, 0] = block_table[5, 0] + 1
    before = (draft.clone(), counts.clone())

    def mask(draft_indices, draft_num_pages):
        # aspire/backends/base.py:1222-1236, on this fixture's tensors
        is_draft = mode == 0
        draft_pages_needed = ((dcl + page - 1) // page).to(torch.int32)
        just_crossed = ((dcl - 1) % page == 0) & is_draft & (dec > 0)
        tail_index = (draft_num_pages.to(torch.long) - 1).clamp(min=0)
        tail_page = draft_indices.gather(1, tail_index.unsqueeze(1)).squeeze(1)
        new_page_index = (draft_pages_needed.to(torch.long) - 1).clamp(min=0)
        new_page = block_table.gather(1, new_page_index.unsqueeze(1)).squeeze(1).to(tail_page.dtype)
        return just_crossed & (tail_page != new_page), draft_pages_needed

    fake = types.SimpleNamespace(_draft_indices=draft, target_block_table=block_table,
                                 _draft_num_pages_per_request=counts, draft_cachelens=dcl,
                                 _get_num_pages=lambda s: (s + page - 1) // page)
    need, needed = mask(draft, counts)
    LMBackendBase._handle_draft_page_spill(fake, need, needed, counts)
    # Host-identified path on a fresh copy: the rows of the mask with room.
    d2, c2 = before[0].clone(), before[1].clone()
    fake2 = types.SimpleNamespace(_draft_indices=d2, target_block_table=block_table,
                                  _draft_num_pages_per_request=c2, draft_cachelens=dcl,
                                  _get_num_pages=lambda s: (s + page - 1) // page)
    need2, _ = mask(d2, c2)
    ids = torch.nonzero(need2 & (c2 < width), as_tuple=True)[0]
    LMBackendBase._handle_draft_page_spill_ids(fake2, ids, B)
    assert torch.equal(d2, draft) and torch.equal(c2, counts), "mask and id spill paths differ"
    out = {"mode_flags": mode, "dec_lens": dec, "draft_cachelens": dcl, "block_table": block_table,
           "draft_before": before[0], "counts_before": before[1], "draft_after": draft, "counts_after": counts,
           "spill_rows": ids}
    print("spill rows", ids.tolist(), "counts", counts.tolist())
    torch.save(out, HERE / "draft_spill.pt")


def main(groups=None):
    """Writes every fixture, or only those of the named groups (selector,
    last_token, ties, append, indices, recent, spill, dump_state)."""
    if not os.environ.get("ASPIRE_REFERENCE") or not REF.exists():
        raise SystemExit("set ASPIRE_REFERENCE to the root of the reference (ASPIRE) checkout")
    want = lambda g: not groups or g in groups  # noqa: E731
    if want("selector"):
        # BASELINE config 1 geometry: 16 heads, 1024-token cache, 8 selected pages.
        selector_case("cfg1", B=4, H=16, max_seq_len=1024, kv_stride=1024, top_k_pages=8, L=2,
                      draft_percent=None, seed=0, q_lens=[1, 1, 5, 5], lens=[1000, 1024, 1021, 1024],
                      stale_rows=(0, 1))
        # Engine defaults (top_k_pages 32, recent 8, draft_percent 7) on a long, padded-stride dump,
        # with a tiny row (num_pages < L) and a row whose first-query LSE is -inf (NaN -> -inf path).
        selector_case("pct", B=3, H=2, max_seq_len=16640, kv_stride=16768, top_k_pages=32, L=8,
                      draft_percent=7.0, seed=1, q_lens=[5, 1, 9], lens=[16633, 70, 9001],
                      stale_rows=(1,), lse_neg_inf_rows=(2,))
        # Config-2-like (budget 128 pages, L 8, draft_percent unset), local heads of TP 4.
        selector_case("budget", B=2, H=4, max_seq_len=16640, kv_stride=16640, top_k_pages=128, L=8,
                      draft_percent=None, seed=2, q_lens=[5, 3], lens=[16500, 16001])
    if want("last_token"):
        # The base backend's selector on its last-token dump: config-1 geometry in
        # fp16, and a padded-stride fp32 dump with draft_percent and a -inf LSE row.
        last_token_case("cfg1", B=4, H=16, max_seq_len=1024, kv_stride=1024, top_k_pages=8, L=2,
                        draft_percent=None, seed=10, q_lens=[1, 1, 5, 5], lens=[1000, 1024, 1021, 1024])
        last_token_case("f32", B=3, H=4, max_seq_len=4000, kv_stride=4096, top_k_pages=32, L=8,
                        draft_percent=7.0, seed=11, q_lens=[5, 1, 9], lens=[3990, 70, 2500],
                        dump_dtype=torch.float32, lse_neg_inf_rows=(2,))
    if want("ties"):
        tie_case()
    if want("append"):
        append_case()
    if want("indices"):
        indices_case()
    if want("recent"):
        recent_case()
    if want("spill"):
        spill_case()
    if want("dump_state"):
        dump_state_case()


if __name__ == "__main__":
    main(sys.argv[1:])
