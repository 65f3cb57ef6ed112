"""CPU restatement of ASPIRE's page selectors (test infrastructure).

Restates, as plain functions over torch CPU tensors:

* ``valid_counts``      - PageSelector.compute_valid_counts
                          (aspire/backends/page_selector.py:52-62)
* ``first_last_scores`` - PageSelectorFirstLastAvg._select_first_last_impl up
                          to the page-score buffer (page_selector.py:163-180):
                          fp16 logit * (sm_scale*log2 e) stays fp16, minus the
                          fp32 LSE of the first / last query, NaN -> -inf,
                          exp2, max over heads, sum of the two slots, zero pad
                          to pages*16, sum of each page's 16 tokens, plus the
                          position bias -page*1e-7 (page_selector.py:34-36).
* ``last_token_scores`` - PageSelector._select_impl up to the page-score
                          buffer (page_selector.py:110-127): logit *
                          (sm_scale*log2 e) in the dump's dtype, minus the
                          fp32 LSE of the row's last query, NaN -> -inf, max
                          over heads, exp2, zero pad, page sums, position bias.
* ``finalize_scores``   - _finalize_scores (page_selector.py:79-108): last L
                          valid pages +inf, pages >= num_pages -inf, top-k,
                          gather block-table ids, keep the valid prefix by
                          rank, ascending sort, zero tail.  The reference
                          leaves the order of tied scores to torch.topk; this
                          restatement fixes it to "lower page index first"
                          (stable descending sort), the rule the GPU kernel
                          implements.
* ``select``            - PageSelectorFirstLastAvg.select (page_selector.py:206-214).
* ``select_last_token`` - PageSelector.select (page_selector.py:140-146).
* ``store_draft_rows``  - LMBackendBase._store_draft_rows with full_prefix
                          (aspire/backends/base.py:1421-1471).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def valid_counts(num_pages: torch.Tensor, k: int, L: int, draft_percent: Optional[float],
                 min_draft_pages: Optional[int]) -> torch.Tensor:
    hi = num_pages.clamp(max=k).to(torch.int32)
    if draft_percent is None:
        if min_draft_pages is not None:
            return num_pages.clamp(max=min_draft_pages).to(torch.int32)
        return hi
    floor = min_draft_pages if min_draft_pages is not None else L
    lo = num_pages.clamp(max=floor).to(torch.int32)
    target = torch.ceil(num_pages.to(torch.float32) * draft_percent / 100).to(torch.int32)
    return torch.clamp(target, lo, hi)


def position_bias(pages_per_slot: int) -> torch.Tensor:
    return -torch.arange(pages_per_slot, dtype=torch.float32) * 1e-7


def first_last_scores(logits: torch.Tensor, first_lse: torch.Tensor, last_lse: torch.Tensor,
                      pages_per_slot: int, page_size: int, head_dim: int = 128) -> torch.Tensor:
    """logits: fp16 [B, H, 2, S]; first_lse / last_lse: fp32 [B, H] -> fp32 [B, pages]."""
    B, _, _, S = logits.shape
    c = (1.0 / math.sqrt(head_dim)) * math.log2(math.e)
    scaled = logits * c                                   # fp16 op: rounded to fp16
    lse = torch.stack([first_lse, last_lse], dim=2)      # [B, H, 2]
    norm = scaled - lse[:, :, :, None]                   # promoted to fp32
    norm = torch.nan_to_num(norm, nan=float("-inf"))
    per_token = torch.exp2(norm).amax(dim=1).sum(dim=1)  # [B, S]
    pad = pages_per_slot * page_size - S
    if pad > 0:
        per_token = F.pad(per_token, (0, pad))
    scores = per_token.view(B, pages_per_slot, page_size).sum(dim=-1)
    return scores + position_bias(pages_per_slot)


def last_token_scores(logits: torch.Tensor, lse: torch.Tensor, pages_per_slot: int, page_size: int,
                      head_dim: int = 128) -> torch.Tensor:
    """logits: fp16 or fp32 [B, H, S]; lse: fp32 [B, H] -> fp32 [B, pages]."""
    B, _, S = logits.shape
    c = (1.0 / math.sqrt(head_dim)) * math.log2(math.e)
    norm = logits * c - lse[:, :, None]                  # fp16 product rounded to fp16, then fp32
    norm = torch.nan_to_num(norm.float(), nan=float("-inf"))
    per_token = torch.exp2(norm.amax(dim=1))             # [B, S]
    pad = pages_per_slot * page_size - S
    if pad > 0:
        per_token = F.pad(per_token, (0, pad))
    scores = per_token.view(B, pages_per_slot, page_size).sum(dim=-1)
    return scores + position_bias(pages_per_slot)


def finalize_scores(scores: torch.Tensor, num_pages: torch.Tensor, block_table: torch.Tensor, k: int,
                    L: int, draft_percent: Optional[float] = None,
                    min_draft_pages: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k page selection from fp32 scores [B, pages]; returns (selected[B,k], valid[B])."""
    scores = scores.clone()
    B, P = scores.shape
    j = torch.arange(P)[None]
    npl = num_pages.long()
    last_start = (npl - L).clamp(min=0)
    scores[(j >= last_start[:, None]) & (j < npl[:, None])] = float("inf")
    scores[j >= npl[:, None]] = float("-inf")
    order = torch.sort(scores, dim=1, descending=True, stable=True).indices[:, :k]
    order = order.clamp(max=block_table.shape[1] - 1)
    selected = torch.gather(block_table.to(torch.int32), 1, order)
    valid = valid_counts(num_pages, k, L, draft_percent, min_draft_pages)
    keep = torch.arange(k)[None, :] < valid[:, None]
    sentinel = torch.iinfo(torch.int32).max
    selected = torch.where(keep, selected, torch.full_like(selected, sentinel))
    selected = selected.sort(dim=1).values
    selected = torch.where(keep, selected, torch.zeros_like(selected))
    return selected, valid


def select(dump: torch.Tensor, lse_buffer: torch.Tensor, num_pages: torch.Tensor, block_table: torch.Tensor,
           qo_indptr: torch.Tensor, *, batch: int, n_heads: int, kv_stride: int, max_seq_len: int,
           pages_per_slot: int, k: int, L: int, page_size: int = 16, head_dim: int = 128,
           draft_percent: Optional[float] = None, min_draft_pages: Optional[int] = None,
           return_scores: bool = False):
    """Whole-batch selection from the flat fp16 dump buffer and the LSE buffer."""
    logits = dump.view(batch, n_heads, 2, kv_stride)[..., :max_seq_len]
    max_q = max(lse_buffer.shape[0] - 1, 0)
    first = qo_indptr[:batch].long().clamp(min=0, max=max_q)
    last = (qo_indptr[1: batch + 1].long() - 1).clamp(min=0, max=max_q)
    scores = first_last_scores(logits, lse_buffer[first], lse_buffer[last], pages_per_slot, page_size,
                               head_dim)
    selected, valid = finalize_scores(scores, num_pages[:batch], block_table[:batch], k, L,
                                      draft_percent, min_draft_pages)
    if return_scores:
        return selected, valid, scores
    return selected, valid


def select_last_token(dump: torch.Tensor, lse_buffer: torch.Tensor, num_pages: torch.Tensor,
                      block_table: torch.Tensor, qo_indptr: torch.Tensor, *, batch: int, n_heads: int,
                      kv_stride: int, max_seq_len: int, pages_per_slot: int, k: int, L: int, page_size: int = 16,
                      head_dim: int = 128, draft_percent: Optional[float] = None,
                      min_draft_pages: Optional[int] = None, return_scores: bool = False):
    """Whole-batch selection from the flat last-token dump buffer and the LSE buffer."""
    logits = dump.view(batch, n_heads, kv_stride)[..., :max_seq_len]
    last = (qo_indptr[1: batch + 1].long() - 1).clamp(min=0)
    scores = last_token_scores(logits, lse_buffer[last], pages_per_slot, page_size, head_dim)
    selected, valid = finalize_scores(scores, num_pages[:batch], block_table[:batch], k, L,
                                      draft_percent, min_draft_pages)
    if return_scores:
        return selected, valid, scores
    return selected, valid


def store_draft_rows(table: torch.Tensor, count_buffer: torch.Tensor, selected: torch.Tensor,
                     valid: torch.Tensor) -> None:
    """Writes the leading rows of `table` / `count_buffer` (full_prefix form)."""
    rows = selected.shape[0]
    count_buffer[:rows] = valid.to(count_buffer.dtype)
    width = table.shape[1]
    n_cols = min(width, selected.shape[1])
    staged = torch.zeros(rows, width, dtype=table.dtype)
    if n_cols > 0:
        keep = torch.arange(n_cols)[None, :] < valid[:, None]
        staged[:, :n_cols] = torch.where(keep, selected[:, :n_cols].to(table.dtype), staged[:, :n_cols])
    table[:rows] = staged


def recent_rows(num_pages, block_table, k, L, draft_percent=None, min_draft_pages=None):
    """Recent-page draft rows (LMBackendBase._build_recent_draft_rows,
    aspire/backends/base.py:1522-1537): valid = compute_valid_counts(num_pages);
    row b lists block_table[b, num_pages[b] - valid[b] + j] for j < valid[b]
    and zeros after, over k = max_draft_pages columns."""
    num_pages = torch.as_tensor(num_pages).to(torch.int64)
    valid = valid_counts(num_pages, k, L, draft_percent, min_draft_pages).to(torch.int64)
    offsets = torch.arange(k, dtype=torch.int64)
    start = (num_pages - valid).clamp(min=0)
    pos = start[:, None] + offsets[None, :]
    rows = torch.as_tensor(block_table).gather(1, pos.clamp(max=block_table.shape[1] - 1))
    rows = torch.where(offsets[None, :] < valid[:, None], rows, torch.zeros_like(rows))
    return rows.to(torch.int32), valid.to(torch.int32)
