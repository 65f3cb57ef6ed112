"""CPU restatement of the draft-page spill insert (test infrastructure).

Follows LMBackendBase.prepare_forward_inputs (aspire/backends/base.py:1222-1236)
and _handle_draft_page_spill (:718-742):

* draft_pages_needed = ceil(draft_cachelens / page_size)
  (_get_num_pages, aspire/models/mixed_runner.py:114-120);
* just_crossed = ((draft_cachelens - 1) % page_size == 0) & is_draft
  & (dec_lens > 0), with Python's floor modulo;
* tail_page = draft_indices[b, max(draft_num_pages[b] - 1, 0)];
  new_page = block_table[b, max(draft_pages_needed[b] - 1, 0)];
* a row spills when it just crossed and tail_page != new_page; the new page
  is written at column draft_num_pages[b] and the count incremented, when
  that column exists (insert_pos < max_width).
"""

from __future__ import annotations

import torch


def draft_page_spill(mode_flags: torch.Tensor, dec_lens: torch.Tensor, draft_cachelens: torch.Tensor,
                     draft_indices: torch.Tensor, draft_num_pages: torch.Tensor, block_table: torch.Tensor,
                     page_size: int = 16) -> None:
    """Edits draft_indices [B, W] and draft_num_pages [B] in place (int32 CPU tensors)."""
    B, width = draft_indices.shape
    for b in range(B):
        length = int(draft_cachelens[b])
        if int(mode_flags[b]) != 0 or int(dec_lens[b]) <= 0:
            continue
        if (length - 1) % page_size != 0:
            continue
        needed = -(-length // page_size)
        tail = int(draft_indices[b, max(int(draft_num_pages[b]) - 1, 0)])
        new_page = int(block_table[b, max(needed - 1, 0)])
        if tail == new_page:
            continue
        pos = int(draft_num_pages[b])
        if pos < width:
            draft_indices[b, pos] = new_page
            draft_num_pages[b] = pos + 1
