"""CPU restatement of mylib::update_kv_padded (test infrastructure).

Follows aspire/attention/kv_ops.py:63-187 with FlashInfer's helpers:
seq_len[b] = clamp(pages[b] - 1, 0) * page_size + last_page_len[b]
(flashinfer/page.py get_seq_lens); token t of row b (append_indptr[b] <= t <
append_indptr[b+1]) gets position t + seq_len[b] - append_indptr[b+1]
(flashinfer/triton/page.py get_batch_indices_positions_kernel), tokens of no
row get position -1; a token is skipped when its position is negative, its
row has no pages, or the position is past the row's length
(kv_ops.py:92-98); otherwise K and V land at
cache[page_indices[page_indptr[b] + pos // page], 0/1, pos % page, head].
"""

from __future__ import annotations

import torch


def positions(append_indptr: torch.Tensor, page_indptr: torch.Tensor, last_page_len: torch.Tensor,
              num_tokens: int, page_size: int = 16):
    """Returns (batch_indices, positions) int64 [num_tokens] as the Triton helper fills them."""
    seq_lens = (torch.clamp(page_indptr[1:] - page_indptr[:-1] - 1, min=0) * page_size
                + last_page_len)
    n_rows = seq_lens.shape[0]
    bidx = torch.zeros(num_tokens, dtype=torch.int64)
    pos = torch.full((num_tokens,), -1, dtype=torch.int64)
    for b in range(n_rows):
        start, end = int(append_indptr[b]), int(append_indptr[b + 1])
        for t in range(start, min(end, num_tokens)):
            bidx[t] = b
            pos[t] = t + int(seq_lens[b]) - end
    return bidx, pos


def update_kv_padded(k: torch.Tensor, v: torch.Tensor, append_indptr: torch.Tensor, kv_cache: torch.Tensor,
                     page_indices: torch.Tensor, page_indptr: torch.Tensor, last_page_len: torch.Tensor,
                     page_size: int = 16) -> None:
    """Writes k / v [T, Hkv, D] into kv_cache [P, 2, page, Hkv, D] in place."""
    T = k.shape[0]
    if T == 0:
        return
    bidx, pos = positions(append_indptr, page_indptr, last_page_len, T, page_size)
    for t in range(T):
        b, p = int(bidx[t]), int(pos[t])
        if p < 0:
            continue
        start, end = int(page_indptr[b]), int(page_indptr[b + 1])
        count = end - start
        if count == 0:
            continue
        length = (count - 1) * page_size + int(last_page_len[b])
        if p >= length:
            continue
        page = int(page_indices[start + p // page_size])
        kv_cache[page, 0, p % page_size] = k[t].to(kv_cache.dtype)
        kv_cache[page, 1, p % page_size] = v[t].to(kv_cache.dtype)
