"""Seeded synthetic mixed draft/verify batches of the benchmark shapes.

A batch is a set of request rows over one layer's paged KV cache
``[pages, 2, 16, Hkv, 128]``.  Row r owns ``pages_per_row`` physical pages
whose order is a random permutation (the block table).  A VERIFY row
attends its whole context (``ctx`` tokens, which include its ``q_len`` new
tokens) with a causal multi-token query; a DRAFT row (q_len 1) attends a
sparse table of ``budget`` pages: ``budget - 1`` distinct random pages of its
context plus its last page, ascending, its last page partially filled as the
reference's append-through-sparse-table invariant leaves it
(aspire/backends/base.py:1204-1213).  Q, K and V are N(0, 1).

Shapes follow the reference's benchmark configs (Qwen3-1.7B heads 16/8/128,
Qwen3-8B heads 32/8/128; page size 16).  Datasets are replaced by these
seeded draws.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

PAGE = 16
HEAD_DIM = 128


@dataclass
class MixedLayout:
    """Host-side metadata of one mixed batch (int32 numpy arrays)."""

    num_qo_heads: int
    num_kv_heads: int
    modes: np.ndarray          # [B] 0 = draft, 1 = verify
    q_lens: np.ndarray         # [B]
    kv_lens: np.ndarray        # [B] attended tokens
    qo_indptr: np.ndarray      # [B + 1]
    kv_indptr: np.ndarray      # [B + 1]
    kv_indices: np.ndarray     # [sum pages]
    block_table: np.ndarray    # [B, pages_per_row] physical ids
    ctx_lens: np.ndarray       # [B] full context length (verify rows: == kv_len)
    pages_per_row: int
    num_pages_total: int
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.modes.shape[0])

    @property
    def total_q(self) -> int:
        return int(self.qo_indptr[-1])

    def attended_tokens(self) -> int:
        return int(self.kv_lens.sum())

    def algorithmic_bytes(self) -> int:
        """KV bytes read once + Q in + O out + page ids (one layer-call)."""
        kv = self.attended_tokens() * self.num_kv_heads * HEAD_DIM * 2 * 2
        qo = self.total_q * self.num_qo_heads * HEAD_DIM * 2 * 2
        return int(kv + qo + self.kv_indices.shape[0] * 4)


def make_layout(*, batch: int, ctx: int, num_qo_heads: int, num_kv_heads: int, draft_fraction: float,
                verify_q_len: Optional[int] = None, draft_len_range=(2, 8), budget_pages: int = 128,
                pages_per_row: Optional[int] = None, draft_rows: Optional[List[int]] = None,
                seed: int = 0, block_table: str = "random") -> MixedLayout:
    """Builds a mixed layout.  verify_q_len=None draws q_len = U{lo..hi} + 1.

    block_table="random" permutes each row's pages (scattered physical pages);
    "arange" gives row r the contiguous pages [r*pages_per_row, (r+1)*pages_per_row),
    the layout of the reference engine (aspire/models/sparse_draft_runner.py:241-250)."""
    rng = np.random.default_rng(seed)
    block_table_kind = block_table
    if block_table_kind not in ("random", "arange"):
        raise ValueError("block_table must be 'random' or 'arange'")
    if pages_per_row is None:
        pages_per_row = (ctx + PAGE - 1) // PAGE
    modes = np.ones(batch, dtype=np.int32)
    if draft_rows is None:
        n_draft = int(round(draft_fraction * batch))
        draft_rows = sorted(rng.permutation(batch)[:n_draft].tolist())
    modes[list(draft_rows)] = 0
    q_lens = np.zeros(batch, dtype=np.int32)
    kv_lens = np.zeros(batch, dtype=np.int32)
    ctx_lens = np.full(batch, ctx, dtype=np.int32)
    block_table = np.zeros((batch, pages_per_row), dtype=np.int32)
    indices: List[np.ndarray] = []
    kv_indptr = np.zeros(batch + 1, dtype=np.int32)
    for r in range(batch):
        perm = rng.permutation(pages_per_row).astype(np.int32)
        block_table[r] = r * pages_per_row + (perm if block_table_kind == "random" else np.arange(pages_per_row, dtype=np.int32))
        ctx_pages = (ctx + PAGE - 1) // PAGE
        if modes[r] == 1:
            ql = verify_q_len if verify_q_len is not None else int(rng.integers(draft_len_range[0], draft_len_range[1] + 1)) + 1
            q_lens[r] = ql
            kv_lens[r] = ctx
            pages = block_table[r, :ctx_pages]
        else:
            q_lens[r] = 1
            nb = min(budget_pages, ctx_pages)
            chosen = np.sort(rng.choice(ctx_pages - 1, size=nb - 1, replace=False)) if nb > 1 else np.zeros(0, np.int64)
            logical = np.concatenate([chosen, [ctx_pages - 1]]).astype(np.int64)
            pages = block_table[r, logical]
            last_len = ctx - (ctx_pages - 1) * PAGE
            kv_lens[r] = (nb - 1) * PAGE + last_len
        indices.append(pages.astype(np.int32))
        kv_indptr[r + 1] = kv_indptr[r] + pages.shape[0]
    qo_indptr = np.zeros(batch + 1, dtype=np.int32)
    qo_indptr[1:] = np.cumsum(q_lens)
    return MixedLayout(num_qo_heads=num_qo_heads, num_kv_heads=num_kv_heads, modes=modes, q_lens=q_lens,
                       kv_lens=kv_lens, qo_indptr=qo_indptr, kv_indptr=kv_indptr,
                       kv_indices=np.concatenate(indices) if indices else np.zeros(0, np.int32),
                       block_table=block_table, ctx_lens=ctx_lens, pages_per_row=pages_per_row,
                       num_pages_total=batch * pages_per_row)


def config1_layout(seed: int = 0) -> MixedLayout:
    """Qwen3-1.7B heads, rows 0-1 draft (8 of 64 pages), rows 2-3 verify q_len 5."""
    return make_layout(batch=4, ctx=1024, num_qo_heads=16, num_kv_heads=8, draft_fraction=0.5,
                       verify_q_len=5, budget_pages=8, draft_rows=[0, 1], seed=seed)


def fill_tensors(layout: MixedLayout, *, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 kv_cache: Optional[torch.Tensor] = None):
    """Draws q [T, Hq, 128] and the cache [pages, 2, 16, Hkv, 128] from N(0, 1)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = torch.randn(layout.total_q, layout.num_qo_heads, HEAD_DIM, generator=gen, device=device,
                    dtype=torch.float32).to(dtype)
    if kv_cache is None:
        kv_cache = torch.empty(layout.num_pages_total, 2, PAGE, layout.num_kv_heads, HEAD_DIM,
                               device=device, dtype=dtype)
        # Chunked draw keeps the fp32 temporary small for multi-GB caches.
        step = max(1, (1 << 28) // (2 * PAGE * layout.num_kv_heads * HEAD_DIM))
        for p0 in range(0, layout.num_pages_total, step):
            p1 = min(layout.num_pages_total, p0 + step)
            kv_cache[p0:p1] = torch.randn(p1 - p0, 2, PAGE, layout.num_kv_heads, HEAD_DIM, generator=gen,
                                          device=device, dtype=torch.float32).to(dtype)
    return q, kv_cache


def full_context_layout(layout: MixedLayout) -> MixedLayout:
    """The refresh layer's program over the same rows: every row attends its whole
    context (draft rows with their single query), as the reference plans its dump
    wrapper over effective cache lengths (aspire/backends/host_plan.py:281-303)."""
    B = layout.batch
    kv_lens = layout.ctx_lens.astype(np.int32).copy()
    pages = (kv_lens + PAGE - 1) // PAGE
    kv_indptr = np.zeros(B + 1, dtype=np.int32)
    kv_indptr[1:] = np.cumsum(pages)
    idx = np.concatenate([layout.block_table[r, :pages[r]] for r in range(B)]).astype(np.int32)
    return MixedLayout(num_qo_heads=layout.num_qo_heads, num_kv_heads=layout.num_kv_heads, modes=layout.modes.copy(),
                       q_lens=layout.q_lens.copy(), kv_lens=kv_lens, qo_indptr=layout.qo_indptr.copy(),
                       kv_indptr=kv_indptr, kv_indices=idx, block_table=layout.block_table,
                       ctx_lens=layout.ctx_lens.copy(), pages_per_row=layout.pages_per_row,
                       num_pages_total=layout.num_pages_total)


def rows_layout(q_lens, kv_lens, num_qo_heads: int, num_kv_heads: int, seed: int = 0) -> MixedLayout:
    """A batch of explicit rows (q_len, kv_len each), e.g. prefill chunks: rows
    with one query are draft rows, the others verify / prefill rows; each row
    owns a shuffled run of whole pages of one pool."""
    rng = np.random.default_rng(seed)
    B = len(q_lens)
    q_lens = np.asarray(q_lens, np.int32)
    kv_lens = np.asarray(kv_lens, np.int32)
    pages = (kv_lens + PAGE - 1) // PAGE
    ppr = max(int(pages.max()) if B else 1, 1)
    bt = np.stack([r * ppr + rng.permutation(ppr) for r in range(B)]).astype(np.int32)
    kv_indptr = np.zeros(B + 1, np.int32)
    kv_indptr[1:] = np.cumsum(pages)
    idx = np.concatenate([bt[r, :pages[r]] for r in range(B)]).astype(np.int32)
    qo = np.zeros(B + 1, np.int32)
    qo[1:] = np.cumsum(q_lens)
    return MixedLayout(num_qo_heads=num_qo_heads, num_kv_heads=num_kv_heads,
                       modes=(q_lens > 1).astype(np.int32), q_lens=q_lens, kv_lens=kv_lens, qo_indptr=qo,
                       kv_indptr=kv_indptr, kv_indices=idx, block_table=bt, ctx_lens=kv_lens.copy(),
                       pages_per_row=ppr, num_pages_total=B * ppr)


def last_page_lens(layout: MixedLayout) -> np.ndarray:
    """Tokens in each row's last attended page: (kv_len - 1) % 16 + 1, 0 when empty."""
    k = layout.kv_lens.astype(np.int64)
    return np.where(k > 0, (k - 1) % PAGE + 1, 0).astype(np.int32)
