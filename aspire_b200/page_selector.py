"""Page selection on the GPU: drop-in for ``PageSelector`` and
``PageSelectorFirstLastAvg``.

Same constructor and ``compute_valid_counts`` / ``select`` /
``select_subset`` surface as ``aspire/backends/page_selector.py:7-233``
(plus ``select_from_compact_first_last`` and
``select_layers_from_compact_first_last`` on the first/last class); scoring
and top-k run as two kernels per call (``aspire_select_pages``) instead of
~20 torch ops.  ``PageSelector`` scores pages from the last-token dump of
``LMBackendBase`` (one slot per head), ``PageSelectorFirstLastAvg`` from the
first/last dump of the ASPIRE backend; either dump may be fp16 or fp32.

``select`` returns ``(selected[B, k] int32, valid_counts[B] int32)`` with the
reference's layout: the valid prefix of each row holds the selected
block-table ids in ascending order and the tail is zero.  ``select_into``
writes the same rows straight into the caller's draft table and count
buffer, fusing ``LMBackendBase._store_draft_rows`` (``base.py:1421-1471``)
into the selection kernel, as ``_whole_batch_replan_impl`` (``base.py:648-667``)
uses it.  Ties between equal page scores are broken by the lower page index.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _capi


class PageSelector:
    """Last verify-token page selector backed by libaspire_b200
    (``PageSelector``, aspire/backends/page_selector.py:7-158): a page's
    score is the sum over its tokens of exp2(max over heads of
    logit * sm_scale * log2(e) - LSE of the row's last query)."""

    _dump_kind = _capi.DUMP_LAST_TOKEN
    _dump_slots = 1

    def __init__(self, max_batch_size, pages_per_slot, subset_cache_size, L, n_heads, page_size,
                 max_seq_length, device, bsz, dec_len, head_dim=128, kv_stride=None,
                 draft_percent=None, min_draft_pages=None):
        self._lib = _capi.load_library()
        self.subset_cache_size = int(subset_cache_size)
        self.L = int(L)
        self._min_draft_pages = min_draft_pages
        self.n_heads = int(n_heads)
        self.page_size = int(page_size)
        self.max_seq_length = int(max_seq_length)
        self._kv_stride = int(kv_stride or max_seq_length)
        self.pages_per_slot = int(pages_per_slot)
        self.device = torch.device(device)
        self._draft_percent = draft_percent
        self._bsz = int(bsz)
        self._dec_len = dec_len
        self._head_dim = int(head_dim)
        self._sm_scale = 1.0 / math.sqrt(head_dim)
        self._max_batch = int(max_batch_size)
        k = self.subset_cache_size
        self._selected_buf = torch.zeros(max_batch_size, max(k, 1), dtype=torch.int32, device=self.device)
        self._valid_counts_buf = torch.zeros(max_batch_size, dtype=torch.int32, device=self.device)
        self._scores = torch.empty(max_batch_size, pages_per_slot, dtype=torch.float32, device=self.device)

    # --------------------------------------------------------------- helpers
    def compute_valid_counts(self, num_pages: torch.Tensor) -> torch.Tensor:
        """Per-request draft page count (``page_selector.py:52-62``)."""
        hi = num_pages.clamp(max=self.subset_cache_size).to(torch.int32)
        if self._draft_percent is None:
            if self._min_draft_pages is not None:
                return num_pages.clamp(max=self._min_draft_pages).to(torch.int32)
            return hi
        floor = self._min_draft_pages if self._min_draft_pages is not None else self.L
        lo = num_pages.clamp(max=floor).to(torch.int32)
        target = (num_pages.float() * self._draft_percent / 100).ceil_().to(torch.int32)
        return torch.clamp(target, lo, hi)

    def _launch(self, *, dump, lse, qo_indptr, row_ids, scores_in, num_pages, block_table, batch,
                table_out, table_width, counts_out, scores_out=None, status=None, order_by_page=False,
                kv_stride=None):
        def ptr(t):
            return t.data_ptr() if t is not None else None

        for name, t in (("num_pages", num_pages), ("block_table", block_table), ("table_out", table_out),
                        ("counts_out", counts_out), ("qo_indptr", qo_indptr), ("row_ids", row_ids)):
            if t is not None and t.dtype != torch.int32:
                raise ValueError(f"{name} must be int32, got {t.dtype}")
        if block_table.stride(1) != 1 or table_out.stride(1) != 1:
            raise ValueError("block_table and table rows must be contiguous")
        if block_table.shape[0] < batch or num_pages.shape[0] < batch or table_out.shape[0] < batch \
                or counts_out.shape[0] < batch:
            raise ValueError("block_table / num_pages / outputs have fewer rows than the batch")
        stride = self._kv_stride if kv_stride is None else int(kv_stride)
        # The scores land in scores_out, or in a scratch buffer of `batch` rows:
        # the selector's own holds max_batch_size rows, so larger batches (the
        # layered entry point) take a temporary one, as the reference's
        # _get_scores_buffer does (page_selector.py:64-67).
        if scores_out is not None and (scores_out.dtype != torch.float32 or not scores_out.is_contiguous()
                                       or scores_out.dim() != 2 or scores_out.shape[0] < batch
                                       or scores_out.shape[1] != self.pages_per_slot):
            raise ValueError("scores_out must be a contiguous fp32 [>= batch, pages_per_slot] tensor")
        scores_ws = self._scores
        if scores_in is None and scores_out is None and batch > self._scores.shape[0]:
            scores_ws = torch.empty(batch, self.pages_per_slot, dtype=torch.float32, device=self.device)
        if dump is not None:
            if dump.dtype not in (torch.float16, torch.float32) or not dump.is_contiguous():
                raise ValueError("dump buffer must be a contiguous float16 or float32 tensor")
            rows = int(row_ids.max().item()) + 1 if row_ids is not None else batch
            if dump.numel() < rows * self.n_heads * self._dump_slots * stride:
                raise ValueError(f"dump buffer smaller than rows * n_heads * {self._dump_slots} * kv_stride")
            if lse is None or lse.dtype != torch.float32 or not lse.is_contiguous() or lse.shape[1] != self.n_heads:
                raise ValueError("lse must be a contiguous fp32 [tokens, n_heads] tensor")
            if qo_indptr.shape[0] < rows + 1:
                raise ValueError("qo_indptr needs rows + 1 entries")
        a = _capi.AspireSelectArgs()
        a.dump = ptr(dump)
        a.dump_kind = self._dump_kind
        a.dump_dtype = _capi.DUMP_F32 if dump is not None and dump.dtype == torch.float32 else _capi.DUMP_F16
        a.kv_stride = stride
        a.max_seq_len = self.max_seq_length
        a.lse = ptr(lse)
        a.lse_rows = lse.shape[0] if lse is not None else 0
        a.qo_indptr = ptr(qo_indptr)
        a.row_ids = ptr(row_ids)
        a.scores_in = ptr(scores_in)
        a.num_pages = num_pages.data_ptr()
        a.block_table = block_table.data_ptr()
        a.block_table_stride = block_table.stride(0)
        a.block_table_cols = block_table.shape[1]
        a.batch = int(batch)
        a.num_heads = self.n_heads
        a.page_size = self.page_size
        a.pages_per_slot = self.pages_per_slot
        a.L = self.L
        a.subset_cache_size = self.subset_cache_size
        a.min_draft_pages = -1 if self._min_draft_pages is None else int(self._min_draft_pages)
        a.draft_percent = -1.0 if self._draft_percent is None else float(self._draft_percent)
        a.sm_scale = self._sm_scale
        a.head_dim = self._head_dim
        a.table_out = table_out.data_ptr()
        a.table_stride = table_out.stride(0)
        a.table_width = int(table_width)
        a.counts_out = counts_out.data_ptr()
        a.scores_out = ptr(scores_out)
        a.scores_ws = scores_ws.data_ptr()
        a.status = ptr(status)
        a.order_by_page = 1 if order_by_page else 0
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _capi.check(self._lib.aspire_select_pages(ctypes.byref(a), ctypes.c_void_p(stream)),
                    "aspire_select_pages")

    def _contig_i32(self, t: torch.Tensor) -> torch.Tensor:
        t = t.to(device=self.device, dtype=torch.int32)
        return t if t.is_contiguous() else t.contiguous()

    # ------------------------------------------------------------------ API
    def select(self, attention_weights_buffer, lse_buffer, num_pages, block_table, qo_indptr,
               scores_out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Whole-batch selection (``page_selector.py:140-146``; first/last:
        ``:206-214``)."""
        B = self._bsz
        sel = self._selected_buf[:B]
        counts = self._valid_counts_buf[:B]
        self._launch(dump=attention_weights_buffer, lse=lse_buffer, qo_indptr=self._contig_i32(qo_indptr),
                     row_ids=None, scores_in=None, num_pages=self._contig_i32(num_pages[:B]),
                     block_table=self._contig_i32(block_table), batch=B, table_out=sel,
                     table_width=self.subset_cache_size, counts_out=counts, scores_out=scores_out)
        return sel, counts

    def select_into(self, table, count_buffer, attention_weights_buffer, lse_buffer, num_pages,
                    block_table, qo_indptr, batch: Optional[int] = None,
                    scores_out: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None):
        """Selection written in place into ``table[:B]`` / ``count_buffer[:B]`` (zero tail)."""
        B = self._bsz if batch is None else int(batch)
        self._launch(dump=attention_weights_buffer, lse=lse_buffer, qo_indptr=self._contig_i32(qo_indptr),
                     row_ids=None, scores_in=None, num_pages=self._contig_i32(num_pages[:B]),
                     block_table=self._contig_i32(block_table), batch=B, table_out=table,
                     table_width=table.shape[1], counts_out=count_buffer, scores_out=scores_out,
                     status=status)

    def select_subset(self, slot_ids, attention_weights_buffer, lse_buffer, num_pages, block_table,
                      qo_indptr) -> Tuple[torch.Tensor, torch.Tensor]:
        """Selection for a subset of slots (``page_selector.py:148-158``; first/last: ``:216-233``)."""
        if slot_ids.numel() == 0:
            empty = block_table.new_empty((0, self.subset_cache_size), dtype=torch.int32)
            return empty, torch.zeros(0, dtype=torch.int32, device=self.device)
        ids = slot_ids.to(device=self.device, dtype=torch.long)
        n = ids.numel()
        sel = torch.zeros(n, self.subset_cache_size, dtype=torch.int32, device=self.device)
        counts = torch.zeros(n, dtype=torch.int32, device=self.device)
        self._launch(dump=attention_weights_buffer, lse=lse_buffer, qo_indptr=self._contig_i32(qo_indptr),
                     row_ids=self._contig_i32(ids), scores_in=None,
                     num_pages=self._contig_i32(num_pages[ids]), block_table=self._contig_i32(block_table[ids]),
                     batch=n, table_out=sel, table_width=self.subset_cache_size, counts_out=counts)
        return sel, counts

    def _index_scores(self) -> torch.Tensor:
        """Page-index scores [max_batch, pages_per_slot] (static, built once)."""
        if getattr(self, "_recent_scores", None) is None:
            idx = torch.arange(self.pages_per_slot, dtype=torch.float32, device=self.device)
            self._recent_scores = idx.expand(self._scores.shape[0], -1).contiguous()
        return self._recent_scores

    def seed_recent(self, num_pages: torch.Tensor, block_table: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Recent-page draft rows for rows with no verify signal yet: the last
        ``compute_valid_counts(num_pages)`` pages of each row's block table in
        page order, zero tail (``LMBackendBase._build_recent_draft_rows``,
        aspire/backends/base.py:1522-1537).  One launch of the selection kernel
        on page-index scores; returns ``(rows [n, k], valid_counts [n])``."""
        n = num_pages.shape[0]
        rows = torch.zeros(n, self.subset_cache_size, dtype=torch.int32, device=self.device)
        counts = torch.zeros(n, dtype=torch.int32, device=self.device)
        if n:
            self.seed_recent_into(rows, counts, num_pages, block_table)
        return rows, counts

    def seed_recent_into(self, table: torch.Tensor, count_buffer: torch.Tensor, num_pages: torch.Tensor,
                         block_table: torch.Tensor) -> None:
        """``seed_recent`` written in place into rows [0, n) of ``table`` and
        ``count_buffer`` (static buffers, so the call can be captured)."""
        n = num_pages.shape[0]
        if n > self._scores.shape[0]:
            raise ValueError("more rows than max_batch_size")
        self._launch(dump=None, lse=None, qo_indptr=None, row_ids=None, scores_in=self._index_scores(),
                     num_pages=self._contig_i32(num_pages), block_table=block_table, batch=n, table_out=table,
                     table_width=table.shape[1], counts_out=count_buffer, order_by_page=True)

    def finalize_scores(self, scores: torch.Tensor, num_pages: torch.Tensor,
                        block_table: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-k stage alone from raw fp32 page scores (``page_selector.py:79-108``)."""
        n = scores.shape[0]
        if scores.dtype != torch.float32 or not scores.is_contiguous() or scores.shape[1] != self.pages_per_slot:
            raise ValueError("scores must be contiguous fp32 [batch, pages_per_slot]")
        sel = torch.zeros(n, self.subset_cache_size, dtype=torch.int32, device=self.device)
        counts = torch.zeros(n, dtype=torch.int32, device=self.device)
        self.finalize_scores_into(sel, counts, scores, num_pages, block_table)
        return sel, counts

    def finalize_scores_into(self, table: torch.Tensor, count_buffer: torch.Tensor, scores: torch.Tensor,
                             num_pages: torch.Tensor, block_table: torch.Tensor) -> None:
        """``finalize_scores`` written in place into rows [0, n) of ``table`` /
        ``count_buffer`` (zero tail); allocates nothing, so it can be captured."""
        n = scores.shape[0]
        if scores.dtype != torch.float32 or not scores.is_contiguous() or scores.shape[1] != self.pages_per_slot:
            raise ValueError("scores must be contiguous fp32 [batch, pages_per_slot]")
        self._launch(dump=None, lse=None, qo_indptr=None, row_ids=None, scores_in=scores,
                     num_pages=self._contig_i32(num_pages), block_table=self._contig_i32(block_table),
                     batch=n, table_out=table, table_width=table.shape[1], counts_out=count_buffer)


class PageSelectorFirstLastAvg(PageSelector):
    """First/last verify-token page selector backed by libaspire_b200
    (``PageSelectorFirstLastAvg``, aspire/backends/page_selector.py:160-233):
    a token's score is the sum over the two dump slots of exp2(max over heads
    of logit * sm_scale * log2(e) - LSE of the slot's query)."""

    _dump_kind = _capi.DUMP_FIRST_LAST
    _dump_slots = 2

    def _compact_launch(self, logits, first_lse, last_lse, num_pages, block_table):
        """Selection from an explicit [rows, n_heads, 2, max_seq_length] logit
        view (a narrowing of a [rows, n_heads, 2, kv_stride] buffer) and the
        first / last query LSE of each row [rows, n_heads]: the LSE rows are
        interleaved so that the kernel's (first, last) query of row b are rows
        2b and 2b + 1."""
        n = logits.shape[0]
        if logits.dim() != 4 or logits.shape[1] != self.n_heads or logits.shape[2] != 2:
            raise ValueError("logits must be [rows, n_heads, 2, seq_len]")
        s = logits.stride(2)
        if logits.stride(3) != 1 or logits.stride(1) != 2 * s or logits.stride(0) != self.n_heads * 2 * s \
                or logits.shape[3] != self.max_seq_length or s < self.max_seq_length:
            raise ValueError("logits must be a [rows, n_heads, 2, max_seq_length] view of a contiguous "
                             "[rows, n_heads, 2, kv_stride] buffer")
        base = logits.as_strided((n * self.n_heads * 2 * s,), (1,))
        lse = torch.stack([first_lse.float(), last_lse.float()], dim=1).reshape(2 * n, self.n_heads).contiguous()
        qo = torch.arange(0, 2 * n + 1, 2, dtype=torch.int32, device=self.device)
        sel = torch.zeros(n, self.subset_cache_size, dtype=torch.int32, device=self.device)
        counts = torch.zeros(n, dtype=torch.int32, device=self.device)
        self._launch(dump=base, lse=lse, qo_indptr=qo, row_ids=None, scores_in=None,
                     num_pages=self._contig_i32(num_pages), block_table=self._contig_i32(block_table), batch=n,
                     table_out=sel, table_width=self.subset_cache_size, counts_out=counts, kv_stride=s)
        return sel, counts

    def select_from_compact_first_last(self, logits, first_lse, last_lse, num_pages, block_table):
        """``page_selector.py:183-184``: logits [B, n_heads, 2, seq_len],
        first_lse / last_lse [B, n_heads]."""
        return self._compact_launch(logits, first_lse, last_lse, num_pages, block_table)

    def select_layers_from_compact_first_last(self, logits, first_lse, last_lse, num_pages, block_table):
        """``page_selector.py:186-204``: logits [n_layers, B, n_heads, 2,
        kv_stride], LSE [n_layers, B, n_heads]; returns
        (selected [n_layers, B, k], valid_counts [B])."""
        n_layers, batch = logits.shape[:2]
        flat = logits.reshape(n_layers * batch, self.n_heads, 2, logits.shape[-1])
        if flat.shape[-1] != self.max_seq_length:
            flat = flat[..., :self.max_seq_length]
        sel, counts = self._compact_launch(flat, first_lse.reshape(n_layers * batch, self.n_heads),
                                           last_lse.reshape(n_layers * batch, self.n_heads),
                                           num_pages.repeat(n_layers), block_table.repeat(n_layers, 1))
        return sel.view(n_layers, batch, self.subset_cache_size), counts[:batch]
