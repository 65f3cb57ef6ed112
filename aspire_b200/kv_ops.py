"""Paged KV append: drop-in for ``mylib::update_kv_padded``.

Same schema and error behaviour as ``aspire/attention/kv_ops.py:127-187``:
``(Tensor k, Tensor v, Tensor kv_append_indptr, Tensor(a!) kv_cache,
Tensor kv_page_indices, Tensor kv_page_indptr, Tensor kv_last_page_len,
int page_size) -> ()``; non-contiguous k/v heads raise ``ValueError``.
Registered as ``aspire_b200::update_kv_padded`` with a fake implementation
so ``torch.compile(fullgraph=True)`` can trace it.

The module also holds the step's other cache and slot bookkeeping:
``build_unified_indices``, ``draft_page_spill``, ``qkv_prologue`` (norm +
RoPE + append) and ``clear_dump_slots`` (dump-state reset of cleared slots).
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi


def append_kv(
    k: torch.Tensor,
    v: torch.Tensor,
    kv_append_indptr: torch.Tensor,
    kv_cache: torch.Tensor,
    kv_page_indices: torch.Tensor,
    kv_page_indptr: torch.Tensor,
    kv_last_page_len: torch.Tensor,
    page_size: int,
    status: torch.Tensor | None = None,
    page_tables: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
) -> None:
    """Writes the step's new K/V rows into their pages (C ABI ``aspire_append_kv``).

    With ``page_tables=(mode_flags, draft_table, block_table)`` and
    ``kv_page_indices=None``, row b's logical page p is read from
    ``draft_table[b, p]`` (mode 0) or ``block_table[b, p]``, as the attention's
    page-table mode does; no flat page list is needed."""
    total_tokens = k.shape[0]
    if total_tokens == 0:
        return
    head_dim = k.shape[2]
    num_heads = k.shape[1]
    if k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError("update_kv_padded requires contiguous k/v head dimensions")
    if k.stride(1) != head_dim or v.stride(1) != head_dim:
        raise ValueError("update_kv_padded requires contiguous k/v heads")
    if kv_cache.stride(-1) != 1:
        raise ValueError("update_kv_padded requires a contiguous cache head dimension")
    if not kv_cache.is_contiguous():
        raise ValueError("aspire_b200 append requires a contiguous [pages, 2, page, heads, dim] cache")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or kv_cache.dtype != torch.bfloat16:
        raise ValueError("aspire_b200 append requires bfloat16 k, v and kv_cache")
    if kv_page_indices is None and page_tables is None:
        raise ValueError("kv_page_indices or page_tables is required")
    checked = [("kv_append_indptr", kv_append_indptr), ("kv_page_indptr", kv_page_indptr),
               ("kv_last_page_len", kv_last_page_len)]
    if kv_page_indices is not None:
        checked.append(("kv_page_indices", kv_page_indices))
    else:
        checked.append(("mode_flags", page_tables[0]))
        for name, t in (("draft_table", page_tables[1]), ("block_table", page_tables[2])):
            if t.dtype != torch.int32 or t.dim() != 2 or t.stride(1) != 1:
                raise ValueError(f"{name} must be a 2-D int32 tensor with contiguous rows")
    for name, t in checked:
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    num_rows = kv_last_page_len.shape[0]
    if kv_append_indptr.shape[0] < num_rows + 1 or kv_page_indptr.shape[0] < num_rows + 1:
        raise ValueError("kv_append_indptr / kv_page_indptr need len(kv_last_page_len) + 1 entries")
    a = _capi.AspireAppendArgs()
    a.k = k.data_ptr()
    a.v = v.data_ptr()
    a.k_stride_n, a.k_stride_h = k.stride(0), k.stride(1)
    a.v_stride_n, a.v_stride_h = v.stride(0), v.stride(1)
    a.num_tokens = total_tokens
    a.append_indptr = kv_append_indptr.data_ptr()
    a.kv_cache = kv_cache.data_ptr()
    a.num_pages_total = kv_cache.shape[0]
    if kv_page_indices is not None:
        a.page_indices = kv_page_indices.data_ptr()
    else:
        a.page_indices = None
        a.mode_flags = page_tables[0].data_ptr()
        a.draft_table = page_tables[1].data_ptr()
        a.draft_stride = page_tables[1].stride(0)
        a.block_table = page_tables[2].data_ptr()
        a.block_table_stride = page_tables[2].stride(0)
    a.page_indptr = kv_page_indptr.data_ptr()
    a.last_page_len = kv_last_page_len.data_ptr()
    a.num_rows = num_rows
    a.num_kv_heads = num_heads
    a.head_dim = head_dim
    a.page_size = int(page_size)
    a.status = status.data_ptr() if status is not None else None
    stream = torch.cuda.current_stream(k.device).cuda_stream
    rc = _capi.load_library().aspire_append_kv(ctypes.byref(a), ctypes.c_void_p(stream))
    _capi.check(rc, "aspire_append_kv")


torch.library.define(
    "aspire_b200::update_kv_padded",
    "(Tensor k, Tensor v, Tensor kv_append_indptr, Tensor(a!) kv_cache, "
    "Tensor kv_page_indices, Tensor kv_page_indptr, Tensor kv_last_page_len, "
    "int page_size) -> ()",
)


@torch.library.impl("aspire_b200::update_kv_padded", "cuda")
def update_kv_padded(k, v, kv_append_indptr, kv_cache, kv_page_indices, kv_page_indptr,
                     kv_last_page_len, page_size):
    append_kv(k, v, kv_append_indptr, kv_cache, kv_page_indices, kv_page_indptr,
              kv_last_page_len, page_size)


@torch.library.register_fake("aspire_b200::update_kv_padded")
def _update_kv_padded_fake(k, v, kv_append_indptr, kv_cache, kv_page_indices, kv_page_indptr,
                           kv_last_page_len, page_size):
    return None


def build_unified_indices(mode_flags: torch.Tensor, draft_indices: torch.Tensor, verify_indices: torch.Tensor,
                          draft_num_pages: torch.Tensor, verify_num_pages: torch.Tensor,
                          paged_kv_indices: torch.Tensor, paged_kv_indptr: torch.Tensor,
                          status: torch.Tensor | None = None) -> None:
    """Drop-in for the reference's build_unified_indices
    (aspire/models/sparse_draft_runner.py:126-153): fills paged_kv_indptr[:B+1]
    and paged_kv_indices with each row's draft-table or block-table prefix
    (mode 0 = draft), in one kernel (C ABI ``aspire_build_unified_indices``)."""
    batch = mode_flags.shape[0]
    tensors = {"mode_flags": mode_flags, "draft_indices": draft_indices, "verify_indices": verify_indices,
               "draft_num_pages": draft_num_pages, "verify_num_pages": verify_num_pages,
               "paged_kv_indices": paged_kv_indices, "paged_kv_indptr": paged_kv_indptr}
    for name, t in tensors.items():
        if t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32, got {t.dtype}")
        if t.device.type != "cuda":
            raise ValueError(f"{name} must be a CUDA tensor")
    if draft_indices.stride(-1) != 1 or verify_indices.stride(-1) != 1:
        raise ValueError("draft / verify tables need contiguous rows")
    if not (mode_flags.is_contiguous() and draft_num_pages.is_contiguous() and verify_num_pages.is_contiguous()
            and paged_kv_indices.is_contiguous() and paged_kv_indptr.is_contiguous()):
        raise ValueError("flags, counts and outputs must be contiguous")
    if paged_kv_indptr.shape[0] < batch + 1 or draft_indices.shape[0] < batch or verify_indices.shape[0] < batch:
        raise ValueError("tables / indptr have fewer rows than mode_flags")
    a = _capi.AspireIndicesArgs()
    a.mode_flags = mode_flags.data_ptr()
    a.draft_indices = draft_indices.data_ptr()
    a.draft_stride = draft_indices.stride(0)
    a.draft_cols = draft_indices.shape[1]
    a.verify_indices = verify_indices.data_ptr()
    a.verify_stride = verify_indices.stride(0)
    a.verify_cols = verify_indices.shape[1]
    a.draft_num_pages = draft_num_pages.data_ptr()
    a.verify_num_pages = verify_num_pages.data_ptr()
    a.batch = batch
    a.indices_out = paged_kv_indices.data_ptr()
    a.indptr_out = paged_kv_indptr.data_ptr()
    a.status = status.data_ptr() if status is not None else None
    a.indices_capacity = paged_kv_indices.numel()
    stream = torch.cuda.current_stream(mode_flags.device).cuda_stream
    rc = _capi.load_library().aspire_build_unified_indices(ctypes.byref(a), ctypes.c_void_p(stream))
    _capi.check(rc, "aspire_build_unified_indices")


def draft_page_spill(mode_flags: torch.Tensor, dec_lens: torch.Tensor, draft_cachelens: torch.Tensor,
                     draft_indices: torch.Tensor, draft_num_pages: torch.Tensor, block_table: torch.Tensor,
                     page_size: int = 16, status: torch.Tensor | None = None) -> None:
    """Draft-page spill insert, in place (C ABI ``aspire_draft_page_spill``):
    a draft row whose newest token opened a new page gets that page
    (``block_table[b, ceil(draft_cachelens[b] / page_size) - 1]``) appended to
    its draft table, unless the table already ends there or is full.  Replaces
    the spill check of LMBackendBase.prepare_forward_inputs
    (aspire/backends/base.py:1222-1236) with _handle_draft_page_spill
    (:718-742): one launch, no host synchronisation, capturable.  All tensors
    are int32 on the GPU; ``dec_lens`` are the step's decode lengths (0 for
    finished rows) and ``draft_cachelens`` count this step's token."""
    batch = mode_flags.shape[0]
    tensors = {"mode_flags": mode_flags, "dec_lens": dec_lens, "draft_cachelens": draft_cachelens,
               "draft_indices": draft_indices, "draft_num_pages": draft_num_pages, "block_table": block_table}
    for name, t in tensors.items():
        if t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32, got {t.dtype}")
        if t.device.type != "cuda":
            raise ValueError(f"{name} must be a CUDA tensor")
    if draft_indices.dim() != 2 or block_table.dim() != 2 or draft_indices.stride(1) != 1 or block_table.stride(1) != 1:
        raise ValueError("draft_indices / block_table must be 2-D with contiguous rows")
    for name in ("mode_flags", "dec_lens", "draft_cachelens", "draft_num_pages"):
        t = tensors[name]
        if not t.is_contiguous() or t.shape[0] < batch:
            raise ValueError(f"{name} must be contiguous with at least batch entries")
    if draft_indices.shape[0] < batch or block_table.shape[0] < batch:
        raise ValueError("tables have fewer rows than mode_flags")
    a = _capi.AspireSpillArgs()
    a.mode_flags = mode_flags.data_ptr()
    a.dec_lens = dec_lens.data_ptr()
    a.draft_cachelens = draft_cachelens.data_ptr()
    a.draft_indices = draft_indices.data_ptr()
    a.draft_stride = draft_indices.stride(0)
    a.draft_cols = draft_indices.shape[1]
    a.draft_num_pages = draft_num_pages.data_ptr()
    a.block_table = block_table.data_ptr()
    a.block_table_stride = block_table.stride(0)
    a.block_table_cols = block_table.shape[1]
    a.batch = batch
    a.page_size = int(page_size)
    a.status = status.data_ptr() if status is not None else None
    stream = torch.cuda.current_stream(mode_flags.device).cuda_stream
    rc = _capi.load_library().aspire_draft_page_spill(ctypes.byref(a), ctypes.c_void_p(stream))
    _capi.check(rc, "aspire_draft_page_spill")


def qkv_prologue(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_append_indptr: torch.Tensor,
                 rope_offsets: torch.Tensor, kv_cache: torch.Tensor, kv_page_indices: torch.Tensor | None,
                 kv_page_indptr: torch.Tensor, kv_last_page_len: torch.Tensor, page_size: int = 16, *,
                 q_norm_weight: torch.Tensor | None = None, k_norm_weight: torch.Tensor | None = None,
                 norm_eps: float = 1e-6, rope_theta: float = 1e4, rope_scale: float = 1.0,
                 llama31: tuple[float, float, float] | None = None, q_out: torch.Tensor | None = None,
                 page_tables: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
                 status: torch.Tensor | None = None) -> torch.Tensor:
    """One launch for a layer's attention prologue (C ABI ``aspire_qkv_prologue``):
    ``q_norm`` / ``k_norm`` with the HF-to-interleaved permutation
    (aspire/models/sparse_draft_transformer.py:150-158) when the norm weights
    are given, the interleaved RoPE of ``mylib::rope`` (FlashInfer
    ``apply_rope_inplace`` or, with ``llama31=(low_freq_factor,
    high_freq_factor, old_context_len)``, ``apply_llama31_rope_inplace``;
    aspire/models/mixed_transformer.py:159-197) at positions
    ``rope_offsets[b] + (t - kv_append_indptr[b])``, and the paged append of
    the rotated k and of v (``mylib::update_kv_padded``).  Returns the rotated
    q (``q_out``, which may be ``q`` itself for the reference's in-place form)."""
    total = q.shape[0]
    if q_out is None:
        q_out = torch.empty_like(q)
    if total == 0:
        return q_out
    for name, t in (("q", q), ("k", k), ("v", v), ("q_out", q_out), ("kv_cache", kv_cache)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bfloat16")
        if t.stride(-1) != 1:
            raise ValueError(f"{name} needs a contiguous head dimension")
    if not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [pages, 2, page, heads, dim] tensor")
    if (q_norm_weight is None) != (k_norm_weight is None):
        raise ValueError("give both norm weights or neither")
    for w in (q_norm_weight, k_norm_weight):
        if w is not None and (w.dtype != torch.bfloat16 or w.numel() != q.shape[2] or not w.is_contiguous()):
            raise ValueError("norm weights must be contiguous bfloat16 [head_dim] tensors")
    ints = [("kv_append_indptr", kv_append_indptr), ("rope_offsets", rope_offsets),
            ("kv_page_indptr", kv_page_indptr), ("kv_last_page_len", kv_last_page_len)]
    if kv_page_indices is not None:
        ints.append(("kv_page_indices", kv_page_indices))
    elif page_tables is None:
        raise ValueError("kv_page_indices or page_tables is required")
    for name, t in ints:
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    num_rows = kv_last_page_len.shape[0]
    if kv_append_indptr.shape[0] < num_rows + 1 or kv_page_indptr.shape[0] < num_rows + 1:
        raise ValueError("kv_append_indptr / kv_page_indptr need len(kv_last_page_len) + 1 entries")
    if rope_offsets.shape[0] < num_rows:
        raise ValueError("rope_offsets needs one entry per row")
    a = _capi.AspirePrologueArgs()
    a.q, a.q_stride_n, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_n, a.k_stride_h = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_n, a.v_stride_h = v.data_ptr(), v.stride(0), v.stride(1)
    a.q_out, a.qo_stride_n, a.qo_stride_h = q_out.data_ptr(), q_out.stride(0), q_out.stride(1)
    a.num_tokens = total
    a.num_qo_heads, a.num_kv_heads, a.head_dim = q.shape[1], k.shape[1], q.shape[2]
    a.q_norm_weight = q_norm_weight.data_ptr() if q_norm_weight is not None else None
    a.k_norm_weight = k_norm_weight.data_ptr() if k_norm_weight is not None else None
    a.norm_eps = float(norm_eps)
    a.rope_offsets = rope_offsets.data_ptr()
    a.rope_theta, a.rope_scale = float(rope_theta), float(rope_scale)
    if llama31 is not None:
        a.low_freq_factor, a.high_freq_factor, a.old_context_len = (float(x) for x in llama31)
    a.append_indptr = kv_append_indptr.data_ptr()
    a.num_rows = num_rows
    a.kv_cache = kv_cache.data_ptr()
    a.num_pages_total = kv_cache.shape[0]
    a.page_size = int(page_size)
    a.page_indptr = kv_page_indptr.data_ptr()
    a.last_page_len = kv_last_page_len.data_ptr()
    if kv_page_indices is not None:
        a.page_indices = kv_page_indices.data_ptr()
    else:
        a.mode_flags = page_tables[0].data_ptr()
        a.draft_table = page_tables[1].data_ptr()
        a.draft_stride = page_tables[1].stride(0)
        a.block_table = page_tables[2].data_ptr()
        a.block_table_stride = page_tables[2].stride(0)
    a.status = status.data_ptr() if status is not None else None
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = _capi.load_library().aspire_qkv_prologue(ctypes.byref(a), ctypes.c_void_p(stream))
    _capi.check(rc, "aspire_qkv_prologue")
    return q_out


def clear_dump_slots(attention_weights_buffer: torch.Tensor, slot_ids: torch.Tensor, num_heads: int,
                     dump_slots: int, kv_stride: int, lse_buffer: torch.Tensor | None = None,
                     qo_indptr: torch.Tensor | None = None, mode_flags: torch.Tensor | None = None,
                     mode_value: int = 1, status: torch.Tensor | None = None) -> None:
    """Dump-state reset of cleared slots in one launch (C ABI
    ``aspire_clear_dump_slots``), replacing
    LMBackendBase._clear_variant_slot_state (aspire/backends/base.py:1404-1419):
    the slots' rows of the flat dump buffer ``[rows, num_heads, dump_slots,
    kv_stride]`` (fp16 or fp32) become -inf, the LSE row of each slot's last
    query (``qo_indptr[slot + 1] - 1``, clamped) becomes 0, and
    ``mode_flags[slot]`` becomes ``mode_value`` (VERIFY_MODE = 1).  Slot ids
    past the buffer's rows are skipped and reported in ``status``."""
    dump = attention_weights_buffer
    if dump.dtype not in (torch.float16, torch.float32) or not dump.is_contiguous() or dump.device.type != "cuda":
        raise ValueError("attention_weights_buffer must be a contiguous fp16 or fp32 CUDA tensor")
    row_elems = int(num_heads) * int(dump_slots) * int(kv_stride)
    if row_elems <= 0 or dump.numel() % row_elems != 0:
        raise ValueError("attention_weights_buffer is not a whole number of [num_heads, slots, kv_stride] rows")
    ids = slot_ids.to(device=dump.device, dtype=torch.int32).contiguous()
    for name, t in (("qo_indptr", qo_indptr), ("mode_flags", mode_flags)):
        if t is not None and (t.dtype != torch.int32 or not t.is_contiguous() or t.device != dump.device):
            raise ValueError(f"{name} must be a contiguous int32 tensor on the dump's device")
    if lse_buffer is not None:
        if (lse_buffer.dtype != torch.float32 or not lse_buffer.is_contiguous() or lse_buffer.dim() != 2
                or lse_buffer.shape[1] != num_heads):
            raise ValueError("lse_buffer must be a contiguous fp32 [tokens, num_heads] tensor")
        if qo_indptr is None:
            raise ValueError("lse_buffer needs qo_indptr")
    a = _capi.AspireClearDumpArgs()
    a.dump = dump.data_ptr()
    a.dump_dtype = _capi.DUMP_F32 if dump.dtype == torch.float32 else _capi.DUMP_F16
    a.num_heads = int(num_heads)
    a.slots = int(dump_slots)
    a.kv_stride = int(kv_stride)
    a.dump_rows = dump.numel() // row_elems
    a.slot_ids = ids.data_ptr()
    a.n_slots = ids.numel()
    if lse_buffer is not None:
        a.lse = lse_buffer.data_ptr()
        a.lse_rows = lse_buffer.shape[0]
        a.qo_indptr = qo_indptr.data_ptr()
        a.qo_len = qo_indptr.numel()
    if mode_flags is not None:
        if mode_flags.numel() < a.dump_rows:
            raise ValueError("mode_flags needs an entry per dump row")
        a.mode_flags = mode_flags.data_ptr()
    a.mode_value = int(mode_value)
    a.status = status.data_ptr() if status is not None else None
    stream = torch.cuda.current_stream(dump.device).cuda_stream
    _capi.check(_capi.load_library().aspire_clear_dump_slots(ctypes.byref(a), ctypes.c_void_p(stream)),
                "aspire_clear_dump_slots")
