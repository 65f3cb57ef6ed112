"""Drop-in replacement for ASPIRE's ``HolisticAttentionWrapper``.

Same constructor, ``plan``, ``plan_host`` and ``run`` surface as
``aspire/attention/holistic_wrapper.py:135-386``; the work is done by
libaspire_b200 (host planner + sm_100a kernels) through its C ABI.

* ``plan`` reads the device indptr / last-page-len arrays back behind a
  stream synchronisation (as the reference does, ``holistic_wrapper.py:237-243``)
  and then plans like ``plan_host``.
* ``plan_host`` takes host ``qo_indptr`` / ``kv_indptr`` / ``kv_len`` arrays,
  renders the work list into one slot of a 4-deep pinned ring and enqueues
  its upload on the current stream; slot reuse is fenced by CUDA events
  (``holistic_wrapper.py:317-342``).
* ``run`` launches the kernels on the current stream.  It allocates nothing
  when ``out`` is given and returns a fresh ``lse`` tensor otherwise (as the
  reference).  Every plan-dependent quantity lives in the device int
  workspace, so ``run`` can be captured in a CUDA graph and replayed after
  later plans.

With ``jit_args`` (the reference's dump-variant JIT arguments,
``holistic_wrapper.py:401-434``) the wrapper runs the first/last logit dump
variant: ``run(q, kv_cache, dump_buffer, num_heads, kv_stride, ...)`` as
``LMBackendBase._register_dump_kernel_op`` calls it (``base.py:461-489``).
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Tuple, Union

import torch

from . import _capi

FLOAT_WORKSPACE_BYTES = 128 * 1024 * 1024
INT_WORKSPACE_BYTES = 8 * 1024 * 1024
PINNED_RING_DEPTH = 4

_WRAPPER_REGISTRY: dict[int, "HolisticAttentionWrapper"] = {}


def _i32_host(t) -> torch.Tensor:
    if isinstance(t, torch.Tensor):
        t = t.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        return t.to(torch.int32).contiguous()
    return torch.as_tensor(t, dtype=torch.int32).contiguous()


def _ptr_i32(t: torch.Tensor):
    return ctypes.cast(ctypes.c_void_p(t.data_ptr()), _capi.c_int32_p)


def _unpack_paged_kv_cache(
    paged_kv_cache: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]], kv_layout: str
) -> torch.Tensor:
    if kv_layout != "NHD":
        raise ValueError(f"aspire_b200 supports the NHD paged layout only, got {kv_layout!r}")
    if isinstance(paged_kv_cache, (tuple, list)):
        raise ValueError("pass the unified [pages, 2, page_size, num_kv_heads, head_dim] cache tensor")
    if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2:
        raise ValueError(
            f"paged_kv_cache must be [pages, 2, page_size, num_kv_heads, head_dim], got {tuple(paged_kv_cache.shape)}"
        )
    if not paged_kv_cache.is_contiguous():
        raise ValueError("paged_kv_cache must be contiguous")
    return paged_kv_cache


def _dump_kind_from_jit_args(jit_args) -> Tuple[str, bool, Optional[torch.dtype]]:
    """Recovers (dump_kind, uses_mode_flags, dump buffer dtype) from the
    reference's JIT argument list (build_holistic_dump_jit_args,
    aspire/attention/holistic_wrapper.py:401-434: tensor names at [7], their
    C types at [8], the struct source at [12])."""
    tensor_names = list(jit_args[7]) if len(jit_args) > 7 else []
    tensor_types = list(jit_args[8]) if len(jit_args) > 8 else []
    code = str(jit_args[12]) if len(jit_args) > 12 else ""
    uses_mode_flags = "mode_flags" in tensor_names
    dtype = {"half": torch.float16, "float": torch.float32}.get(str(tensor_types[0]) if tensor_types else "")
    if "qo_slot" in code:
        return "first_last_compact", uses_mode_flags, dtype
    if "attn_weights[" in code:
        return "last_token", uses_mode_flags, dtype
    return "noop", False, None


class HolisticAttentionWrapper:
    """Mixed draft/verify paged attention over libaspire_b200."""

    def __init__(
        self,
        float_workspace_buffer: torch.Tensor,
        kv_layout: str = "NHD",
        use_cuda_graph: bool = False,
        qo_indptr_buf: Optional[torch.Tensor] = None,
        paged_kv_indptr_buf: Optional[torch.Tensor] = None,
        paged_kv_indices_buf: Optional[torch.Tensor] = None,
        paged_kv_last_page_len_buf: Optional[torch.Tensor] = None,
        jit_args: Optional[list] = None,
        jit_kwargs: Optional[dict] = None,
        float_workspace_bytes: int = FLOAT_WORKSPACE_BYTES,
        int_workspace_bytes: int = INT_WORKSPACE_BYTES,
        num_sms: Optional[int] = None,
        **_ignored,
    ):
        self._lib = _capi.load_library()
        self._kv_layout = kv_layout
        device = float_workspace_buffer.device
        if device.type != "cuda":
            raise RuntimeError("HolisticAttentionWrapper needs a CUDA device (no CPU fallback)")
        self._device = device
        self._float_workspace = torch.empty(float_workspace_bytes, dtype=torch.uint8, device=device)
        self._int_workspace = torch.zeros(int_workspace_bytes, dtype=torch.uint8, device=device)
        self._pinned_ring = [
            torch.empty(int_workspace_bytes, dtype=torch.uint8, pin_memory=True)
            for _ in range(PINNED_RING_DEPTH)
        ]
        self._pinned_ring_events: List[Optional[torch.cuda.Event]] = [None] * PINNED_RING_DEPTH
        self._pinned_slot = 0
        if num_sms is None:
            num_sms = torch.cuda.get_device_properties(device).multi_processor_count
        self._num_sms = int(num_sms)

        self._dump_kind = "noop"
        self._dump_mode_flags = False
        self._dump_dtype: Optional[torch.dtype] = None
        if jit_args is not None:
            self._dump_kind, self._dump_mode_flags, self._dump_dtype = _dump_kind_from_jit_args(jit_args)
        self._has_jit = jit_args is not None

        self._plan_info: Optional[_capi.AspirePlanInfo] = None
        self._kv_indices: Optional[torch.Tensor] = None
        self._page_tables: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None
        self._page_size = 0
        self._sm_scale: Optional[float] = None
        self._causal = False
        self._num_qo_heads = 0
        self._num_kv_heads = 0
        self._id = id(self)
        _WRAPPER_REGISTRY[self._id] = self

    # ------------------------------------------------------------ page tables
    def set_page_tables(self, mode_flags: Optional[torch.Tensor], draft_table: Optional[torch.Tensor] = None,
                        block_table: Optional[torch.Tensor] = None) -> None:
        """Lets run() read each row's pages straight from the engine's tables
        instead of a flat page list: row b's logical page p is
        ``draft_table[b, p]`` when ``mode_flags[b] == 0`` (draft row) and
        ``block_table[b, p]`` otherwise.  This absorbs ``build_unified_indices``
        (aspire/models/sparse_draft_runner.py:126-153) into the attention; a
        plan's ``paged_kv_indices`` may then be None.  The tensors must stay
        allocated (CUDA graphs capture their addresses).  ``None`` turns the
        tables off."""
        if mode_flags is None:
            self._page_tables = None
            return
        for name, t in (("mode_flags", mode_flags), ("draft_table", draft_table), ("block_table", block_table)):
            if t is None or t.dtype != torch.int32 or t.device.type != "cuda":
                raise ValueError(f"{name} must be an int32 CUDA tensor")
        if draft_table.dim() != 2 or block_table.dim() != 2 or draft_table.stride(1) != 1 or block_table.stride(1) != 1:
            raise ValueError("draft_table / block_table must be 2-D with contiguous rows")
        if not mode_flags.is_contiguous():
            raise ValueError("mode_flags must be contiguous")
        self._page_tables = (mode_flags, draft_table, block_table)

    # ------------------------------------------------------------------ plan
    def plan(
        self,
        qo_indptr: torch.Tensor,
        paged_kv_indptr: torch.Tensor,
        paged_kv_indices: Optional[torch.Tensor],
        paged_kv_last_page_len: torch.Tensor,
        num_qo_heads: int,
        num_kv_heads: int,
        head_dim_qk: int,
        page_size: int,
        head_dim_vo: Optional[int] = None,
        q_data_type: Union[str, torch.dtype] = "float16",
        causal: bool = False,
        sm_scale: Optional[float] = None,
        **kwargs,
    ) -> None:
        """Plans from device arrays (reads them back behind a stream sync)."""
        pages = paged_kv_indptr[1:] - paged_kv_indptr[:-1]
        n = paged_kv_last_page_len.shape[0]
        kv_len = torch.clamp(pages[:n] - 1, min=0) * page_size + paged_kv_last_page_len
        qo_host = qo_indptr.to("cpu", non_blocking=True)
        kvp_host = paged_kv_indptr.to("cpu", non_blocking=True)
        kvl_host = kv_len.to("cpu", non_blocking=True)
        torch.cuda.current_stream().synchronize()
        self.plan_host(
            qo_host, kvp_host, kvl_host, paged_kv_indices, num_qo_heads, num_kv_heads,
            head_dim_qk, page_size, head_dim_vo=head_dim_vo, causal=causal, sm_scale=sm_scale,
        )

    def plan_host(
        self,
        qo_indptr_host: torch.Tensor,
        kv_indptr_host: torch.Tensor,
        kv_len_host: torch.Tensor,
        paged_kv_indices: Optional[torch.Tensor],
        num_qo_heads: int,
        num_kv_heads: int,
        head_dim_qk: int,
        page_size: int,
        head_dim_vo: Optional[int] = None,
        causal: bool = False,
        sm_scale: Optional[float] = None,
    ) -> None:
        """Plans from host arrays with no device readback or synchronisation."""
        if head_dim_vo is not None and head_dim_vo != head_dim_qk:
            raise ValueError("head_dim_vo must equal head_dim_qk")
        if paged_kv_indices is None and self._page_tables is None:
            raise ValueError("paged_kv_indices is required unless set_page_tables() was called")
        qo = _i32_host(qo_indptr_host)
        kvp = _i32_host(kv_indptr_host)
        kvl = _i32_host(kv_len_host)
        batch = int(kvl.shape[0])
        if qo.shape[0] < batch + 1 or kvp.shape[0] < batch + 1:
            raise ValueError("qo_indptr / kv_indptr need batch_size + 1 entries")

        slot = self._pinned_slot
        event = self._pinned_ring_events[slot]
        if event is not None:
            event.synchronize()
        buf = self._pinned_ring[slot]
        info = _capi.AspirePlanInfo()
        stream = torch.cuda.current_stream(self._device).cuda_stream
        rc = self._lib.aspire_plan(
            _ptr_i32(qo), _ptr_i32(kvp), _ptr_i32(kvl), batch, int(num_qo_heads), int(num_kv_heads),
            int(head_dim_qk), int(page_size), 1 if causal else 0, self._num_sms,
            ctypes.c_void_p(buf.data_ptr()), buf.numel(),
            ctypes.c_void_p(self._int_workspace.data_ptr()), self._int_workspace.numel(),
            self._float_workspace.numel(), ctypes.c_void_p(stream), ctypes.byref(info),
        )
        _capi.check(rc, "aspire_plan")
        if event is None:
            event = torch.cuda.Event()
            self._pinned_ring_events[slot] = event
        event.record(torch.cuda.current_stream(self._device))
        self._pinned_slot = (slot + 1) % PINNED_RING_DEPTH

        self._plan_info = info
        self._plan_q_total = int(qo[batch])
        self._plan_max_kv_len = int(kvl.max()) if batch else 0
        self._plan_rows = batch
        self._kv_indices = paged_kv_indices
        self._page_size = int(page_size)
        self._sm_scale = sm_scale
        self._causal = bool(causal)
        self._num_qo_heads = int(num_qo_heads)
        self._num_kv_heads = int(num_kv_heads)

    def plan_device(
        self,
        qo_indptr: torch.Tensor,
        paged_kv_indptr: torch.Tensor,
        paged_kv_last_page_len: torch.Tensor,
        num_qo_heads: int,
        num_kv_heads: int,
        head_dim_qk: int,
        page_size: int,
        paged_kv_indices: Optional[torch.Tensor] = None,
        causal: bool = False,
        sm_scale: Optional[float] = None,
        batch_size: Optional[int] = None,
    ) -> None:
        """Plans on the device from device arrays (C ABI ``aspire_plan_device``):
        no readback and no synchronisation, so the call can be captured in a
        CUDA graph with the step and re-plans on every replay from whatever the
        arrays then hold.  Replaces the per-step host planning of
        ``plan`` / ``plan_host`` (aspire/attention/holistic_wrapper.py:200-342).
        Row b attends ``max(pages_b - 1, 0) * page_size + last_page_len[b]``
        tokens.  Problems found on the device (a malformed row, a plan beyond
        the workspaces) are reported in ``device_status()`` and the program
        then writes nothing."""
        batch = int(paged_kv_last_page_len.shape[0] if batch_size is None else batch_size)
        for name, t in (("qo_indptr", qo_indptr), ("paged_kv_indptr", paged_kv_indptr),
                        ("paged_kv_last_page_len", paged_kv_last_page_len)):
            if t.dtype != torch.int32 or not t.is_contiguous() or t.device.type != "cuda":
                raise ValueError(f"{name} must be a contiguous int32 CUDA tensor")
        if qo_indptr.shape[0] < batch + 1 or paged_kv_indptr.shape[0] < batch + 1 or \
                paged_kv_last_page_len.shape[0] < batch:
            raise ValueError("qo_indptr / paged_kv_indptr need batch_size + 1 entries")
        if paged_kv_indices is None and self._page_tables is None:
            raise ValueError("paged_kv_indices is required unless set_page_tables() was called")
        info = _capi.AspirePlanInfo()
        stream = torch.cuda.current_stream(self._device).cuda_stream
        rc = self._lib.aspire_plan_device(
            _dev_i32(qo_indptr), _dev_i32(paged_kv_indptr), _dev_i32(paged_kv_last_page_len), batch, int(num_qo_heads), int(num_kv_heads),
            int(head_dim_qk), int(page_size), 1 if causal else 0, self._num_sms,
            ctypes.c_void_p(self._int_workspace.data_ptr()), self._int_workspace.numel(),
            self._float_workspace.numel(), ctypes.c_void_p(stream), ctypes.byref(info),
        )
        _capi.check(rc, "aspire_plan_device")
        self._plan_info = info
        self._plan_q_total = 0      # checked on the device: rows past q are skipped
        self._plan_max_kv_len = 0   # checked on the device: dump writes past kv_stride are skipped
        self._plan_rows = batch
        self._kv_indices = paged_kv_indices
        self._page_size = int(page_size)
        self._sm_scale = sm_scale
        self._causal = bool(causal)
        self._num_qo_heads = int(num_qo_heads)
        self._num_kv_heads = int(num_kv_heads)

    @property
    def plan_info(self) -> Optional[_capi.AspirePlanInfo]:
        return self._plan_info

    # ------------------------------------------------------------------- run
    def run(
        self,
        q: torch.Tensor,
        paged_kv_cache: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]],
        *args,
        out: Optional[torch.Tensor] = None,
        return_lse: bool = False,
        lse: Optional[torch.Tensor] = None,
        append: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
        **kwargs,
    ) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
        """Runs the planned program.  ``append=(k_new, v_new)`` (bf16
        [tokens, num_kv_heads, 128], the queries' own keys and values) also
        writes each row's new tokens into the cache before the row's keys are
        read, as ``append_kv`` with the same qo_indptr and page source would
        (one launch instead of two); host plans of tcgen05 decode rows only."""
        if self._plan_info is None:
            raise RuntimeError("run() before plan()/plan_host()")
        kv = _unpack_paged_kv_cache(paged_kv_cache, self._kv_layout)
        if q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
            raise ValueError("q and paged_kv_cache must be bfloat16")
        if q.dim() != 3 or q.shape[1] != self._num_qo_heads or q.shape[2] != kv.shape[4]:
            raise ValueError(f"q shape {tuple(q.shape)} does not match the plan")
        if q.stride(2) != 1:
            raise ValueError("q head_dim must be contiguous")
        if kv.shape[2] != self._page_size or kv.shape[3] != self._num_kv_heads:
            raise ValueError("paged_kv_cache geometry does not match the plan")
        if q.shape[0] < self._plan_q_total:
            raise ValueError(f"q has {q.shape[0]} rows but the plan addresses {self._plan_q_total}")
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        if out.stride(2) != 1 or out.shape != q.shape:
            raise ValueError("out must match q's shape with a contiguous head_dim")
        want_lse = return_lse or lse is not None
        if want_lse and lse is None:
            lse = torch.empty(q.shape[0], q.shape[1], device=q.device, dtype=torch.float32)
        if lse is not None and (lse.dtype != torch.float32 or not lse.is_contiguous()
                                or tuple(lse.shape) != (q.shape[0], q.shape[1])):
            raise ValueError("lse must be a contiguous fp32 [tokens, num_qo_heads] tensor")

        # Dump variants take run(q, kv, dump_buffer, [mode_flags,] num_heads,
        # kv_stride): the struct's tensors, then its scalars
        # (holistic_wrapper.py:411-416, base.py:468-473).
        dump = None
        dump_flags = None
        dump_heads = 0
        dump_stride = 0
        if self._has_jit and self._dump_kind != "noop":
            n_t = 2 if self._dump_mode_flags else 1
            if len(args) < n_t + 2:
                raise ValueError("dump variant run(q, kv, dump_buffer, " + ("mode_flags, " if n_t == 2 else "")
                                 + "num_heads, kv_stride)")
            dump = args[0]
            dump_flags = args[1] if n_t == 2 else None
            dump_heads = int(args[n_t])
            dump_stride = int(args[n_t + 1])
            if dump.dtype not in (torch.float16, torch.float32) or not dump.is_contiguous():
                raise ValueError("dump buffer must be a contiguous float16 or float32 tensor")
            if self._dump_dtype is not None and dump.dtype != self._dump_dtype:
                raise ValueError(f"dump buffer is {dump.dtype}, the dump variant writes {self._dump_dtype}")
            if dump_heads < self._num_qo_heads or dump_stride < self._plan_max_kv_len:
                raise ValueError("dump buffer heads/stride smaller than the planned heads/kv_len")
            slots = 2 if self._dump_kind == "first_last_compact" else 1
            if dump.numel() < self._plan_rows * dump_heads * slots * dump_stride:
                raise ValueError(f"dump buffer smaller than rows * num_heads * {slots} * kv_stride")
            if dump_flags is not None and (dump_flags.dtype != torch.int32 or not dump_flags.is_contiguous()
                                           or dump_flags.device != dump.device
                                           or dump_flags.numel() < self._plan_rows):
                raise ValueError("mode_flags must be a contiguous int32 tensor with one entry per row")

        sm_scale = self._sm_scale if self._sm_scale is not None else 1.0 / math.sqrt(q.shape[2])
        a = _capi.AspireAttnArgs()
        a.q = q.data_ptr()
        a.q_stride_n = q.stride(0)
        a.q_stride_h = q.stride(1)
        a.q_rows = q.shape[0]
        a.kv_cache = kv.data_ptr()
        a.num_pages_total = kv.shape[0]
        if self._kv_indices is not None and self._page_tables is None:
            a.kv_indices = self._kv_indices.data_ptr()
        else:
            if self._page_tables is None:
                raise RuntimeError("no page list: plan with paged_kv_indices or call set_page_tables()")
            mode_flags, draft_table, block_table = self._page_tables
            a.kv_indices = None
            a.mode_flags = mode_flags.data_ptr()
            a.draft_table = draft_table.data_ptr()
            a.draft_stride = draft_table.stride(0)
            a.block_table = block_table.data_ptr()
            a.block_table_stride = block_table.stride(0)
        a.out = out.data_ptr()
        a.o_stride_n = out.stride(0)
        a.o_stride_h = out.stride(1)
        a.lse = lse.data_ptr() if lse is not None else None
        a.dump = dump.data_ptr() if dump is not None else None
        a.dump_num_heads = dump_heads
        a.dump_kv_stride = dump_stride
        if append is not None:
            k_new, v_new = append
            for name, t in (("k_new", k_new), ("v_new", v_new)):
                if t.dtype != torch.bfloat16 or t.dim() != 3 or t.stride(2) != 1 or t.device != q.device:
                    raise ValueError(f"{name} must be a bf16 [tokens, num_kv_heads, 128] tensor on q's device")
                if t.shape[1] != self._num_kv_heads or t.shape[2] != q.shape[2] or t.shape[0] < q.shape[0]:
                    raise ValueError(f"{name} shape {tuple(t.shape)} does not match the plan")
            a.k_new, a.v_new = k_new.data_ptr(), v_new.data_ptr()
            a.k_new_stride_n, a.k_new_stride_h = k_new.stride(0), k_new.stride(1)
            a.v_new_stride_n, a.v_new_stride_h = v_new.stride(0), v_new.stride(1)
        a.dump_kind = _capi.DUMP_LAST_TOKEN if self._dump_kind == "last_token" else _capi.DUMP_FIRST_LAST
        a.dump_dtype = _capi.DUMP_F32 if dump is not None and dump.dtype == torch.float32 else _capi.DUMP_F16
        a.dump_flags = dump_flags.data_ptr() if dump_flags is not None else None
        a.sm_scale = float(sm_scale)
        a.num_qo_heads = self._num_qo_heads
        a.num_kv_heads = self._num_kv_heads
        a.head_dim = q.shape[2]
        a.page_size = self._page_size
        a.int_ws = self._int_workspace.data_ptr()
        a.int_ws_bytes = self._int_workspace.numel()
        a.float_ws = self._float_workspace.data_ptr()
        a.float_ws_bytes = self._float_workspace.numel()
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = self._lib.aspire_mixed_attention(ctypes.byref(a), ctypes.byref(self._plan_info),
                                              ctypes.c_void_p(stream))
        _capi.check(rc, "aspire_mixed_attention")
        if return_lse:
            return out, lse
        return out

    # ------------------------------------------------------------- diagnostics
    def device_status(self) -> int:
        """Reads the device status word (synchronises; debug use only)."""
        word = self._int_workspace[:4].view(torch.int32)
        return int(word.item())

    def clear_device_status(self) -> None:
        self._int_workspace[:4].zero_()


def _dev_i32(t: torch.Tensor):
    """Device address of an int32 tensor as the C ABI's int32 pointer."""
    return ctypes.cast(ctypes.c_void_p(t.data_ptr()), _capi.c_int32_p)


def wrapper_from_id(wrapper_id: int) -> HolisticAttentionWrapper:
    return _WRAPPER_REGISTRY[wrapper_id]


def dump_jit_args(dump_kind: str = "first_last_compact", head_dim: int = 128, use_mode_flags: bool = False,
                  dump_buffer_dtype: torch.dtype = torch.float16) -> list:
    """JIT-argument list with the layout of the reference's
    ``build_holistic_dump_jit_args(dtype, head_dim, dump_kind, ...,
    use_mode_flags, dump_buffer_dtype)`` (aspire/attention/holistic_wrapper.py:
    401-434), for callers that do not import the reference's builder.  Only
    the tensor names and types and the marker of the dump kind in the source
    slot are read."""
    if dump_kind not in ("noop", "last_token", "first_last_compact"):
        raise ValueError(f"unknown dump_kind {dump_kind!r}")
    attn_type = {torch.float16: "half", torch.float32: "float"}[dump_buffer_dtype]
    names, types = ["attention_weights"], [attn_type]
    if use_mode_flags and dump_kind != "noop":
        names.append("mode_flags")
        types.append("int32_t")
    marker = {"noop": "noop", "last_token": "last_token: attn_weights[...] = logits",
              "first_last_compact": "first_last_compact: qo_slot = (qo_idx == 0u) ? 0u : 1u"}[dump_kind]
    return [
        "holistic_batch_dump_attention_weights_" + dump_kind.replace("_", ""), torch.bfloat16, torch.bfloat16,
        torch.bfloat16, torch.int32, head_dim, head_dim, names, types,
        ["num_heads", "jit_kv_stride"], ["int64_t", "int64_t"], "HolisticDumpAttentionWeights", marker,
    ]


def first_last_dump_jit_args(head_dim: int = 128) -> list:
    """``dump_jit_args("first_last_compact", head_dim)``: the ASPIRE backend's
    fp16 first/last dump."""
    return dump_jit_args("first_last_compact", head_dim)
