"""ctypes binding of the C ABI declared in include/aspire_b200.h.

The library is loaded from the package directory (built in-tree by
``aspire_b200.build``).  There is no fallback: if the library is missing or
cannot be loaded, importing the ops raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaspire_b200.so"

ASPIRE_OK = 0
ASPIRE_ERR_INVALID = -1
ASPIRE_ERR_CUDA = -2
ASPIRE_ERR_CAPACITY = -3
ASPIRE_ERR_DEVICE = -4

# Built-in workspaces of aspire_mixed_attention_noalloc (include/aspire_b200.h).
NOALLOC_INT_BYTES = 512 * 1024
NOALLOC_FLOAT_BYTES = 8 * 1024 * 1024

STATUS_BAD_PAGE = 1
STATUS_BAD_PLAN = 2
STATUS_BAD_ROW = 4
STATUS_TIMEOUT = 8
DUMP_FIRST_LAST = 0
DUMP_LAST_TOKEN = 1
DUMP_F16 = 0
DUMP_F32 = 1

c_int32_p = ctypes.POINTER(ctypes.c_int32)


class AspirePlanInfo(ctypes.Structure):
    _fields_ = [
        ("num_items", ctypes.c_int32),
        ("num_items_gather", ctypes.c_int32),
        ("num_items_tc", ctypes.c_int32),
        ("num_ctas", ctypes.c_int32),
        ("num_merge", ctypes.c_int32),
        ("chunk_tokens", ctypes.c_int32),
        ("partial_rows", ctypes.c_int64),
        ("int_bytes", ctypes.c_int64),
        ("float_bytes", ctypes.c_int64),
        ("num_qo_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("batch_size", ctypes.c_int32),
        ("max_q_len", ctypes.c_int32),
        ("tc_enabled", ctypes.c_int32),
        ("on_device", ctypes.c_int32),
        ("num_items_prefill", ctypes.c_int32),
    ]


class AspireAttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_n", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("kv_cache", ctypes.c_void_p),
        ("num_pages_total", ctypes.c_int64),
        ("kv_indices", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("o_stride_n", ctypes.c_int64),
        ("o_stride_h", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("dump", ctypes.c_void_p),
        ("dump_num_heads", ctypes.c_int64),
        ("dump_kv_stride", ctypes.c_int64),
        ("sm_scale", ctypes.c_float),
        ("num_qo_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("int_ws", ctypes.c_void_p),
        ("int_ws_bytes", ctypes.c_size_t),
        ("float_ws", ctypes.c_void_p),
        ("float_ws_bytes", ctypes.c_size_t),
        ("q_rows", ctypes.c_int64),
        ("mode_flags", ctypes.c_void_p),
        ("draft_table", ctypes.c_void_p),
        ("draft_stride", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("dump_kind", ctypes.c_int32),
        ("dump_dtype", ctypes.c_int32),
        ("dump_flags", ctypes.c_void_p),
        ("k_new", ctypes.c_void_p),
        ("v_new", ctypes.c_void_p),
        ("k_new_stride_n", ctypes.c_int64),
        ("k_new_stride_h", ctypes.c_int64),
        ("v_new_stride_n", ctypes.c_int64),
        ("v_new_stride_h", ctypes.c_int64),
    ]


class AspireAppendArgs(ctypes.Structure):
    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("k_stride_n", ctypes.c_int64),
        ("k_stride_h", ctypes.c_int64),
        ("v_stride_n", ctypes.c_int64),
        ("v_stride_h", ctypes.c_int64),
        ("num_tokens", ctypes.c_int64),
        ("append_indptr", ctypes.c_void_p),
        ("kv_cache", ctypes.c_void_p),
        ("num_pages_total", ctypes.c_int64),
        ("page_indices", ctypes.c_void_p),
        ("page_indptr", ctypes.c_void_p),
        ("last_page_len", ctypes.c_void_p),
        ("num_rows", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("mode_flags", ctypes.c_void_p),
        ("draft_table", ctypes.c_void_p),
        ("draft_stride", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
    ]


class AspireSelectArgs(ctypes.Structure):
    _fields_ = [
        ("dump", ctypes.c_void_p),
        ("kv_stride", ctypes.c_int64),
        ("max_seq_len", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("lse_rows", ctypes.c_int64),
        ("qo_indptr", ctypes.c_void_p),
        ("row_ids", ctypes.c_void_p),
        ("scores_in", ctypes.c_void_p),
        ("num_pages", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("block_table_cols", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("pages_per_slot", ctypes.c_int32),
        ("L", ctypes.c_int32),
        ("subset_cache_size", ctypes.c_int32),
        ("min_draft_pages", ctypes.c_int32),
        ("draft_percent", ctypes.c_float),
        ("sm_scale", ctypes.c_float),
        ("head_dim", ctypes.c_int32),
        ("table_out", ctypes.c_void_p),
        ("table_stride", ctypes.c_int64),
        ("table_width", ctypes.c_int32),
        ("counts_out", ctypes.c_void_p),
        ("scores_out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("scores_ws", ctypes.c_void_p),
        ("order_by_page", ctypes.c_int32),
        ("dump_kind", ctypes.c_int32),
        ("dump_dtype", ctypes.c_int32),
    ]


class AspireIndicesArgs(ctypes.Structure):
    _fields_ = [
        ("mode_flags", ctypes.c_void_p),
        ("draft_indices", ctypes.c_void_p),
        ("draft_stride", ctypes.c_int64),
        ("draft_cols", ctypes.c_int32),
        ("verify_indices", ctypes.c_void_p),
        ("verify_stride", ctypes.c_int64),
        ("verify_cols", ctypes.c_int32),
        ("draft_num_pages", ctypes.c_void_p),
        ("verify_num_pages", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("indices_out", ctypes.c_void_p),
        ("indptr_out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("indices_capacity", ctypes.c_int64),
    ]


class AspirePrologueArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_n", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("k", ctypes.c_void_p),
        ("k_stride_n", ctypes.c_int64),
        ("k_stride_h", ctypes.c_int64),
        ("v", ctypes.c_void_p),
        ("v_stride_n", ctypes.c_int64),
        ("v_stride_h", ctypes.c_int64),
        ("q_out", ctypes.c_void_p),
        ("qo_stride_n", ctypes.c_int64),
        ("qo_stride_h", ctypes.c_int64),
        ("num_tokens", ctypes.c_int64),
        ("num_qo_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("q_norm_weight", ctypes.c_void_p),
        ("k_norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
        ("rope_offsets", ctypes.c_void_p),
        ("rope_theta", ctypes.c_float),
        ("rope_scale", ctypes.c_float),
        ("low_freq_factor", ctypes.c_float),
        ("high_freq_factor", ctypes.c_float),
        ("old_context_len", ctypes.c_float),
        ("append_indptr", ctypes.c_void_p),
        ("num_rows", ctypes.c_int32),
        ("kv_cache", ctypes.c_void_p),
        ("num_pages_total", ctypes.c_int64),
        ("page_size", ctypes.c_int32),
        ("page_indices", ctypes.c_void_p),
        ("page_indptr", ctypes.c_void_p),
        ("last_page_len", ctypes.c_void_p),
        ("mode_flags", ctypes.c_void_p),
        ("draft_table", ctypes.c_void_p),
        ("draft_stride", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("status", ctypes.c_void_p),
    ]


class AspireSpillArgs(ctypes.Structure):
    _fields_ = [
        ("mode_flags", ctypes.c_void_p),
        ("dec_lens", ctypes.c_void_p),
        ("draft_cachelens", ctypes.c_void_p),
        ("draft_indices", ctypes.c_void_p),
        ("draft_stride", ctypes.c_int64),
        ("draft_cols", ctypes.c_int32),
        ("draft_num_pages", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("block_table_cols", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


class AspireClearDumpArgs(ctypes.Structure):
    _fields_ = [
        ("dump", ctypes.c_void_p),
        ("dump_dtype", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("slots", ctypes.c_int32),
        ("kv_stride", ctypes.c_int64),
        ("dump_rows", ctypes.c_int64),
        ("slot_ids", ctypes.c_void_p),
        ("n_slots", ctypes.c_int32),
        ("lse", ctypes.c_void_p),
        ("lse_rows", ctypes.c_int64),
        ("qo_indptr", ctypes.c_void_p),
        ("qo_len", ctypes.c_int64),
        ("mode_flags", ctypes.c_void_p),
        ("mode_value", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


# Exported symbols and their signatures (must match include/aspire_b200.h).
_SIGNATURES = {
    "aspire_plan": (
        ctypes.c_int,
        [c_int32_p, c_int32_p, c_int32_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
         ctypes.POINTER(AspirePlanInfo)],
    ),
    "aspire_plan_host_only": (
        ctypes.c_int,
        [c_int32_p, c_int32_p, c_int32_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(AspirePlanInfo)],
    ),
    "aspire_mixed_attention": (
        ctypes.c_int,
        [ctypes.POINTER(AspireAttnArgs), ctypes.POINTER(AspirePlanInfo), ctypes.c_void_p],
    ),
    "aspire_mixed_attention_noalloc": (
        ctypes.c_int,
        [ctypes.POINTER(AspireAttnArgs), ctypes.POINTER(AspirePlanInfo), ctypes.c_void_p, ctypes.c_void_p],
    ),
    "aspire_noalloc_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32, ctypes.c_void_p]),
    "aspire_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "aspire_append_kv": (ctypes.c_int, [ctypes.POINTER(AspireAppendArgs), ctypes.c_void_p]),
    "aspire_select_pages": (ctypes.c_int, [ctypes.POINTER(AspireSelectArgs), ctypes.c_void_p]),
    "aspire_build_unified_indices": (ctypes.c_int, [ctypes.POINTER(AspireIndicesArgs), ctypes.c_void_p]),
    "aspire_qkv_prologue": (ctypes.c_int, [ctypes.POINTER(AspirePrologueArgs), ctypes.c_void_p]),
    "aspire_draft_page_spill": (ctypes.c_int, [ctypes.POINTER(AspireSpillArgs), ctypes.c_void_p]),
    "aspire_clear_dump_slots": (ctypes.c_int, [ctypes.POINTER(AspireClearDumpArgs), ctypes.c_void_p]),
    "aspire_plan_device": (
        ctypes.c_int,
        [c_int32_p, c_int32_p, c_int32_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
         ctypes.c_void_p, ctypes.POINTER(AspirePlanInfo)],
    ),
    "aspire_last_error": (ctypes.c_char_p, []),
    "aspire_abi_version": (ctypes.c_int, []),
    "aspire_status_offset": (ctypes.c_size_t, []),
    "aspire_kernel_names": (ctypes.c_char_p, []),
}

EXPECTED_ABI_VERSION = 5

_lib = None
_lock = threading.Lock()


def load_library(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Loads libaspire_b200.so once and binds the exported signatures."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m aspire_b200.build` "
                "(the CUDA library is required; there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(p), mode=ctypes.RTLD_LOCAL)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.aspire_abi_version()
        if version != EXPECTED_ABI_VERSION:
            raise RuntimeError(f"libaspire_b200 ABI version {version}, expected {EXPECTED_ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    """Raises RuntimeError (ValueError for bad arguments) on a nonzero return code."""
    if rc == ASPIRE_OK:
        return
    msg = load_library().aspire_last_error().decode(errors="replace")
    if rc == ASPIRE_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


def status_offset() -> int:
    return int(load_library().aspire_status_offset())


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)
