"""aspire_b200: sm_100a implementation of ASPIRE's unified mixed forward hot path.

Public surface (drop-in for the reference's Python interfaces):

* ``aspire_b200.attention.HolisticAttentionWrapper`` - mixed draft/verify
  paged attention with ``plan`` / ``plan_host`` / ``run``; with the
  reference's dump ``jit_args`` it also writes the first/last logit dump.
* ``aspire_b200.kv_ops.update_kv_padded`` and the torch op
  ``torch.ops.aspire_b200.update_kv_padded`` - paged KV append.
* ``aspire_b200.page_selector.PageSelectorFirstLastAvg`` - fused page
  scoring + top-k re-selection, optionally written in place.

All of it runs through libaspire_b200.so (C ABI in include/aspire_b200.h).
There is no CPU fallback: a missing library or GPU raises.
"""

from ._capi import load_library  # noqa: F401

__all__ = ["load_library"]
