"""CPU restatement of the dump-state reset of cleared slots (test
infrastructure): LMBackendBase._clear_variant_slot_state
(aspire/backends/base.py:1404-1419), as three torch indexing statements on
CPU tensors:

  dump.view(B, H, slots, kv_stride)[slot_ids] = -inf
  lse[(qo_indptr[slot_ids + 1] - 1).clamp(0, lse_rows - 1)] = 0
  mode_flags[slot_ids] = VERIFY_MODE (1)
"""

from __future__ import annotations

import torch

VERIFY_MODE = 1


def clear_variant_slot_state(dump: torch.Tensor, lse: torch.Tensor, qo_indptr: torch.Tensor,
                             mode_flags: torch.Tensor, slot_ids: torch.Tensor, *, num_heads: int,
                             dump_slots: int, kv_stride: int) -> None:
    """In place on CPU tensors; `dump` is the flat dump buffer."""
    rows = dump.numel() // (num_heads * dump_slots * kv_stride)
    view = dump.view(rows, num_heads, dump_slots, kv_stride)
    ids = slot_ids.long()
    view[ids] = float("-inf")
    old_lse_rows = (qo_indptr[ids + 1].long() - 1).clamp(min=0, max=lse.shape[0] - 1)
    lse[old_lse_rows] = 0
    mode_flags[ids] = VERIFY_MODE
