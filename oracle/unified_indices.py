"""CPU restatement of build_unified_indices (test infrastructure).

Follows aspire/models/sparse_draft_runner.py:126-153 and its Triton
_copy_indices_kernel (:93-123): n[b] = draft_num_pages[b] when
mode_flags[b] == 0 (DRAFT_MODE) else verify_num_pages[b];
indptr[0] = 0, indptr[1:B+1] = cumsum(n); row b's n[b] ids are copied from
draft_indices[b, :n] or verify_indices[b, :n] to indices[indptr[b]:].
Entries of indptr past B and of indices past indptr[B] are left as they were.
A count larger than its table's width reads past the row in the reference;
here (as in the sm_100a kernel) only the width is copied and the rest of the
row's span is left untouched.
"""

from __future__ import annotations

import numpy as np


def build_unified_indices(mode_flags, draft_indices, verify_indices, draft_num_pages, verify_num_pages,
                          indices, indptr):
    """Fills ``indices`` and ``indptr`` (numpy int32 arrays) in place."""
    mode = np.asarray(mode_flags)
    n = np.where(mode == 0, np.asarray(draft_num_pages), np.asarray(verify_num_pages)).astype(np.int64)
    batch = mode.shape[0]
    indptr[0] = 0
    indptr[1:batch + 1] = np.cumsum(n)
    for b in range(batch):
        table = draft_indices if mode[b] == 0 else verify_indices
        m = min(int(n[b]), table.shape[1])
        if m > 0:
            start = int(indptr[b])
            indices[start:start + m] = table[b, :m]
    return indices, indptr
