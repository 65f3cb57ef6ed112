"""GPU parity of the mixed page-list build (aspire_build_unified_indices)
against the reference's build_unified_indices (golden fixture, run by the
Triton interpreter) and the CPU oracle."""

import numpy as np
import pytest
import torch

from aspire_b200.kv_ops import build_unified_indices
from oracle import unified_indices as oracle_indices

pytestmark = pytest.mark.gpu


def _run(dev, mode, draft, verify, dn, vn, indices0, indptr0, status=None):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    indices, indptr = t(indices0), t(indptr0)
    build_unified_indices(t(mode), t(draft), t(verify), t(dn), t(vn), indices, indptr, status=status)
    torch.cuda.synchronize()
    return indices.cpu().numpy(), indptr.cpu().numpy()


def test_indices_match_reference_golden(cuda_device, golden_dir):
    g = torch.load(golden_dir / "unified_indices.pt", weights_only=False)
    indices, indptr = _run(cuda_device, *(g[k].numpy() for k in (
        "mode_flags", "draft_indices", "verify_indices", "draft_num_pages", "verify_num_pages",
        "indices_before", "indptr_before")))
    np.testing.assert_array_equal(indptr, g["indptr"].numpy())
    np.testing.assert_array_equal(indices, g["indices"].numpy())


@pytest.mark.parametrize("batch,dcols,vcols", [(1, 8, 64), (64, 128, 2080), (257, 37, 1031), (300, 5, 3)])
def test_indices_random_vs_oracle(cuda_device, batch, dcols, vcols):
    """Random mixed batches, including odd table widths (unaligned rows take
    the scalar path) and batches wider than one CTA's reduction."""
    rng = np.random.default_rng(batch * 7 + dcols)
    mode = rng.integers(0, 2, size=batch).astype(np.int32)
    dn = rng.integers(0, dcols + 1, size=batch).astype(np.int32)
    vn = rng.integers(0, vcols + 1, size=batch).astype(np.int32)
    draft = rng.integers(0, 1 << 20, size=(batch, dcols)).astype(np.int32)
    verify = rng.integers(0, 1 << 20, size=(batch, vcols)).astype(np.int32)
    total = int(np.where(mode == 0, dn, vn).sum())
    indices0 = np.full(total + 33, -5, np.int32)
    indptr0 = np.full(batch + 3, -6, np.int32)
    indices, indptr = _run(cuda_device, mode, draft, verify, dn, vn, indices0, indptr0)
    ei, ep = oracle_indices.build_unified_indices(mode, draft, verify, dn, vn, indices0.copy(), indptr0.copy())
    np.testing.assert_array_equal(indptr, ep)
    np.testing.assert_array_equal(indices, ei)


def test_indices_count_past_table_width_sets_status(cuda_device):
    """A count wider than its table copies the width only and reports BAD_ROW
    (the reference would read past the row)."""
    dev = cuda_device
    mode = np.array([1, 0], np.int32)
    verify = np.arange(8, dtype=np.int32).reshape(1, 8).repeat(2, 0)
    draft = np.arange(100, 104, dtype=np.int32).reshape(1, 4).repeat(2, 0)
    dn = np.array([0, 3], np.int32)
    vn = np.array([10, 0], np.int32)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    indices0 = np.full(16, -1, np.int32)
    indices, indptr = _run(dev, mode, draft, verify, dn, vn, indices0, np.zeros(3, np.int32), status=status)
    from aspire_b200._capi import STATUS_BAD_ROW
    assert int(status.item()) & STATUS_BAD_ROW
    np.testing.assert_array_equal(indptr, [0, 10, 13])
    np.testing.assert_array_equal(indices[:8], np.arange(8))
    np.testing.assert_array_equal(indices[8:10], [-1, -1])
    np.testing.assert_array_equal(indices[10:13], [100, 101, 102])


def test_indices_empty_batch_writes_only_indptr0(cuda_device):
    """As in the reference, an empty batch still sets indptr[0] = 0."""
    e = torch.empty(0, dtype=torch.int32, device=cuda_device)
    indptr = torch.full((2,), 4, dtype=torch.int32, device=cuda_device)
    build_unified_indices(e, e.view(0, 1), e.view(0, 1), e, e, e, indptr)
    assert indptr.tolist() == [0, 4]


def test_indices_stop_at_the_output_capacity(cuda_device):
    """Counts summing past the output buffer (a malformed step) write nothing
    beyond it: the buffer handed over is a view of a larger one, whose guard
    tail must keep its fill; a negative count counts as 0.  Both report
    BAD_ROW; rows that fit are copied as usual."""
    from aspire_b200._capi import STATUS_BAD_ROW

    dev = cuda_device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
    mode = np.array([1, 1, 0, 1], np.int32)
    verify = (np.arange(4 * 16, dtype=np.int32).reshape(4, 16) + 1000)
    draft = (np.arange(4 * 8, dtype=np.int32).reshape(4, 8) + 5000)
    vn = np.array([6, -3, 0, 16], np.int32)
    dn = np.array([0, 0, 8, 0], np.int32)
    backing = torch.full((20 + 64,), -7, dtype=torch.int32, device=dev)
    indices = backing[:20]
    indptr = torch.zeros(5, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    build_unified_indices(t(mode), t(draft), t(verify), t(dn), t(vn), indices, indptr, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & STATUS_BAD_ROW
    # Row 1's -3 counts as 0; row 3 starts at 14 and has room for 6 of its 16.
    assert indptr.tolist() == [0, 6, 6, 14, 30]
    got = backing.cpu().numpy()
    np.testing.assert_array_equal(got[:6], verify[0, :6])
    np.testing.assert_array_equal(got[6:14], draft[2, :8])
    np.testing.assert_array_equal(got[14:20], verify[3, :6])
    assert (got[20:] == -7).all(), "wrote past the output buffer"
