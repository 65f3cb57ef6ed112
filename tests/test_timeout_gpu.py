"""Bounded waits of the tcgen05 attention kernel, made to expire on purpose.

Every mbarrier wait of the kernel gives up after a bound (1 s by default);
the CTA then records ASPIRE_STATUS_TIMEOUT, waits for its own copies and
MMAs in flight (with a fixed 1 s bound), frees its tensor memory and
returns, so the host learns of the problem from the status word and the
context stays usable.  Here the bound is set to 1 ns with
aspire_set_wait_limit_ns, so the first wait of a launch that needs more than
a few hundred polls gives up: the status must show TIMEOUT, the stream must
complete without a CUDA error, and the same wrapper, with the default bound
restored, must then produce the oracle's output with a clean status.  The
decode phase and the prefill phase are each driven to a timeout.
"""

import numpy as np
import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.attention import HolisticAttentionWrapper
from aspire_b200.workloads import fill_tensors, make_layout, rows_layout
from gpu_helpers import assert_attention_close, oracle_attention

pytestmark = pytest.mark.gpu


def _plan(w, lay, dev):
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                torch.from_numpy(lay.kv_indices).to(dev), lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)


@pytest.mark.parametrize("kind", ["decode", "prefill"])
def test_expired_waits_report_timeout_and_leave_the_device_usable(cuda_device, kind):
    dev = cuda_device
    lib = _capi.load_library()
    if kind == "decode":
        lay = make_layout(batch=16, ctx=16384, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5,
                          budget_pages=128, seed=71)
    else:
        lay = rows_layout([512, 300], [4096, 2048], 32, 8, seed=72)
    q, kv = fill_tensors(lay, device=dev, seed=73)
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    _plan(w, lay, dev)
    if kind == "prefill":
        assert w.plan_info.num_items_prefill > 0 and w.plan_info.num_items_tc == 0
    try:
        _capi.check(lib.aspire_set_wait_limit_ns(1), "aspire_set_wait_limit_ns")
        w.clear_device_status()
        w.run(q, kv)
        torch.cuda.synchronize()  # no CUDA error: every CTA stopped and returned
        status = w.device_status()
        assert status & _capi.STATUS_TIMEOUT, f"status {status:#x}: no wait expired"
    finally:
        _capi.check(lib.aspire_set_wait_limit_ns(0), "aspire_set_wait_limit_ns")

    # The device and the wrapper stay usable: plan again, run with the default bound.
    w.clear_device_status()
    _plan(w, lay, dev)
    out, lse = w.run(q, kv, return_lse=True)
    torch.cuda.synchronize()
    assert w.device_status() == 0
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)
    # Plain torch work on the same device still runs.
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum().item()) == float(np.arange(1024).sum())
