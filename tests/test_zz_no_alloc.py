"""The allocation-free attention entry point agrees with the regular one.

aspire_mixed_attention_noalloc serves callers that may not allocate device
memory (a plug-in inside a host application that owns all GPU memory, or a
serving loop whose memory is fixed at start-up).  It keeps its plan and
split-KV partials in arrays built into the library.  These tests call it
through the C ABI several times in a row (each call runs on the contents the
previous one left in the shared arrays) and compare each output with the
regular entry point's, which uses caller-owned workspaces, and with the fp32
oracle; after every call the kernels' status word, read back with
aspire_noalloc_status, must be clear.  They also check the capacity limit of
the built-in partials array from both sides, the status reports of a bad
page id, and that a rejected call leaves the arrays untouched.  The file is
collected last and passes on its own in a fresh process too.
"""

import ctypes

import numpy as np
import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.attention import HolisticAttentionWrapper
from aspire_b200.workloads import fill_tensors, make_layout, rows_layout
from oracle import attention as oracle_attn

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _attn_args(q, kv, kv_indices, out, lse, hq, hkv):
    a = _capi.AspireAttnArgs()
    a.q = q.data_ptr()
    a.q_stride_n, a.q_stride_h = q.stride(0), q.stride(1)
    a.q_rows = q.shape[0]
    a.kv_cache = kv.data_ptr()
    a.num_pages_total = kv.shape[0]
    a.kv_indices = kv_indices.data_ptr()
    a.out = out.data_ptr()
    a.o_stride_n, a.o_stride_h = out.stride(0), out.stride(1)
    a.lse = lse.data_ptr()
    a.dump = None
    a.sm_scale = 0.0
    a.num_qo_heads, a.num_kv_heads = hq, hkv
    a.head_dim, a.page_size = 128, 16
    return a


def _host_plan(lib, lay, num_sms, float_ws_bytes=_capi.NOALLOC_FLOAT_BYTES):
    """Renders the layout's plan on the host into a pinned buffer."""
    qo = np.ascontiguousarray(lay.qo_indptr, dtype=np.int32)
    kvp = np.ascontiguousarray(lay.kv_indptr, dtype=np.int32)
    kvl = np.ascontiguousarray(lay.kv_lens, dtype=np.int32)
    host_plan = torch.empty(_capi.NOALLOC_INT_BYTES, dtype=torch.uint8, pin_memory=True)
    info = _capi.AspirePlanInfo()
    i32 = lambda a: a.ctypes.data_as(_capi.c_int32_p)  # noqa: E731
    rc = lib.aspire_plan_host_only(i32(qo), i32(kvp), i32(kvl), lay.batch, lay.num_qo_heads, lay.num_kv_heads,
                                   128, 16, 1, num_sms, ctypes.c_void_p(host_plan.data_ptr()), host_plan.numel(),
                                   float_ws_bytes, ctypes.byref(info))
    _capi.check(rc, "aspire_plan_host_only")
    return host_plan, info


def _status(lib, dev, clear=False) -> int:
    word = ctypes.c_uint32(0xFFFFFFFF)
    rc = lib.aspire_noalloc_status(ctypes.byref(word), 1 if clear else 0,
                                   ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _capi.check(rc, "aspire_noalloc_status")
    torch.cuda.synchronize()
    return int(word.value)


def _run_noalloc(lib, dev, lay, q, kv, kv_indices, host_plan, info):
    out = torch.full_like(q, float("nan"))
    lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=dev, dtype=torch.float32)
    args = _attn_args(q, kv, kv_indices, out, lse, lay.num_qo_heads, lay.num_kv_heads)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args), ctypes.byref(info),
                                            ctypes.c_void_p(host_plan.data_ptr()), ctypes.c_void_p(stream))
    return rc, out, lse


def _regular(lay, q, kv, kv_indices, dev):
    w = HolisticAttentionWrapper(torch.empty(1, device=dev))
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                kv_indices, lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)
    return w.run(q, kv, return_lse=True)


def _assert_close(out, lse, ref_out, ref_lse):
    err = (out.float() - ref_out.float()).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, err.max().item()
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    assert (lse[fin] - ref_lse[fin]).abs().max().item() <= 2e-3


def test_noalloc_matches_regular_entry_point_twice(cuda_device):
    lib = _capi.load_library()
    dev = cuda_device
    num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    # Rows long enough to be split into chunks, so the built-in partials array is used.
    layouts = [
        make_layout(batch=6, ctx=5000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=40,
                    seed=21),
        make_layout(batch=4, ctx=3000, num_qo_heads=16, num_kv_heads=8, draft_fraction=0.25, budget_pages=24,
                    seed=22),
        # Prefill chunks beside decode rows (the prefill phase of the same launch).
        rows_layout([150, 1, 5, 64], [1000, 1500, 800, 64], 32, 8, seed=23),
    ]
    for call, lay in enumerate(layouts):
        q, kv = fill_tensors(lay, device=dev, seed=30 + call)
        kv_indices = torch.from_numpy(lay.kv_indices).to(dev)
        ref_out, ref_lse = _regular(lay, q, kv, kv_indices, dev)

        host_plan, info = _host_plan(lib, lay, num_sms)
        assert info.num_merge > 0, "the case must exercise the split-KV partials"
        rc, out, lse = _run_noalloc(lib, dev, lay, q, kv, kv_indices, host_plan, info)
        _capi.check(rc, "aspire_mixed_attention_noalloc")
        torch.cuda.synchronize()
        assert _status(lib, dev) == 0, f"call {call}: kernels reported a problem"
        _assert_close(out, lse, ref_out, ref_lse)
        # And against the fp32 oracle, not only the other entry point.
        o_ref, l_ref = oracle_attn.paged_attention(q.float().cpu(), kv.cpu(), lay.qo_indptr, lay.kv_indptr,
                                                   lay.kv_indices, lay.kv_lens, causal=True)
        _assert_close(out.cpu(), lse.cpu(), o_ref, l_ref)


def _near_limit_layouts(lib, num_sms):
    """Two all-verify layouts of the same shape family whose split-KV partials
    need just under and just over the built-in 8 MiB (searched with the host
    planner at this device's SM count)."""
    lim = _capi.NOALLOC_FLOAT_BYTES
    under = over = None
    for ctx in (6000, 5000, 4096, 3000, 2048):
        for b in range(2, 40):
            lay = make_layout(batch=b, ctx=ctx, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.0, seed=40 + b)
            _, info = _host_plan(lib, lay, num_sms, float_ws_bytes=1 << 40)
            fb = int(info.float_bytes)
            if fb <= lim and (under is None or fb > under[1]):
                under = (lay, fb)
            if fb > lim and (over is None or fb < over[1]):
                over = (lay, fb)
    return under, over


def test_noalloc_capacity_boundary(cuda_device):
    lib = _capi.load_library()
    dev = cuda_device
    num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    under, over = _near_limit_layouts(lib, num_sms)
    lim = _capi.NOALLOC_FLOAT_BYTES
    assert under is not None and under[1] >= lim * 0.95, under and under[1]
    assert over is not None and over[1] <= lim * 1.1, over and over[1]

    # Just under the limit: runs, matches the regular entry point, clean status.
    lay = under[0]
    q, kv = fill_tensors(lay, device=dev, seed=50)
    kv_indices = torch.from_numpy(lay.kv_indices).to(dev)
    ref_out, ref_lse = _regular(lay, q, kv, kv_indices, dev)
    host_plan, info = _host_plan(lib, lay, num_sms)
    rc, out, lse = _run_noalloc(lib, dev, lay, q, kv, kv_indices, host_plan, info)
    _capi.check(rc, "aspire_mixed_attention_noalloc")
    torch.cuda.synchronize()
    assert _status(lib, dev) == 0
    _assert_close(out, lse, ref_out, ref_lse)

    # Just over: rejected before anything is launched (output untouched).
    lay = over[0]
    q, kv = fill_tensors(lay, device=dev, seed=51)
    kv_indices = torch.from_numpy(lay.kv_indices).to(dev)
    host_plan, info = _host_plan(lib, lay, num_sms, float_ws_bytes=1 << 40)
    rc, out, lse = _run_noalloc(lib, dev, lay, q, kv, kv_indices, host_plan, info)
    torch.cuda.synchronize()
    assert rc == _capi.ASPIRE_ERR_CAPACITY
    assert b"partials" in lib.aspire_last_error()
    assert bool(torch.isnan(out.float()).all())


def test_noalloc_reports_bad_page_and_rejects_without_touching_the_arrays(cuda_device):
    lib = _capi.load_library()
    dev = cuda_device
    num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    lay = make_layout(batch=4, ctx=3000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=24,
                      seed=60)
    q, kv = fill_tensors(lay, device=dev, seed=60)
    bad = lay.kv_indices.copy()
    bad[lay.kv_indptr[1] + 3] = lay.num_pages_total + 7  # a page id past the cache
    bad_indices = torch.from_numpy(bad).to(dev)
    host_plan, info = _host_plan(lib, lay, num_sms)

    rc, _, _ = _run_noalloc(lib, dev, lay, q, kv, bad_indices, host_plan, info)
    _capi.check(rc, "aspire_mixed_attention_noalloc")
    torch.cuda.synchronize()
    assert _status(lib, dev) & _capi.STATUS_BAD_PAGE

    # Rejected calls change nothing on the device: the status word keeps the
    # previous call's report.
    args_bad = _attn_args(q, kv, bad_indices, torch.empty_like(q), torch.empty(q.shape[0], q.shape[1], device=dev),
                          lay.num_qo_heads, lay.num_kv_heads)
    args_bad.head_dim = 64
    rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args_bad), ctypes.byref(info),
                                            ctypes.c_void_p(host_plan.data_ptr()), None)
    assert rc == _capi.ASPIRE_ERR_INVALID
    dev_plan = _capi.AspirePlanInfo.from_buffer_copy(info)
    dev_plan.on_device = 1
    args_ok = _attn_args(q, kv, bad_indices, torch.empty_like(q), torch.empty(q.shape[0], q.shape[1], device=dev),
                         lay.num_qo_heads, lay.num_kv_heads)
    rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args_ok), ctypes.byref(dev_plan),
                                            ctypes.c_void_p(host_plan.data_ptr()), None)
    assert rc == _capi.ASPIRE_ERR_INVALID and b"aspire_plan_host_only" in lib.aspire_last_error()
    big = _capi.AspirePlanInfo.from_buffer_copy(info)
    big.int_bytes = _capi.NOALLOC_INT_BYTES  # plus the status block: too large
    rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args_ok), ctypes.byref(big),
                                            ctypes.c_void_p(host_plan.data_ptr()), None)
    assert rc == _capi.ASPIRE_ERR_CAPACITY and b"plan scratch" in lib.aspire_last_error()
    assert _status(lib, dev, clear=True) & _capi.STATUS_BAD_PAGE
    assert _status(lib, dev) == 0  # cleared by the read above

    # A clean call after the bad one: correct output, clean status.
    kv_indices = torch.from_numpy(lay.kv_indices).to(dev)
    ref_out, ref_lse = _regular(lay, q, kv, kv_indices, dev)
    rc, out, lse = _run_noalloc(lib, dev, lay, q, kv, kv_indices, host_plan, info)
    _capi.check(rc, "aspire_mixed_attention_noalloc")
    torch.cuda.synchronize()
    assert _status(lib, dev) == 0
    _assert_close(out, lse, ref_out, ref_lse)
