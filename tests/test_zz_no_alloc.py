"""The allocation-free attention entry point agrees with the regular one.

aspire_mixed_attention_noalloc serves callers that may not allocate device
memory (a plug-in inside a host application that owns all GPU memory, or a
serving loop whose memory is fixed at start-up).  It keeps its plan and
split-KV partials in arrays built into the library.  This test calls it
through the C ABI twice in a row (the second call runs on the contents the
first left in the shared arrays) and compares each output with the regular
entry point's, which uses caller-owned workspaces.  It lives in its own file,
collected last, and passes on its own in a fresh process too.
"""

import ctypes

import numpy as np
import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.attention import HolisticAttentionWrapper
from aspire_b200.workloads import fill_tensors, make_layout, rows_layout

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

        # Regular entry point (caller-owned workspaces).
        w = HolisticAttentionWrapper(torch.empty(1, device=dev))
        w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                    kv_indices, lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)
        ref_out, ref_lse = w.run(q, kv, return_lse=True)

        # Allocation-free entry point: host-rendered plan, built-in device arrays.
        qo = np.ascontiguousarray(lay.qo_indptr, dtype=np.int32)
        kvp = np.ascontiguousarray(lay.kv_indptr, dtype=np.int32)
        kvl = np.ascontiguousarray(lay.kv_lens, dtype=np.int32)
        host_plan = torch.empty(_capi.NOALLOC_INT_BYTES, dtype=torch.uint8, pin_memory=True)
        info = _capi.AspirePlanInfo()
        i32 = lambda a: a.ctypes.data_as(_capi.c_int32_p)  # noqa: E731
        rc = lib.aspire_plan_host_only(i32(qo), i32(kvp), i32(kvl), lay.batch, lay.num_qo_heads, lay.num_kv_heads,
                                       128, 16, 1, num_sms, ctypes.c_void_p(host_plan.data_ptr()),
                                       host_plan.numel(), _capi.NOALLOC_FLOAT_BYTES, ctypes.byref(info))
        _capi.check(rc, "aspire_plan_host_only")
        assert info.num_merge > 0, "the case must exercise the split-KV partials"
        out = torch.full_like(q, float("nan"))
        lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=dev, dtype=torch.float32)
        args = _attn_args(q, kv, kv_indices, out, lse, lay.num_qo_heads, lay.num_kv_heads)
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args), ctypes.byref(info),
                                                ctypes.c_void_p(host_plan.data_ptr()), ctypes.c_void_p(stream))
        _capi.check(rc, "aspire_mixed_attention_noalloc")
        torch.cuda.synchronize()

        err = (out.float() - ref_out.float()).abs()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, (call, err.max().item())
        fin = torch.isfinite(ref_lse)
        assert torch.equal(torch.isfinite(lse), fin)
        assert (lse[fin] - ref_lse[fin]).abs().max().item() <= 2e-3


def test_noalloc_rejects_oversized_plans(cuda_device):
    lib = _capi.load_library()
    info = _capi.AspirePlanInfo()
    info.int_bytes = _capi.NOALLOC_INT_BYTES  # plus the status block: too large
    info.num_qo_heads, info.num_kv_heads = 32, 8
    host_plan = torch.zeros(16, dtype=torch.uint8)
    args = _capi.AspireAttnArgs()
    rc = lib.aspire_mixed_attention_noalloc(ctypes.byref(args), ctypes.byref(info),
                                            ctypes.c_void_p(host_plan.data_ptr()), None)
    assert rc == _capi.ASPIRE_ERR_CAPACITY
    assert b"plan scratch" in lib.aspire_last_error()
