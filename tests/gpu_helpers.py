"""Shared helpers of the GPU parity tests (drive the product through its C ABI
wrappers; the oracle is only used as the checker)."""

from __future__ import annotations

import torch

from aspire_b200.attention import HolisticAttentionWrapper, dump_jit_args
from aspire_b200.workloads import MixedLayout, fill_tensors
from oracle import attention as oracle_attn

# Tolerances of the north star: bf16 output vs the fp32 oracle.
MAX_ABS = 2e-2
MEAN_ABS = 2e-3
LSE_ATOL = 2e-3


def _slots(kind: str) -> int:
    return 2 if kind == "first_last_compact" else 1


def run_attention(layout: MixedLayout, q: torch.Tensor, kv: torch.Tensor, *, dump: bool = False,
                  dump_stride: int = 0, wrapper: HolisticAttentionWrapper | None = None, causal: bool = True,
                  dump_kind: str = "first_last_compact", dump_dtype: torch.dtype = torch.float16,
                  dump_flags: torch.Tensor | None = None):
    dev = q.device
    if wrapper is None:
        jit = dump_jit_args(dump_kind, use_mode_flags=dump_flags is not None, dump_buffer_dtype=dump_dtype)
        wrapper = HolisticAttentionWrapper(torch.empty(1, device=dev), jit_args=jit if dump else None)
    kv_indices = torch.from_numpy(layout.kv_indices).to(dev)
    wrapper.plan_host(torch.from_numpy(layout.qo_indptr), torch.from_numpy(layout.kv_indptr),
                      torch.from_numpy(layout.kv_lens), kv_indices, layout.num_qo_heads, layout.num_kv_heads,
                      128, 16, causal=causal)
    dump_buf = None
    args = []
    if dump:
        dump_buf = torch.full((layout.batch * layout.num_qo_heads * _slots(dump_kind) * dump_stride,),
                              float("-inf"), dtype=dump_dtype, device=dev)
        flags = [dump_flags.to(dev)] if dump_flags is not None else []
        args = [dump_buf, *flags, layout.num_qo_heads, dump_stride]
    out, lse = wrapper.run(q, kv, *args, return_lse=True)
    return out, lse, dump_buf, wrapper


def oracle_attention(layout: MixedLayout, q: torch.Tensor, kv: torch.Tensor, *, dump_stride: int = 0,
                     causal: bool = True, dump_kind: str = "first_last_compact",
                     dump_dtype: torch.dtype = torch.float16, dump_flags: torch.Tensor | None = None):
    dump = None
    if dump_stride:
        dump = torch.full((layout.batch * layout.num_qo_heads * _slots(dump_kind) * dump_stride,), float("-inf"),
                          dtype=dump_dtype)
    out, lse = oracle_attn.paged_attention(
        q.float().cpu(), kv.cpu(), layout.qo_indptr, layout.kv_indptr, layout.kv_indices, layout.kv_lens,
        causal=causal, dump=dump, dump_num_heads=layout.num_qo_heads, dump_kv_stride=dump_stride,
        dump_kind=dump_kind, dump_flags=dump_flags)
    return out, lse, dump


def assert_attention_close(out, lse, ref_out, ref_lse, rows=None):
    o = out.float().cpu()
    if rows is not None:
        o, ref_out = o[rows], ref_out[rows]
        lse, ref_lse = lse[rows], ref_lse[rows]
    err = (o - ref_out).abs()
    assert err.max().item() <= MAX_ABS, f"max-abs {err.max().item():.3e}"
    assert err.mean().item() <= MEAN_ABS, f"mean-abs {err.mean().item():.3e}"
    l, r = lse.float().cpu(), ref_lse
    fin = torch.isfinite(r)
    assert torch.equal(torch.isfinite(l), fin), "LSE finiteness differs"
    if fin.any():
        d = (l[fin] - r[fin]).abs().max().item()
        assert d <= LSE_ATOL, f"lse max-abs {d:.3e}"


def assert_dump_close(dump, ref_dump, layout: MixedLayout, stride: int, *, dump_kind: str = "first_last_compact",
                      dump_flags: torch.Tensor | None = None):
    """Dumps agree to one fp16 rounding step on every written position (the
    values are fp16-rounded in an fp32 buffer too); positions past kv_len,
    unwritten slots and rows whose flag is 0 keep their -inf fill."""
    S = _slots(dump_kind)
    d = dump.cpu().view(layout.batch, layout.num_qo_heads, S, stride).float()
    r = ref_dump.view(layout.batch, layout.num_qo_heads, S, stride).float()
    if dump.dtype == torch.float32:
        assert torch.equal(d, d.half().float()), "fp32 dump holds values that are not fp16-rounded"
    for b in range(layout.batch):
        if dump_flags is not None and int(dump_flags[b]) == 0:
            assert bool(torch.isinf(d[b]).all()), f"row {b} is flagged off but was written"
            continue
        L = int(layout.kv_lens[b])
        written = [0] + ([1] if S == 2 and int(layout.q_lens[b]) > 1 else [])
        for s in written:
            a, e = d[b, :, s, :L], r[b, :, s, :L]
            tol = e.abs() * 2.0 ** -10 + 2.0 ** -14 + 2e-3
            assert bool(((a - e).abs() <= tol).all()), f"dump row {b} slot {s}"
        # Positions past kv_len and unwritten slots keep their previous contents.
        assert bool(torch.isinf(d[b, :, :, L:]).all())
        if S == 2 and int(layout.q_lens[b]) == 1:
            assert bool(torch.isinf(d[b, :, 1, :]).all())


def make_inputs(layout: MixedLayout, device, seed: int = 0):
    return fill_tensors(layout, device=device, dtype=torch.bfloat16, seed=seed)
