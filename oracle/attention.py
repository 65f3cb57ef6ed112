"""fp32 CPU restatement of the paged mixed attention (test infrastructure).

Follows FlashInfer's persistent paged attention as ASPIRE drives it through
HolisticAttentionWrapper.run (aspire/attention/holistic_wrapper.py:344-386):

* GQA: query head h reads KV head h // (Hq / Hkv)
  (flashinfer include/flashinfer/attention/persistent.cuh:290, q_ptr_base).
* Row b attends KV tokens [0, kv_len[b]) of the pages
  kv_indices[kv_indptr[b]:] (16 tokens per page, NHD layout
  [pages, 2, 16, Hkv, D]).
* Causal mask is bottom-right aligned: query i of a row with q_len queries
  is masked at kv_idx when kv_idx + q_len > kv_len + i
  (flashinfer include/flashinfer/attention/prefill.cuh logits_mask).
* Softmax scale sm_scale (default 1/sqrt(D), holistic_wrapper.py:359-361),
  applied in the log2 domain; the returned LSE is base 2:
  lse = log2(sum_j exp2(s_j * sm_scale * log2(e)))
  (persistent.cuh:466-476 writes ptx_log2(d) + m with m scaled by
  sm_scale_log2; consumed as exp2(x*scale*log2e - lse) by
  aspire/backends/page_selector.py:118-119).
* Fully masked rows produce out = 0 and lse = -inf.

The first/last dump restates the ``first_last_compact`` logits transform
(aspire/backends/jit_kernels.py:188-193 body, :252-256 offsets): for
q_idx == 0 (slot 0) and q_idx == q_len - 1 (slot 1; only when q_len > 1) the
raw fp32 q.k, before scaling and before the causal mask, is written rounded
to fp16 at dump[b, h, slot, kv_idx] for every kv_idx < kv_len.  The
``last_token`` transform (:180-184 body, :240-243 offsets) writes only
q_idx == q_len - 1, at dump[b, h, kv_idx].  With ``dump_flags`` (the
use_mode_flags variant, :196-203, :300-301) row b writes nothing when its
flag is 0.  An fp32 dump buffer receives the fp16-rounded value, as the
transform's ``__float2half`` result assigned to a float element does.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

PAGE_SIZE = 16
LOG2E = 1.4426950408889634


def paged_attention(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    qo_indptr,
    kv_indptr,
    kv_indices,
    kv_len,
    *,
    causal: bool = True,
    sm_scale: Optional[float] = None,
    dump: Optional[torch.Tensor] = None,
    dump_num_heads: int = 0,
    dump_kv_stride: int = 0,
    dump_kind: str = "first_last_compact",
    dump_flags=None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (out fp32 [T, Hq, D], lse fp32 [T, Hq]); fills `dump` in place.

    q: [T, Hq, D]; kv_cache: [P, 2, 16, Hkv, D] (any float dtype, computed in
    fp32); qo_indptr / kv_indptr: [B + 1]; kv_len: [B]; kv_indices: page ids.
    Rows with q_len 0 are skipped; output rows not covered stay zero.
    """
    q = q.float()
    T, Hq, D = q.shape
    Hkv = kv_cache.shape[3]
    group = Hq // Hkv
    scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
    qo = [int(x) for x in torch.as_tensor(qo_indptr).tolist()]
    kvp = [int(x) for x in torch.as_tensor(kv_indptr).tolist()]
    kvl = [int(x) for x in torch.as_tensor(kv_len).tolist()]
    idx = torch.as_tensor(kv_indices).long()
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    lse = torch.full((T, Hq), float("-inf"), dtype=torch.float32)
    dump_view = None
    if dump is not None:
        if dump_kind == "first_last_compact":
            dump_view = dump.view(-1, dump_num_heads, 2, dump_kv_stride)
        elif dump_kind == "last_token":
            dump_view = dump.view(-1, dump_num_heads, dump_kv_stride)
        else:
            raise ValueError(f"unknown dump_kind {dump_kind!r}")
    flags = None if dump_flags is None else [int(x) for x in torch.as_tensor(dump_flags).tolist()]
    for b in range(len(kvl)):
        q0, q1 = qo[b], qo[b + 1]
        ql = q1 - q0
        if ql <= 0:
            continue
        L = kvl[b]
        if L <= 0:
            continue
        npages = (L + PAGE_SIZE - 1) // PAGE_SIZE
        pages = idx[kvp[b]: kvp[b] + npages]
        K = kv_cache[pages, 0].float().reshape(npages * PAGE_SIZE, Hkv, D)[:L]
        V = kv_cache[pages, 1].float().reshape(npages * PAGE_SIZE, Hkv, D)[:L]
        Kh = K.repeat_interleave(group, dim=1)  # [L, Hq, D]
        Vh = V.repeat_interleave(group, dim=1)
        s = torch.einsum("qhd,khd->hqk", q[q0:q1], Kh)  # raw logits [Hq, ql, L]
        if dump_view is not None and (flags is None or flags[b] != 0):
            as_dump = lambda t: t.to(torch.float16).to(dump.dtype)  # noqa: E731
            if dump_kind == "first_last_compact":
                dump_view[b, :Hq, 0, :L] = as_dump(s[:, 0, :])
                if ql > 1:
                    dump_view[b, :Hq, 1, :L] = as_dump(s[:, ql - 1, :])
            else:
                dump_view[b, :Hq, :L] = as_dump(s[:, ql - 1, :])
        x = s * (scale * LOG2E)
        if causal:
            kv_idx = torch.arange(L).view(1, 1, L)
            q_idx = torch.arange(ql).view(1, ql, 1)
            x = x.masked_fill(kv_idx + ql > L + q_idx, float("-inf"))
        m = x.amax(dim=-1, keepdim=True)
        m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        e = torch.exp2(x - m_safe)
        ssum = e.sum(dim=-1, keepdim=True)
        row_lse = torch.where(ssum > 0, m_safe + torch.log2(ssum), torch.full_like(ssum, float("-inf")))
        p = torch.where(ssum > 0, e / ssum, torch.zeros_like(e))
        o = torch.einsum("hqk,khd->qhd", p, Vh)
        out[q0:q1] = o
        lse[q0:q1] = row_lse.squeeze(-1).transpose(0, 1)
    return out, lse


def algorithmic_bytes(q_tokens: int, num_qo_heads: int, num_kv_heads: int, attended_tokens: int,
                      pages: int, head_dim: int = 128) -> int:
    """KV bytes read once per layer-call + Q in + O out + page ids."""
    return (attended_tokens * num_kv_heads * head_dim * 2 * 2
            + q_tokens * num_qo_heads * head_dim * 2 * 2 + pages * 4)
