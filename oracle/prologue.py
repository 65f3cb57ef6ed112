"""CPU restatement of a layer's attention prologue (test infrastructure).

q/k RMSNorm as the reference's module (aspire/models/transformer.py:505-515):
(x.float() * rsqrt(mean(x^2) + eps)).to(bf16) * weight (bf16 product); the
HF-to-interleaved permutation (transformer.py:360-364); FlashInfer's
interleaved RoPE as mylib::rope calls it (aspire/models/mixed_transformer.py:
159-197; flashinfer pos_enc.cuh BatchQKApplyRotaryKernel): pair (2p, 2p+1)
rotated by pos * freq_p, freq_p = (1/theta)^(2p/d), scaled by 1/rope_scale
with FlashInfer's Llama-3.1 smoothing, pos = offsets[b] + (t - indptr[b]),
tokens outside the rows unrotated; then the paged append of the rotated k
and of v (oracle.kv_append).  The rotation runs in float64 here, so it
agrees with FlashInfer's fast-intrinsic kernel to a bf16 rounding step.
"""

from __future__ import annotations

import math

import torch

from oracle import kv_append


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = (xf * torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)).to(x.dtype)
    return y * weight


def permute_for_rope(x: torch.Tensor) -> torch.Tensor:
    *lead, d = x.shape
    return x.view(*lead, 2, d // 2).transpose(-2, -1).reshape(*lead, d)


def rope_freqs(d: int, theta: float, scale: float, llama31=None) -> torch.Tensor:
    rcp_theta = 1.0 / theta
    rcp_scale = 1.0 / scale
    if llama31 is not None:
        lf, hf, old = llama31
        sa = old / (2 * math.pi * hf - 2 * math.pi * lf)
        sb = -1.0 / (hf / lf - 1.0)
    else:
        sa = sb = 0.0
    out = []
    for i in range(d):
        f = rcp_theta ** (2 * (i // 2) / d)
        s = min(max(f * sa + sb, 0.0), 1.0)
        out.append((1 - s) * (f * rcp_scale) + s * f)
    return torch.tensor(out, dtype=torch.float64)


def rope_interleaved(x: torch.Tensor, indptr, offsets, theta: float, scale: float, llama31=None) -> torch.Tensor:
    """x [T, H, d] bf16 -> rotated copy (tokens outside [indptr[0], indptr[-1]) unchanged)."""
    out = x.clone()
    d = x.shape[-1]
    freq = rope_freqs(d, theta, scale, llama31)
    for b in range(len(indptr) - 1):
        for t in range(int(indptr[b]), int(indptr[b + 1])):
            pos = int(offsets[b]) + t - int(indptr[b])
            ang = pos * freq
            c, s = torch.cos(ang), torch.sin(ang)
            v = x[t].double()
            even, odd = v[:, 0::2], v[:, 1::2]
            r = torch.empty_like(v)
            r[:, 0::2] = even * c[0::2] - odd * s[0::2]
            r[:, 1::2] = odd * c[1::2] + even * s[1::2]
            out[t] = r.to(x.dtype)
    return out


def prologue(q, k, v, append_indptr, offsets, cache, page_indices, page_indptr, last_page_len, *,
             q_norm_weight=None, k_norm_weight=None, eps=1e-6, theta=1e4, scale=1.0, llama31=None,
             page_size=16):
    """Returns (q_rotated, cache_after) for CPU tensors; `cache` is not modified."""
    if q_norm_weight is not None:
        q = permute_for_rope(rms_norm(q, q_norm_weight, eps))
        k = permute_for_rope(rms_norm(k, k_norm_weight, eps))
    n_rows = len(last_page_len)
    indptr = [int(x) for x in append_indptr[:n_rows + 1]]
    q_rot = rope_interleaved(q, indptr, offsets, theta, scale, llama31)
    k_rot = rope_interleaved(k, indptr, offsets, theta, scale, llama31)
    after = cache.clone()
    kv_append.update_kv_padded(k_rot, v, torch.as_tensor(append_indptr), after, torch.as_tensor(page_indices),
                               torch.as_tensor(page_indptr), torch.as_tensor(last_page_len), page_size)
    return q_rot, after
