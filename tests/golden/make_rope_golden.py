"""Golden outputs of the reference's attention prologue math on the GPU.

The reference runs, per layer (aspire/models/sparse_draft_transformer.py:
150-162): q_norm / k_norm (its RMSNorm module, aspire/models/transformer.py:
505-515), the HF-to-interleaved permutation (transformer.py:360-364), then
mylib::rope, i.e. FlashInfer's apply_rope_inplace or
apply_llama31_rope_inplace with interleave=True (aspire/models/
mixed_transformer.py:159-197).  This script restates the norm and the
permutation with the same torch operations, runs them and FlashInfer's RoPE
(the library installed in this image) on a CUDA device, and saves the rotated
q and k.  Inputs are regenerated bit-identically on CPU from the stored seed.

    python tests/golden/make_rope_golden.py [out.pt]
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def case_inputs(seed, T, hq, hkv, rows, pos_base):
    """Inputs of one case on CPU: q, k, v [T, H, 128] bf16 (as the wqkv split
    yields them), norm weights, append indptr over `rows` segments (the last
    tokens are bucket padding) and the rows' RoPE offsets."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(T, hq, 128, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(T, hkv, 128, generator=g) * 2).to(torch.bfloat16)
    v = torch.randn(T, hkv, 128, generator=g).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    lens = torch.randint(1, 10, (rows,), generator=g)
    indptr = torch.zeros(rows + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(lens, 0).to(torch.int32)
    assert int(indptr[-1]) <= T
    offsets = (pos_base + torch.randint(0, 4096, (rows,), generator=g)).to(torch.int32)
    return q, k, v, qw, kw, indptr, offsets


CASES = {
    # Qwen3-8B heads, qk-norm, theta 1e6, positions up to ~37k (large RoPE angles)
    "qwen3_8b": dict(seed=1, T=64, hq=32, hkv=8, rows=9, pos_base=32768, norm=True, theta=1e6, scale=1.0,
                     llama31=None, eps=1e-6),
    # Qwen3-1.7B heads, near the start of the context
    "qwen3_1_7b": dict(seed=2, T=40, hq=16, hkv=8, rows=5, pos_base=0, norm=True, theta=1e6, scale=1.0,
                       llama31=None, eps=1e-6),
    # Llama-3.1 style: no qk-norm, smoothed frequencies
    "llama31": dict(seed=3, T=48, hq=32, hkv=8, rows=6, pos_base=8000, norm=False, theta=5e5, scale=8.0,
                    llama31=(1.0, 4.0, 8192.0), eps=1e-5),
}


def rms_norm(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)).type_as(x) * w


def permute_for_rope(x):
    *lead, d = x.shape
    return x.view(*lead, 2, d // 2).transpose(-2, -1).reshape(*lead, d)


def main():
    import flashinfer

    out_path = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "rope_prologue.pt"
    dev = torch.device("cuda:0")
    result = {"flashinfer_version": flashinfer.__version__, "cases": {}}
    for name, c in CASES.items():
        q, k, v, qw, kw, indptr, offsets = case_inputs(c["seed"], c["T"], c["hq"], c["hkv"], c["rows"],
                                                      c["pos_base"])
        qd, kd = q.to(dev), k.to(dev)
        if c["norm"]:
            qd = permute_for_rope(rms_norm(qd.view(1, *qd.shape), qw.to(dev), c["eps"])).reshape(qd.shape)
            kd = permute_for_rope(rms_norm(kd.view(1, *kd.shape), kw.to(dev), c["eps"])).reshape(kd.shape)
        qd, kd = qd.contiguous(), kd.contiguous()
        normed_q, normed_k = qd.clone(), kd.clone()
        if c["llama31"] is None:
            flashinfer.rope.apply_rope_inplace(qd, kd, indptr.to(dev), offsets.to(dev), interleave=True,
                                               rope_scale=c["scale"], rope_theta=c["theta"])
        else:
            lf, hf, old = c["llama31"]
            flashinfer.rope.apply_llama31_rope_inplace(qd, kd, indptr.to(dev), offsets.to(dev), interleave=True,
                                                       rope_scale=c["scale"], rope_theta=c["theta"],
                                                       low_freq_factor=lf, high_freq_factor=hf,
                                                       old_context_len=int(old))
        torch.cuda.synchronize()
        result["cases"][name] = {"params": c, "indptr": indptr, "offsets": offsets,
                                 "q_normed": normed_q.cpu(), "k_normed": normed_k.cpu(),
                                 "q_rot": qd.cpu(), "k_rot": kd.cpu()}
        print(name, tuple(qd.shape), flush=True)
    torch.save(result, out_path)
    print("saved", out_path)


if __name__ == "__main__":
    main()
