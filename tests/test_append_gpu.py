"""GPU parity of the paged KV append (aspire_append_kv) against the reference's
Triton kernel (golden fixture) and the CPU oracle."""

import numpy as np
import pytest
import torch

import aspire_b200.kv_ops  # noqa: F401  (registers torch.ops.aspire_b200.update_kv_padded)
from aspire_b200.kv_ops import append_kv
from oracle import kv_append as oracle_append

pytestmark = pytest.mark.gpu


def test_append_matches_reference_kernel_golden(cuda_device, golden_dir):
    g = torch.load(golden_dir / "kv_append.pt", weights_only=False)
    dev = cuda_device
    cache = g["cache_before"].to(torch.bfloat16).to(dev)
    args = [g[n].to(dev) for n in ("append_indptr",)]
    torch.ops.aspire_b200.update_kv_padded(
        g["k"].to(torch.bfloat16).to(dev), g["v"].to(torch.bfloat16).to(dev), args[0], cache,
        g["page_indices"].to(dev), g["page_indptr"].to(dev), g["last_page_len"].to(dev), 16)
    torch.cuda.synchronize()
    assert torch.equal(cache.cpu(), g["cache_after"].to(torch.bfloat16))


@pytest.mark.parametrize("hkv", [1, 2, 8])
def test_append_random_mixed_batch(cuda_device, hkv):
    rng = np.random.default_rng(hkv)
    B = 9
    q_lens = rng.integers(0, 10, size=B)
    q_lens[3] = 0
    pages_per_row = 20
    seq = rng.integers(1, pages_per_row * 16, size=B)
    seq = np.maximum(seq, q_lens)
    append_indptr = np.zeros(B + 2, np.int32)
    append_indptr[1:B + 1] = np.cumsum(q_lens)
    T = int(append_indptr[B]) + 5  # bucket padding tokens
    append_indptr[B + 1] = T
    page_indptr = np.zeros(B + 2, np.int32)
    last = np.zeros(B + 1, np.int32)
    idx = []
    for b in range(B):
        n = (int(seq[b]) + 15) // 16
        idx.append(b * pages_per_row + rng.permutation(pages_per_row)[:n])
        page_indptr[b + 1] = page_indptr[b] + n
        last[b] = (int(seq[b]) - 1) % 16 + 1
    page_indptr[B + 1] = page_indptr[B]
    idx = np.concatenate(idx).astype(np.int32)
    P = B * pages_per_row
    k = torch.randn(T, hkv, 128)
    v = torch.randn(T, hkv, 128)
    cache_cpu = torch.randn(P, 2, 16, hkv, 128).to(torch.bfloat16)
    ref = cache_cpu.clone()
    oracle_append.update_kv_padded(k.to(torch.bfloat16), v.to(torch.bfloat16), torch.from_numpy(append_indptr),
                                   ref, torch.from_numpy(idx), torch.from_numpy(page_indptr), torch.from_numpy(last))
    dev = cuda_device
    cache = cache_cpu.to(dev)
    append_kv(k.to(torch.bfloat16).to(dev), v.to(torch.bfloat16).to(dev), torch.from_numpy(append_indptr).to(dev),
              cache, torch.from_numpy(idx).to(dev), torch.from_numpy(page_indptr).to(dev),
              torch.from_numpy(last).to(dev), 16)
    torch.cuda.synchronize()
    assert torch.equal(cache.cpu(), ref)


def test_append_rejects_strided_heads(cuda_device):
    k = torch.zeros(4, 2, 256, dtype=torch.bfloat16, device=cuda_device)[:, :, :128]
    cache = torch.zeros(4, 2, 16, 2, 128, dtype=torch.bfloat16, device=cuda_device)
    i32 = lambda *x: torch.tensor(x, dtype=torch.int32, device=cuda_device)  # noqa: E731
    with pytest.raises(ValueError):
        append_kv(k, k, i32(0, 4), cache, i32(0), i32(0, 1), i32(4), 16)
