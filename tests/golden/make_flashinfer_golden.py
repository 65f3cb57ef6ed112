"""Golden attention outputs from FlashInfer's persistent (holistic) attention.

The reference's attention is FlashInfer's BatchAttention persistent kernel,
driven by aspire/attention/holistic_wrapper.py (plan: :253-265, run: :344-386);
the reference pins FlashInfer 56ed5409 plus a patch that changes the CTA tile
size and the work-to-request indexing but not the arithmetic semantics
(bottom-right causal mask, base-2 LSE, GQA mapping).  This script runs the
FlashInfer installed in this image (flashinfer.BatchAttention, the same
holistic module) on seeded mixed batches and saves its outputs, so the CPU
oracle and the sm_100a kernels are checked against FlashInfer itself.

Needs a CUDA GPU (FlashInfer JIT-compiles its kernel on first use):

    python tests/golden/make_flashinfer_golden.py [out.pt]
    python tests/golden/make_flashinfer_golden.py --prefill [out.pt]

`--prefill` runs FlashInfer's BatchPrefillWithPagedKVCacheWrapper, the
library the reference runs its prefill chunks through
(aspire/models/sparse_draft_runner.py:270, encode_slots in
aspire/backends/base.py:1559-1674), on seeded prefill chunks, into
flashinfer_prefill.pt.

Inputs are regenerated bit-identically on CPU from the stored layout and
seed (aspire_b200.workloads.fill_tensors on the CPU generator), so only the
layouts and outputs are stored.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from aspire_b200.workloads import (config1_layout, fill_tensors, full_context_layout, last_page_lens,  # noqa: E402
                                   make_layout, rows_layout)


def cases():
    yield "cfg1", config1_layout(seed=0), 0
    lay = make_layout(batch=5, ctx=3000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.4, budget_pages=40,
                      seed=5)
    yield "qwen8b_mixed", lay, 5
    yield "qwen8b_full", full_context_layout(lay), 6
    yield "qwen8b_q9", make_layout(batch=3, ctx=700, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.0,
                                   verify_q_len=9, seed=7), 7


def prefill_cases():
    # A chunk after a cached prefix and a chunk from position 0 (group 4), and
    # a row with one query head per KV head (group 1).
    yield "prefill_g4", rows_layout([200, 64], [330, 64], 8, 2, seed=11), 11
    yield "prefill_g1", rows_layout([150], [400], 4, 4, seed=12), 12


def prefill_main(out_path):
    import flashinfer

    dev = torch.device("cuda:0")
    result = {"flashinfer_version": flashinfer.__version__, "cases": {}}
    for name, lay, seed in prefill_cases():
        q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=seed)
        q, kv = q.to(dev), kv.to(dev)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
        ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(i32(lay.qo_indptr), i32(lay.kv_indptr), i32(lay.kv_indices), i32(last_page_lens(lay)),
               lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True, q_data_type=torch.bfloat16,
               kv_data_type=torch.bfloat16)
        out, lse = w.run(q, kv, return_lse=True)
        torch.cuda.synchronize()
        result["cases"][name] = {
            "seed": seed,
            "layout": {k: getattr(lay, k) for k in ("num_qo_heads", "num_kv_heads", "modes", "q_lens", "kv_lens",
                                                    "qo_indptr", "kv_indptr", "kv_indices", "block_table",
                                                    "ctx_lens", "pages_per_row", "num_pages_total")},
            "out": out.cpu(),
            "lse": lse.float().cpu(),
        }
        print(name, "out", tuple(out.shape), "lse", tuple(lse.shape), flush=True)
    torch.save(result, out_path)
    print("saved", out_path)


def main():
    import flashinfer

    args = [a for a in sys.argv[1:] if a != "--prefill"]
    if "--prefill" in sys.argv[1:]:
        prefill_main(Path(args[0]) if args else HERE / "flashinfer_prefill.pt")
        return
    out_path = Path(args[0]) if args else HERE / "flashinfer_attention.pt"
    dev = torch.device("cuda:0")
    result = {"flashinfer_version": flashinfer.__version__, "cases": {}}
    for name, lay, seed in cases():
        q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=seed)
        q, kv = q.to(dev), kv.to(dev)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
        w = flashinfer.BatchAttention(kv_layout="NHD", device="cuda")
        w.plan(i32(lay.qo_indptr), i32(lay.kv_indptr), i32(lay.kv_indices), i32(lay.kv_lens), lay.num_qo_heads,
               lay.num_kv_heads, 128, 128, 16, causal=True, q_data_type=torch.bfloat16,
               kv_data_type=torch.bfloat16)
        out, lse = w.run(q, kv)
        torch.cuda.synchronize()
        result["cases"][name] = {
            "seed": seed,
            "layout": {k: getattr(lay, k) for k in ("num_qo_heads", "num_kv_heads", "modes", "q_lens", "kv_lens",
                                                    "qo_indptr", "kv_indptr", "kv_indices", "block_table",
                                                    "ctx_lens", "pages_per_row", "num_pages_total")},
            "out": out.cpu(),
            "lse": lse.float().cpu(),
        }
        print(name, "out", tuple(out.shape), "lse", tuple(lse.shape), flush=True)
    torch.save(result, out_path)
    print("saved", out_path)


if __name__ == "__main__":
    main()
