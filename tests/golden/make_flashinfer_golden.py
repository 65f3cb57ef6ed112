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
    python tests/golden/make_flashinfer_golden.py --dump [out.pt]
    python tests/golden/make_flashinfer_golden.py --dump-last [out.pt]

`--dump` runs the reference's first/last logit-dump transform inside
FlashInfer (aspire/backends/jit_kernels.py:188-193, offsets :252-256): a
custom attention variant of FlashInfer's FA2 paged-prefill kernel, JIT-built
with the argument layout of the reference's build_dump_jit_args
(jit_kernels.py:356-390: one fp16 dump tensor, scalars sm_scale, num_heads,
jit_kv_stride), on the refresh layer's full-context program of seeded mixed
batches, into flashinfer_dump.pt.  The installed FlashInfer's holistic
kernel builds its variant with batch index 0 for every request (the request
index is what the reference's patch adds), so it cannot place a per-request
dump; the FA2 kernel passes the request index, and in both kernels the
transform sees the raw q.k (sm_scale is applied afterwards, in the softmax
update).

`--dump-last` does the same for the last-token transform (jit_kernels.py:
180-184, offsets :240-243) with the use_mode_flags guard (:196-203,
:300-301): one variant writing an fp32 buffer whose rows are enabled by an
int32 mode_flags tensor (every other row on), one writing fp16 with no flags,
into flashinfer_dump_last.pt.

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


# The first/last dump as a FlashInfer attention variant (FA2 form): for
# query 0 (slot 0) and the row's last query (slot 1) the raw logit of every
# key the kernel visits is written as fp16 to
# dump[row, head, slot, kv_idx]; the logit itself passes through unchanged.
# Written for this fixture from the transform's description; like the
# reference's variant it does not test kv_idx < kv_len.
DUMP_VARIANT = r"""
struct FirstLastDumpFA2 : AttentionVariantBase {
  static constexpr bool use_softmax = true;
  uint32_t window_left, qo_len, kv_len;
  float sm_scale_log2;
  half* out_dump;
  uint64_t slot_stride, head_stride, row_offset;

  template <typename Params>
  __device__ __host__ FirstLastDumpFA2(const Params& params, uint32_t batch_idx, uint8_t* smem_ptr) {
    qo_len = params.get_qo_len(batch_idx);
    kv_len = params.get_kv_len(batch_idx);
    window_left = kv_len;
    sm_scale_log2 = params.sm_scale * math::log2e;
    out_dump = params.attention_weights;
    slot_stride = (uint64_t)params.jit_kv_stride;
    head_stride = 2u * slot_stride;
    row_offset = (uint64_t)batch_idx * (uint64_t)params.num_heads * head_stride;
  }

  REGISTER_LOGITS_TRANSFORM(params, logits, batch_idx, qo_idx, kv_idx, qo_head_idx, kv_head_idx, {
    if (qo_idx == 0u || qo_idx + 1u == qo_len) {
      const uint64_t slot = (qo_idx == 0u) ? 0u : 1u;
      out_dump[row_offset + (uint64_t)qo_head_idx * head_stride + slot * slot_stride + kv_idx] =
          __float2half(logits);
    }
    return logits;
  })
};
"""


# The last-token transform: the logit of the last query of a row (q_len >= 1)
# goes to dump[row, head, kv_idx] as __float2half(logit), converted to the
# buffer's element type; with DUMP_FLAGS a row whose mode flag is 0 writes
# nothing.  Written for this fixture from the transform's description.
LAST_VARIANT = r"""
struct LastTokenDumpFA2 : AttentionVariantBase {
  static constexpr bool use_softmax = true;
  uint32_t window_left, qo_len, kv_len, dump_on;
  float sm_scale_log2;
  DUMP_T* out_dump;
  uint64_t head_stride, row_offset;

  template <typename Params>
  __device__ __host__ LastTokenDumpFA2(const Params& params, uint32_t batch_idx, uint8_t* smem_ptr) {
    qo_len = params.get_qo_len(batch_idx);
    kv_len = params.get_kv_len(batch_idx);
    window_left = kv_len;
    sm_scale_log2 = params.sm_scale * math::log2e;
    out_dump = params.attention_weights;
    head_stride = (uint64_t)params.jit_kv_stride;
    row_offset = (uint64_t)batch_idx * (uint64_t)params.num_heads * head_stride;
    dump_on = DUMP_ON;
  }

  REGISTER_LOGITS_TRANSFORM(params, logits, batch_idx, qo_idx, kv_idx, qo_head_idx, kv_head_idx, {
    if (dump_on && qo_idx + 1u == qo_len) {
      out_dump[row_offset + (uint64_t)qo_head_idx * head_stride + kv_idx] = __float2half(logits);
    }
    return logits;
  })
};
"""


def dump_last_main(out_path):
    """Last-token dump fixtures: (fp32 buffer, mode flags) and (fp16, no flags)."""
    import flashinfer

    dev = torch.device("cuda:0")
    result = {"flashinfer_version": flashinfer.__version__, "variant": LAST_VARIANT, "cases": {}}
    variants = {
        "f32_flags": ("float", torch.float32, "(params.mode_flags[batch_idx] != 0) ? 1u : 0u", True),
        "f16": ("half", torch.float16, "1u", False),
    }
    for vname, (ctype, dtype, on, flagged) in variants.items():
        src = LAST_VARIANT.replace("LastTokenDumpFA2", "LastTokenDumpFA2_" + vname) \
            .replace("DUMP_T", ctype).replace("DUMP_ON", on)
        names, types = ["attention_weights"], [ctype]
        if flagged:
            names.append("mode_flags")
            types.append("int32_t")
        jit_args = ["aspire_golden_last_dump_" + vname, torch.bfloat16, torch.bfloat16, torch.bfloat16, torch.int32,
                    128, 128, names, types, ["sm_scale", "num_heads", "jit_kv_stride"],
                    ["double", "int64_t", "int64_t"], "LastTokenDumpFA2_" + vname, src]
        for name, lay, seed in dump_cases():
            q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=seed)
            q, kv = q.to(dev), kv.to(dev)
            i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
            stride = (lay.pages_per_row * 16 + 127) // 128 * 128
            H = lay.num_qo_heads
            dump = torch.full((lay.batch * H * stride,), float("-inf"), dtype=dtype, device=dev)
            flags = (torch.arange(lay.batch, dtype=torch.int32, device=dev) + 1) % 2  # rows 0, 2, ... on
            ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
            w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD", backend="fa2", jit_args=jit_args)
            w.plan(i32(lay.qo_indptr), i32(lay.kv_indptr), i32(lay.kv_indices), i32(last_page_lens(lay)), H,
                   lay.num_kv_heads, 128, 16, causal=True, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
                   disable_split_kv=True)
            sm_scale = 1.0 / 128 ** 0.5
            run_args = [dump, flags] if flagged else [dump]
            out, lse = w.run(q, kv, *run_args, sm_scale, H, stride, return_lse=True)
            torch.cuda.synchronize()
            result["cases"][f"{vname}/{name}"] = {
                "seed": seed, "kv_stride": stride, "flags": flags.cpu() if flagged else None,
                "layout": {k: getattr(lay, k) for k in ("num_qo_heads", "num_kv_heads", "modes", "q_lens", "kv_lens",
                                                        "qo_indptr", "kv_indptr", "kv_indices", "block_table",
                                                        "ctx_lens", "pages_per_row", "num_pages_total")},
                "dump": dump.view(lay.batch, H, stride).cpu(),
                "out": out.cpu(),
                "lse": lse.float().cpu(),
            }
            print(vname, name, "dump", (lay.batch, H, stride), dtype, "finite", int(torch.isfinite(dump).sum()),
                  flush=True)
    torch.save(result, out_path)
    print("saved", out_path)


def dump_cases():
    from aspire_b200.workloads import config1_layout as c1
    yield "cfg1_full", full_context_layout(c1(seed=0)), 0
    lay = make_layout(batch=4, ctx=2000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=24,
                      seed=8)
    yield "qwen8b_full", full_context_layout(lay), 8


def dump_main(out_path):
    import flashinfer

    dev = torch.device("cuda:0")
    jit_args = ["aspire_golden_first_last_dump", torch.bfloat16, torch.bfloat16, torch.bfloat16, torch.int32,
                128, 128, ["attention_weights"], ["half"], ["sm_scale", "num_heads", "jit_kv_stride"],
                ["double", "int64_t", "int64_t"], "FirstLastDumpFA2", DUMP_VARIANT]
    result = {"flashinfer_version": flashinfer.__version__, "variant": DUMP_VARIANT, "cases": {}}
    for name, lay, seed in dump_cases():
        q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=seed)
        q, kv = q.to(dev), kv.to(dev)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)  # noqa: E731
        # Padded to a multiple of the kernel's key tile, as the engine pads its
        # dump stride (compute_max_cta_tile_kv, aspire/attention/flashinfer.py:63-105):
        # the transform has no kv_idx < kv_len test, so the last tile's
        # positions past kv_len land in the padding.
        stride = (lay.pages_per_row * 16 + 127) // 128 * 128
        H = lay.num_qo_heads
        dump = torch.full((lay.batch * H * 2 * stride,), float("-inf"), dtype=torch.float16, device=dev)
        ws = torch.empty(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD", backend="fa2", jit_args=jit_args)
        # One KV chunk per request: with split-KV chunks the last key tile of
        # a chunk runs past the chunk's end and, with no kv_idx test in the
        # transform, overwrites the next chunk's positions with logits of
        # other keys (seen as windows of wrong values every chunk length).
        w.plan(i32(lay.qo_indptr), i32(lay.kv_indptr), i32(lay.kv_indices), i32(last_page_lens(lay)), H,
               lay.num_kv_heads, 128, 16, causal=True, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
               disable_split_kv=True)
        sm_scale = 1.0 / 128 ** 0.5
        out, lse = w.run(q, kv, dump, sm_scale, H, stride, return_lse=True)
        torch.cuda.synchronize()
        result["cases"][name] = {
            "seed": seed, "kv_stride": stride,
            "layout": {k: getattr(lay, k) for k in ("num_qo_heads", "num_kv_heads", "modes", "q_lens", "kv_lens",
                                                    "qo_indptr", "kv_indptr", "kv_indices", "block_table",
                                                    "ctx_lens", "pages_per_row", "num_pages_total")},
            "dump": dump.view(lay.batch, H, 2, stride).cpu(),
            "out": out.cpu(),
            "lse": lse.float().cpu(),
        }
        print(name, "dump", (lay.batch, H, 2, stride), "finite", int(torch.isfinite(dump).sum()), flush=True)
    torch.save(result, out_path)
    print("saved", out_path)


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

    args = [a for a in sys.argv[1:] if a not in ("--prefill", "--dump", "--dump-last")]
    if "--dump-last" in sys.argv[1:]:
        dump_last_main(Path(args[0]) if args else HERE / "flashinfer_dump_last.pt")
        return
    if "--prefill" in sys.argv[1:]:
        prefill_main(Path(args[0]) if args else HERE / "flashinfer_prefill.pt")
        return
    if "--dump" in sys.argv[1:]:
        dump_main(Path(args[0]) if args else HERE / "flashinfer_dump.pt")
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
