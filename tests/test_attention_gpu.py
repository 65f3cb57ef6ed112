"""GPU parity of the mixed paged attention against the fp32 CPU oracle."""

import os

import numpy as np
import pytest
import torch

from aspire_b200.attention import HolisticAttentionWrapper
from aspire_b200.workloads import MixedLayout, config1_layout, full_context_layout, make_layout, rows_layout

from gpu_helpers import (assert_attention_close, assert_dump_close, make_inputs, oracle_attention,
                         run_attention)

pytestmark = pytest.mark.gpu

# Set by test_gather_route_gpu.py, which reruns this file with narrow rows on
# the CUDA-core kernel or with tcgen05 off.
ROUTING_VARS = ("ASPIRE_B200_DISABLE_TC", "ASPIRE_B200_TC_MIN_ROWS", "ASPIRE_B200_TC_MIN_KV")


def test_config1_mixed_attention(cuda_device):
    lay = config1_layout(seed=0)
    q, kv = make_inputs(lay, cuda_device, seed=0)
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_config1_refresh_dump(cuda_device):
    lay = config1_layout(seed=1)
    q, kv = make_inputs(lay, cuda_device, seed=1)
    stride = 1024 + 64
    out, lse, dump, _ = run_attention(lay, q, kv, dump=True, dump_stride=stride)
    ref_out, ref_lse, ref_dump = oracle_attention(lay, q, kv, dump_stride=stride)
    assert_attention_close(out, lse, ref_out, ref_lse)
    assert_dump_close(dump, ref_dump, lay, stride)


def test_refresh_dump_multi_tile_rows(cuda_device):
    """The dump of rows whose packed queries span several tiles (q_len 20 and
    30 at group 4): query 0's logits are recorded at every key, also in
    planners that stop later tiles at their causal span."""
    lay = _custom_layout(q_lens=[20, 1, 30], kv_lens=[700, 300, 1030], hq=32, hkv=8, seed=9)
    q, kv = make_inputs(lay, cuda_device, seed=9)
    stride = 1040
    out, lse, dump, _ = run_attention(lay, q, kv, dump=True, dump_stride=stride)
    ref_out, ref_lse, ref_dump = oracle_attention(lay, q, kv, dump_stride=stride)
    assert_attention_close(out, lse, ref_out, ref_lse)
    assert_dump_close(dump, ref_dump, lay, stride)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 8), (8, 1), (4, 2)])
@pytest.mark.parametrize("draft_fraction", [0.0, 0.5, 1.0])
def test_mixed_ragged_split_kv(cuda_device, hq, hkv, draft_fraction):
    """Verify q_len 3..9, ragged contexts, split-KV chunks merged on device."""
    lay = make_layout(batch=6, ctx=2999, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=draft_fraction,
                      budget_pages=37, seed=hq + hkv)
    q, kv = make_inputs(lay, cuda_device, seed=5)
    out, lse, _, w = run_attention(lay, q, kv)
    assert w.plan_info.num_merge > 0 or lay.kv_lens.max() <= w.plan_info.chunk_tokens
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_exact_widths_with_long_chunks(cuda_device):
    """A plan with more than two items per SM and split-KV chunks above 4096
    tokens: every item runs at its own width (16/32/48 columns), and a CTA
    moves between widths from item to item."""
    lay = make_layout(batch=24, ctx=24000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=40,
                      seed=21)
    q, kv = make_inputs(lay, cuda_device, seed=21)
    out, lse, _, w = run_attention(lay, q, kv)
    assert w.plan_info.chunk_tokens > 4096
    assert w.plan_info.num_merge > 0 or lay.kv_lens.max() <= w.plan_info.chunk_tokens
    assert len(set(((lay.q_lens * 4 + 15) // 16).tolist())) > 1, "the case must mix item widths"
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


def _tc_item_columns(lay, num_sms):
    """(packed rows, planned columns) of every tcgen05 decode item, from the
    library's host planner for this layout (WorkItem words 8, 9 and 15)."""
    import ctypes

    from aspire_b200 import _capi

    lib = _capi.load_library()
    buf = np.zeros(1 << 22, dtype=np.uint8)
    info = _capi.AspirePlanInfo()
    p = lambda a: np.ascontiguousarray(a, dtype=np.int32).ctypes.data_as(_capi.c_int32_p)  # noqa: E731
    arrays = [np.ascontiguousarray(a, dtype=np.int32) for a in (lay.qo_indptr, lay.kv_indptr, lay.kv_lens)]
    rc = lib.aspire_plan_host_only(p(arrays[0]), p(arrays[1]), p(arrays[2]), lay.batch, lay.num_qo_heads,
                                   lay.num_kv_heads, 128, 16, 1, num_sms, buf.ctypes.data_as(ctypes.c_void_p),
                                   buf.nbytes, 1 << 30, ctypes.byref(info))
    assert rc == 0, lib.aspire_last_error()
    w = buf.view(np.int32)
    items = w[w[5]: w[5] + info.num_items * 16].reshape(-1, 16)
    tc = items[items[:, 14] == 1]
    return tc[:, 9] - tc[:, 8], tc[:, 15]


def test_padded_long_items(cuda_device):
    """Few items per SM (8 rows): the plan gives the verify rows' items (3 to
    9 queries x 4 heads: 16, 32 and 48 columns of their own) one width, the
    widest, while the drafting rows' items keep their 16 columns; the padded
    columns hold no query and must not reach the output."""
    lay = make_layout(batch=8, ctx=6000, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.5, budget_pages=16,
                      seed=31)
    if not any(k in os.environ for k in ROUTING_VARS):  # the plan's shape under the default routing
        num_sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
        rows, cols = _tc_item_columns(lay, num_sms)
        exact = (rows + 15) // 16 * 16
        padded = cols > exact
        assert padded.any() and (cols[padded] == cols.max()).all(), "the case must pad some verify items"
        assert (cols[~padded] == 0).any(), "the drafting rows' items keep their own width"
    q, kv = make_inputs(lay, cuda_device, seed=31)
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("hq,hkv", [(40, 8), (56, 8), (24, 1)])
def test_common_width_groups_not_dividing_the_tile(cuda_device, hq, hkv):
    """GQA groups of 5, 7 and 24: the query tile holds 45, 42 and 48 rows, so
    the item's 48 columns include rows past its queries, which must not reach
    the output."""
    lay = make_layout(batch=7, ctx=1900, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.4, budget_pages=23,
                      seed=hq)
    q, kv = make_inputs(lay, cuda_device, seed=hq)
    out, lse, _, w = run_attention(lay, q, kv)
    assert w.plan_info.chunk_tokens <= 4096 or not w.plan_info.tc_enabled
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


def _custom_layout(q_lens, kv_lens, hq=16, hkv=8, seed=0):
    rng = np.random.default_rng(seed)
    B = len(q_lens)
    pages = [(k + 15) // 16 for k in kv_lens]
    ppr = max(max(pages), 1)
    bt = np.stack([r * ppr + rng.permutation(ppr) for r in range(B)]).astype(np.int32)
    kv_indptr = np.zeros(B + 1, np.int32)
    idx = []
    for r in range(B):
        idx.append(bt[r, :pages[r]])
        kv_indptr[r + 1] = kv_indptr[r] + pages[r]
    qo = np.zeros(B + 1, np.int32)
    qo[1:] = np.cumsum(q_lens)
    return MixedLayout(num_qo_heads=hq, num_kv_heads=hkv, modes=np.array([1 if q > 1 else 0 for q in q_lens]),
                       q_lens=np.array(q_lens, np.int32), kv_lens=np.array(kv_lens, np.int32), qo_indptr=qo,
                       kv_indptr=kv_indptr, kv_indices=np.concatenate(idx).astype(np.int32), block_table=bt,
                       ctx_lens=np.array(kv_lens, np.int32), pages_per_row=ppr, num_pages_total=B * ppr)


def test_edge_rows(cuda_device):
    """Empty rows, a padding row (queries, no KV), kv shorter than q (fully masked
    queries), single-token KV, lengths off the page boundary."""
    lay = _custom_layout(q_lens=[0, 3, 1, 5, 9, 2, 1], kv_lens=[40, 0, 1, 3, 4100, 17, 1023], seed=2)
    q, kv = make_inputs(lay, cuda_device, seed=2)
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)
    # padding row: zero output, -inf lse
    r0, r1 = int(lay.qo_indptr[1]), int(lay.qo_indptr[2])
    assert out[r0:r1].abs().max().item() == 0.0
    assert torch.isinf(lse[r0:r1]).all()


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 8), (40, 8)])
def test_prefill_rows(cuda_device, hq, hkv):
    """Long-query causal rows (prefill chunks, with and without a cached
    prefix, and one shorter than its chunk): each query tile of a row stops at
    its causal span, and the tiles of one row are planned independently."""
    lay = _custom_layout(q_lens=[200, 77, 300, 1, 13], kv_lens=[200, 1077, 350, 900, 9], hq=hq, hkv=hkv, seed=7)
    q, kv = make_inputs(lay, cuda_device, seed=7)
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (48, 8), (64, 8)])
def test_prefill_items_halves_chunks_and_dump(cuda_device, hq, hkv):
    """Prefill items (rows of >= 128 packed query rows) next to decode items
    in one launch: two-half items, single-half tail items, a long cached
    prefix split into KV chunks merged on device, groups that do not divide
    128 (group 6: halves of 126 rows), and the first/last logit dump."""
    lay = _custom_layout(q_lens=[700, 150, 40, 1, 260], kv_lens=[5000, 150, 2100, 3000, 900], hq=hq, hkv=hkv,
                         seed=21)
    q, kv = make_inputs(lay, cuda_device, seed=21)
    stride = 5008
    out, lse, dump, w = run_attention(lay, q, kv, dump=True, dump_stride=stride)
    assert w.plan_info.num_items_prefill > 0 or not w.plan_info.tc_enabled
    ref_out, ref_lse, ref_dump = oracle_attention(lay, q, kv, dump_stride=stride)
    assert_attention_close(out, lse, ref_out, ref_lse)
    assert_dump_close(dump, ref_dump, lay, stride)


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_rows_mask_modes(cuda_device, causal):
    """Prefill rows with and without the causal mask (a chunk of 300 queries
    after a 500-token prefix, and a row whose keys are fewer than its queries)."""
    lay = _custom_layout(q_lens=[300, 64, 200], kv_lens=[800, 64, 130], hq=32, hkv=8, seed=13)
    q, kv = make_inputs(lay, cuda_device, seed=13)
    out, lse, _, _ = run_attention(lay, q, kv, causal=causal)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv, causal=causal)
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_nan_in_unused_page_slots(cuda_device):
    """A page's slots past a row's last token may hold anything: NaN there
    (zero weight) must not reach the output, on the decode and prefill paths."""
    lay = _custom_layout(q_lens=[1, 5, 300, 2, 40], kv_lens=[17, 1000, 333, 130, 77], hq=32, hkv=8, seed=4)
    q, kv = make_inputs(lay, cuda_device, seed=4)
    for r in range(lay.batch):
        n = int(lay.kv_lens[r])
        if n % 16:
            page = int(lay.kv_indices[int(lay.kv_indptr[r + 1]) - 1])
            kv[page, :, n % 16:] = float("nan")
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert torch.isfinite(out.float()).all()
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_long_context_rows(cuda_device):
    lay = make_layout(batch=3, ctx=32768 + 7, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.34,
                      budget_pages=128, seed=11)
    q, kv = make_inputs(lay, cuda_device, seed=11)
    out, lse, _, _ = run_attention(lay, q, kv)
    ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_deterministic_and_graph_replay(cuda_device):
    """Bitwise-identical reruns; a captured graph stays valid across re-plans that
    rewrite the static page-index buffer in place (as the engine's step loop does)."""
    common = dict(batch=5, num_qo_heads=32, num_kv_heads=8, draft_fraction=0.4, budget_pages=20,
                  verify_q_len=5, draft_rows=[1, 3], pages_per_row=128)
    lay1 = make_layout(ctx=2048, seed=4, **common)
    lay2 = make_layout(ctx=1500, seed=9, **common)
    q, kv = make_inputs(lay1, cuda_device, seed=4)
    static_idx = torch.zeros(lay1.kv_indices.shape[0] + lay2.kv_indices.shape[0], dtype=torch.int32,
                             device=cuda_device)
    w = HolisticAttentionWrapper(torch.empty(1, device=cuda_device))

    def plan(lay):
        n = lay.kv_indices.shape[0]
        static_idx[:n] = torch.from_numpy(lay.kv_indices).to(cuda_device)
        w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr),
                    torch.from_numpy(lay.kv_lens), static_idx, 32, 8, 128, 16, causal=True)

    out = torch.empty_like(q)
    lse = torch.empty(q.shape[0], q.shape[1], device=cuda_device, dtype=torch.float32)
    plan(lay1)
    w.run(q, kv, out=out, lse=lse)
    first = out.clone(), lse.clone()
    w.run(q, kv, out=out, lse=lse)
    torch.cuda.synchronize()
    assert torch.equal(first[0], out) and torch.equal(first[1], lse)

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        w.run(q, kv, out=out, lse=lse)
    for lay in (lay2, lay1):
        plan(lay)
        g.replay()
        torch.cuda.synchronize()
        ref_out, ref_lse, _ = oracle_attention(lay, q, kv)
        assert_attention_close(out, lse, ref_out, ref_lse)


def test_bad_page_ids_are_reported_not_faulted(cuda_device):
    lay = config1_layout(seed=3)
    q, kv = make_inputs(lay, cuda_device, seed=3)
    lay.kv_indices = lay.kv_indices.copy()
    lay.kv_indices[3] = lay.num_pages_total + 5  # out of range: the kernel skips it and flags it
    w = HolisticAttentionWrapper(torch.empty(1, device=cuda_device))
    w.clear_device_status()
    run_attention(lay, q, kv, wrapper=w)
    torch.cuda.synchronize()
    assert w.device_status() & 1


@pytest.mark.parametrize("case", ["cfg1", "qwen8b_mixed", "qwen8b_full", "qwen8b_q9"])
def test_matches_flashinfer_golden(cuda_device, golden_dir, case):
    """The sm_100a kernels against FlashInfer's persistent attention on the same
    seeded inputs (fixture from tests/golden/make_flashinfer_golden.py)."""
    from aspire_b200.workloads import fill_tensors

    g = torch.load(golden_dir / "flashinfer_attention.pt", weights_only=False)["cases"][case]
    lay = MixedLayout(**g["layout"])
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse, _, _ = run_attention(lay, q.to(cuda_device), kv.to(cuda_device))
    err = (out.float().cpu() - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, err.max().item()
    assert (lse.cpu() - g["lse"]).abs().max().item() <= 2e-3


DUMP_VARIANTS = [("last_token", torch.float16, False), ("last_token", torch.float32, True),
                 ("first_last_compact", torch.float32, False), ("first_last_compact", torch.float16, True)]


@pytest.mark.parametrize("kind,dtype,flagged", DUMP_VARIANTS,
                         ids=["last_f16", "last_f32_flags", "first_last_f32", "first_last_f16_flags"])
@pytest.mark.parametrize("shape", ["refresh", "prefill"])
def test_dump_variants(cuda_device, kind, dtype, flagged, shape):
    """The reference's other dump variants (jit_kernels.py:180-203,
    holistic_wrapper.py:401-434): last-token (one slot, the last query of
    every row, q_len 1 included), the use_mode_flags guard (rows 0, 2, 4, ...
    on, the others untouched) and an fp32 buffer holding fp16-rounded logits,
    against the oracle, on a refresh-layer program (draft rows with one query,
    verify rows with 3-9) and on prefill chunks beside decode rows."""
    if shape == "refresh":
        lay = full_context_layout(make_layout(batch=6, ctx=2999, num_qo_heads=32, num_kv_heads=8,
                                              draft_fraction=0.5, budget_pages=37, seed=31))
    else:
        lay = rows_layout([150, 1, 5, 64], [1000, 1500, 800, 64], 32, 8, seed=32)
    q, kv = make_inputs(lay, cuda_device, seed=33)
    stride = (int(lay.kv_lens.max()) + 127) // 128 * 128 + 16
    flags = (torch.arange(lay.batch, dtype=torch.int32) + 1) % 2 if flagged else None
    out, lse, dump, w = run_attention(lay, q, kv, dump=True, dump_stride=stride, dump_kind=kind, dump_dtype=dtype,
                                      dump_flags=flags)
    ref_out, ref_lse, ref_dump = oracle_attention(lay, q, kv, dump_stride=stride, dump_kind=kind, dump_dtype=dtype,
                                                  dump_flags=flags)
    assert dump.dtype == dtype
    assert w.device_status() == 0
    if shape == "prefill":
        assert w.plan_info.num_items_prefill > 0 or not w.plan_info.tc_enabled
    assert_attention_close(out, lse, ref_out, ref_lse)
    assert_dump_close(dump, ref_dump, lay, stride, dump_kind=kind, dump_flags=flags)


def test_dump_variant_arguments_are_checked(cuda_device):
    """run() refuses a dump buffer of the wrong element type for the variant,
    one too small for its slots, and missing mode flags."""
    from aspire_b200.attention import dump_jit_args

    lay = config1_layout(seed=2)
    q, kv = make_inputs(lay, cuda_device, seed=2)
    stride = 1024
    w = HolisticAttentionWrapper(torch.empty(1, device=cuda_device),
                                 jit_args=dump_jit_args("last_token", use_mode_flags=True,
                                                        dump_buffer_dtype=torch.float32))
    kvi = torch.from_numpy(lay.kv_indices).to(cuda_device)
    w.plan_host(torch.from_numpy(lay.qo_indptr), torch.from_numpy(lay.kv_indptr), torch.from_numpy(lay.kv_lens),
                kvi, lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)
    H = lay.num_qo_heads
    flags = torch.ones(lay.batch, dtype=torch.int32, device=cuda_device)
    f16 = torch.full((lay.batch * H * stride,), float("-inf"), dtype=torch.float16, device=cuda_device)
    f32 = torch.full((lay.batch * H * stride,), float("-inf"), dtype=torch.float32, device=cuda_device)
    with pytest.raises(ValueError, match="dump variant writes"):
        w.run(q, kv, f16, flags, H, stride)
    with pytest.raises(ValueError, match="smaller than"):
        w.run(q, kv, f32[:-1], flags, H, stride)
    with pytest.raises(ValueError, match="mode_flags"):
        w.run(q, kv, f32, H, stride)
    w.run(q, kv, f32, flags, H, stride)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(f32).any())


@pytest.mark.parametrize("case", ["cfg1_full", "qwen8b_full"])
def test_dump_matches_flashinfer_variant(cuda_device, golden_dir, case):
    """The refresh-layer dump of the sm_100a kernels against the reference's
    first/last transform run inside FlashInfer as a custom attention variant
    (fixture from tests/golden/make_flashinfer_golden.py --dump), on the same
    seeded inputs: every defined position (slot 0; slot 1 of multi-query
    rows; keys [0, kv_len)) within one fp16 step, plus the outputs and LSE.
    FlashInfer's variant also writes logits past kv_len up to its key tile
    (the reference omits that test, aspire/backends/jit_kernels.py:128-177);
    this kernel writes only [0, kv_len), which the selector's masking makes
    equivalent."""
    from aspire_b200.workloads import fill_tensors
    from test_oracle_golden import dump_positions_close

    g = torch.load(golden_dir / "flashinfer_dump.pt", weights_only=False)["cases"][case]
    lay = MixedLayout(**g["layout"])
    S = g["kv_stride"]
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse, dump, _ = run_attention(lay, q.to(cuda_device), kv.to(cuda_device), dump=True, dump_stride=S)
    torch.cuda.synchronize()
    dump_positions_close(dump.cpu().view(lay.batch, lay.num_qo_heads, 2, S), g["dump"], lay)
    err = (out.float().cpu() - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, err.max().item()
    assert (lse.cpu() - g["lse"]).abs().max().item() <= 2e-3


@pytest.mark.parametrize("case", ["f32_flags/cfg1_full", "f32_flags/qwen8b_full", "f16/cfg1_full",
                                  "f16/qwen8b_full"])
def test_last_token_dump_matches_flashinfer_variant(cuda_device, golden_dir, case):
    """The last-token dump of the sm_100a kernels (fp32 buffer with mode
    flags, fp16 without) against the reference's last_token transform run
    inside FlashInfer (tests/golden/make_flashinfer_golden.py --dump-last)."""
    from aspire_b200.workloads import fill_tensors
    from test_oracle_golden import last_dump_positions_close

    g = torch.load(golden_dir / "flashinfer_dump_last.pt", weights_only=False)["cases"][case]
    lay = MixedLayout(**g["layout"])
    S = g["kv_stride"]
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse, dump, _ = run_attention(lay, q.to(cuda_device), kv.to(cuda_device), dump=True, dump_stride=S,
                                      dump_kind="last_token", dump_dtype=g["dump"].dtype, dump_flags=g["flags"])
    torch.cuda.synchronize()
    last_dump_positions_close(dump.cpu().view(lay.batch, lay.num_qo_heads, S), g["dump"], lay, g["flags"])
    err = (out.float().cpu() - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, err.max().item()
    assert (lse.cpu() - g["lse"]).abs().max().item() <= 2e-3


@pytest.mark.parametrize("case", ["prefill_g4", "prefill_g1"])
def test_prefill_matches_flashinfer_golden(cuda_device, golden_dir, case):
    """The prefill phase against FlashInfer's prefill wrapper on the same seeded
    chunks (fixture from tests/golden/make_flashinfer_golden.py --prefill)."""
    from aspire_b200.workloads import fill_tensors

    g = torch.load(golden_dir / "flashinfer_prefill.pt", weights_only=False)["cases"][case]
    lay = MixedLayout(**g["layout"])
    q, kv = fill_tensors(lay, device="cpu", dtype=torch.bfloat16, seed=g["seed"])
    out, lse, _, w = run_attention(lay, q.to(cuda_device), kv.to(cuda_device))
    assert w.plan_info.num_items_prefill > 0 or not w.plan_info.tc_enabled
    err = (out.float().cpu() - g["out"].float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, err.max().item()
    assert (lse.cpu() - g["lse"]).abs().max().item() <= 2e-3
