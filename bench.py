"""Benchmark of the unified mixed forward hot path on B200.

One step = one decode step's hot path of a Qwen3-8B-shaped model (config 3 of
the reference's benchmark list: 36 layers, 32 q / 8 KV heads, head_dim 128,
batch 64, 32k context, sparse budget 128 pages, refresh layer -2):

  * 35 ordinary layers: paged KV append + mixed draft/verify attention
    (draft rows: 128 selected pages, q_len 1; verify rows: full context,
    q_len = U{2..8} + 1, causal);
  * the refresh layer: append + full-context attention of every row with the
    first/last logit dump;
  (the append runs inside the attention launch, `run(..., append=(k, v))`;
  `--separate-append` launches it as its own kernel before each attention)
  * page scoring + top-k re-selection written in place into the draft table.

Every layer reads one resident single-layer KV cache (8.7 GB at TP 1, far
larger than the 126 MB L2, so nothing is served from cache between layers);
a real model holds 36 such caches, which do not fit one GPU.  Under torchrun
each rank holds its tensor-parallel share of the heads (KV-head ranges, as
the reference's aspire/tp.py shards them) for the same batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aspire_b200|reference]

`--workload prefill` measures the prefill phase instead (long-query causal
rows through the same wrapper, the reference's chunked `encode_slots`
attention): TFLOP/s of the attention over the visible (query, key) pairs,
beside FlashInfer's BatchPrefillWithPagedKVCacheWrapper (the library the
reference runs prefill through) on the same inputs when it is installed.

`--workload sweep` runs the reference's config-5 kernel sweep: the mixed
attention plus the top-k page selection alone at Qwen3-8B heads over context
lengths 4k/16k/32k/80k, batch 1 to 128, drafting fraction 0/0.5/1, verify
q_len 1/5/9 and budgets of 64 and 512 pages, HBM GB/s against the measured
peak per point.

After the timed region the step's outputs are checked (outside the timing):
two rows of a mixed layer and of the refresh layer against a plain torch
fp32 attention on the GPU, and the new draft table against the properties
the selection guarantees; a failed check ends the run with an error.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from aspire_b200.tp import local_head_counts  # noqa: E402

METRIC = "mixed-attn HBM GB/s (% of peak); accepted tokens/s per box at 1/2/4/8 B200"
UNIT = "GB/s"

CFG = dict(model="qwen3-8b-heads", n_layer=36, refresh_layer=34, num_qo_heads=32, num_kv_heads=8, batch=64,
           ctx=32768, pages_per_row=2080, draft_fraction=0.5, budget_pages=128, L=8, seed=0)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="aspire_b200", choices=["aspire_b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # Smaller cases of the same step (profiling captures); the headline run uses the defaults.
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--block-table", default="arange", choices=["arange", "random"],
                    help="arange: the reference engine's contiguous per-row pages; random: scattered pages")
    ap.add_argument("--workload", default="step", choices=["step", "prefill", "sweep", "decode"])
    ap.add_argument("--no-decode", action="store_true", help="skip the end-to-end decode leg of the step run")
    ap.add_argument("--separate-append", action="store_true",
                    help="launch each layer's KV append as its own kernel instead of inside the attention launch")
    ap.add_argument("--decode-config", type=int, default=2, choices=[2, 3, 4],
                    help="the reference's end-to-end config the decode leg runs (2 by default)")
    ap.add_argument("--decode-batch", type=int, default=None)
    ap.add_argument("--decode-prompt", type=int, default=None)
    ap.add_argument("--decode-new", type=int, default=None)
    ap.add_argument("--sweep-ctx", default="4096,16384,32768,81920")
    ap.add_argument("--sweep-batch", default="1,4,16,64,128")
    ap.add_argument("--prefill-cases", default="1x8192+0,4x2048+16384,8x1024+4096,2x4096+0",
                    help="comma-separated ROWSxQLEN+PREFIX prefill chunks (Qwen3-8B heads, causal)")
    args = ap.parse_args()
    if args.batch is not None:
        CFG["batch"] = args.batch
    if args.ctx is not None:
        CFG["ctx"] = args.ctx
        CFG["pages_per_row"] = (args.ctx + 512 + 15) // 16
    CFG["block_table"] = args.block_table
    if args.layers is not None:
        CFG["n_layer"] = args.layers
        CFG["refresh_layer"] = max(args.layers - 2, 0)
    return args


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons while the
    timed region runs: through NVML every 20 ms (read-only queries on the
    device with this CUDA device's PCI bus id), else nvidia-smi every 0.2 s."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = torch.device(device)
        self.gpu_index = self.device.index or 0
        self.rows = []
        self.source = "nvidia-smi"
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self._nvml = pynvml
            self.source = "nvml"
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        nv = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(self._handle, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        masks = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                 nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        flags = ["Active" if bits & m else "Not Active" for m in masks]
        self.rows.append([str(self.gpu_index), str(sm), str(mx), "", hex(bits)] + flags)

    def _run(self):
        while not self._stop.is_set():
            try:
                if self._nvml is not None:
                    self._sample_nvml()
                else:
                    out = subprocess.run(["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                         timeout=5)
                    for line in out.stdout.strip().splitlines():
                        self.rows.append([x.strip() for x in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.02 if self._nvml is not None else 0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows), "source": self.source}


# ----------------------------------------------------------------------------- workload
def build_workload(device, rank: int, world: int):
    from aspire_b200.workloads import full_context_layout, make_layout, last_page_lens

    hq, hkv = local_head_counts(CFG["num_qo_heads"], CFG["num_kv_heads"], rank, world)
    lay = make_layout(batch=CFG["batch"], ctx=CFG["ctx"], num_qo_heads=hq, num_kv_heads=hkv,
                      draft_fraction=CFG["draft_fraction"], budget_pages=CFG["budget_pages"],
                      pages_per_row=CFG["pages_per_row"], seed=CFG["seed"],
                      block_table=CFG.get("block_table", "arange"))
    full = full_context_layout(lay)
    return lay, full, last_page_lens(lay), last_page_lens(full)


def step_bytes(lay, full, n_layer: int, kv_stride: int, k: int) -> dict:
    """Algorithmic bytes of one step (each byte counted once per layer-call)."""
    hd = 128
    T = lay.total_q
    append = T * lay.num_kv_heads * hd * 2 * 2 * 2          # read new K,V + write them
    mixed = lay.algorithmic_bytes()
    refresh = full.algorithmic_bytes()
    dump_write = sum(int(full.kv_lens[b]) * (2 if full.q_lens[b] > 1 else 1) for b in range(full.batch)) \
        * full.num_qo_heads * 2
    select = full.batch * full.num_qo_heads * 2 * min(kv_stride, lay.pages_per_row * 16) * 2 \
        + full.batch * lay.pages_per_row * 4 + full.batch * k * 4 + T * full.num_qo_heads * 4
    total = (n_layer - 1) * mixed + refresh + n_layer * append + dump_write + select
    return dict(total=total, mixed=mixed, refresh=refresh, append=append, dump_write=dump_write, select=select)


class HotPath:
    """All device state of the benchmark step, driven through the public API."""

    def __init__(self, device, lay, full, lpl_mixed, lpl_full, fused_append: bool = True):
        from aspire_b200.attention import HolisticAttentionWrapper, first_last_dump_jit_args
        from aspire_b200.kv_ops import append_kv
        from aspire_b200.page_selector import PageSelectorFirstLastAvg
        from aspire_b200.workloads import fill_tensors

        self.append_kv = append_kv
        self.fused_append = fused_append
        self.device = device
        self.lay, self.full = lay, full
        n_layer = CFG["n_layer"]
        T, hq, hkv = lay.total_q, lay.num_qo_heads, lay.num_kv_heads
        # Inputs: per-layer q and new K/V (rows of the bucket), one resident layer cache.
        _, self.kv = fill_tensors(lay, device=device, seed=CFG["seed"])
        g = torch.Generator(device=device)
        g.manual_seed(CFG["seed"] + 1)
        self.q = torch.randn(n_layer, T, hq, 128, generator=g, device=device).to(torch.bfloat16)
        self.k_new = torch.randn(n_layer, T, hkv, 128, generator=g, device=device).to(torch.bfloat16)
        self.v_new = torch.randn(n_layer, T, hkv, 128, generator=g, device=device).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        self.lse = torch.empty(T, hq, device=device, dtype=torch.float32)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(device)  # noqa: E731
        self.qo_indptr = i32(lay.qo_indptr)
        self.mixed_indptr, self.mixed_last = i32(lay.kv_indptr), i32(lpl_mixed)
        self.full_indptr, self.full_last = i32(full.kv_indptr), i32(lpl_full)
        self.block_table = i32(lay.block_table)
        self.num_pages = i32((lay.ctx_lens + 15) // 16)
        # The engine's page tables, read directly by the kernels (page-table
        # mode: the reference's build_unified_indices copy is absorbed): mode
        # flags, the draft rows' page tables and the block table.  The mixed
        # program reads draft rows from their tables; the refresh program reads
        # every row's block-table prefix (all rows in verify mode).
        counts = np.diff(lay.kv_indptr)
        draft_tab = np.zeros((lay.batch, max(1, int(counts.max()))), np.int32)
        for b in range(lay.batch):
            if lay.modes[b] == 0:
                draft_tab[b, :counts[b]] = lay.kv_indices[lay.kv_indptr[b]:lay.kv_indptr[b + 1]]
        self.mode_flags = i32(lay.modes)
        self.full_modes = i32(np.ones(lay.batch, np.int32))
        self.draft_indices = i32(draft_tab)
        self.mixed_tables = (self.mode_flags, self.draft_indices, self.block_table)
        self.full_tables = (self.full_modes, self.draft_indices, self.block_table)
        self.kv_stride = lay.pages_per_row * 16
        self.dump = torch.full((lay.batch * hq * 2 * self.kv_stride,), float("-inf"), dtype=torch.float16,
                               device=device)
        self.k_sel = CFG["budget_pages"]
        self.draft_table = torch.zeros(lay.batch, self.k_sel, dtype=torch.int32, device=device)
        self.draft_counts = torch.zeros(lay.batch, dtype=torch.int32, device=device)
        ws = torch.empty(1, device=device)
        self.mixed = HolisticAttentionWrapper(ws)
        self.mixed.set_page_tables(*self.mixed_tables)
        self.refresh = HolisticAttentionWrapper(ws, jit_args=first_last_dump_jit_args())
        self.refresh.set_page_tables(*self.full_tables)
        self.selector = PageSelectorFirstLastAvg(
            max_batch_size=lay.batch, pages_per_slot=lay.pages_per_row, subset_cache_size=self.k_sel, L=CFG["L"],
            n_heads=hq, page_size=16, max_seq_length=self.kv_stride, device=device, bsz=lay.batch, dec_len=9,
            kv_stride=self.kv_stride, draft_percent=None, min_draft_pages=self.k_sel)
        self.graph = None

    def plan(self):
        lay, full = self.lay, self.full
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
        self.mixed.plan_host(t(lay.qo_indptr), t(lay.kv_indptr), t(lay.kv_lens), None,
                             lay.num_qo_heads, lay.num_kv_heads, 128, 16, causal=True)
        self.refresh.plan_host(t(full.qo_indptr), t(full.kv_indptr), t(full.kv_lens), None,
                               full.num_qo_heads, full.num_kv_heads, 128, 16, causal=True)

    def layer(self, layer: int):
        """Append + attention of one layer (the refresh layer with the dump):
        one launch with the append inside the attention, or the append kernel
        and then the attention."""
        new = (self.k_new[layer], self.v_new[layer])
        fused = new if self.fused_append else None
        if layer == CFG["refresh_layer"]:
            if not self.fused_append:
                self.append_kv(*new, self.qo_indptr, self.kv, None, self.full_indptr, self.full_last, 16,
                               page_tables=self.full_tables)
            self.refresh.run(self.q[layer], self.kv, self.dump, self.lay.num_qo_heads, self.kv_stride,
                             out=self.out[layer], lse=self.lse, append=fused)
        else:
            if not self.fused_append:
                self.append_kv(*new, self.qo_indptr, self.kv, None, self.mixed_indptr, self.mixed_last, 16,
                               page_tables=self.mixed_tables)
            self.mixed.run(self.q[layer], self.kv, out=self.out[layer], append=fused)

    def select(self):
        self.selector.select_into(self.draft_table, self.draft_counts, self.dump, self.lse, self.num_pages,
                                  self.block_table, self.qo_indptr)

    def step_eager(self):
        for layer in range(CFG["n_layer"]):
            self.layer(layer)
        self.select()

    def capture(self):
        self.step_eager()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.step_eager()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step_eager()
        torch.cuda.synchronize()

    def launches_per_step(self) -> int:
        # Per layer: append + attention (tcgen05 kernel, plus the CUDA-core
        # kernel unless every row routes to tcgen05, plus the split-KV merge);
        # then the selection (page scoring + top-k).
        tc = bool(self.mixed.plan_info.tc_enabled)
        all_tc = tc and int(os.environ.get("ASPIRE_B200_TC_MIN_ROWS", "1") or "1") <= 1
        per_attn = (1 if tc else 0) + (0 if all_tc else 1) + 1
        return CFG["n_layer"] * ((0 if self.fused_append else 1) + per_attn) + 2


def time_device(fn, steps, warmup, dist_on):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    return start.elapsed_time(end) / steps


def kernel_roofline(hp: HotPath, steps: int, peak: float, peak_kind: str):
    """Average device duration of the mixed attention layer-call: its kernels
    (tcgen05 attention + split-KV merge) and the gaps between them."""
    q, out = hp.q[0], hp.out[0]
    for _ in range(3):
        hp.mixed.run(q, hp.kv, out=out)
    torch.cuda.synchronize()
    # A CUDA graph of back-to-back launches timed between two events on the
    # launching stream: device time only, under the sustained load of a step;
    # the average over three replays (90+ launches), and the median of three
    # such measurements (the first, right after the timed steps, can run a few
    # per cent slow while the power cap settles).
    ms = statistics.median(graph_time(lambda: hp.mixed.run(q, hp.kv, out=out), max(steps, 30), replays=3)
                           for _ in range(3))
    bytes_ = hp.lay.algorithmic_bytes()
    achieved = bytes_ / (ms * 1e-3) / 1e9
    # DRAM bytes (read + write) per algorithmic byte of the mixed layer-call,
    # from the ncu capture summarised under profiles/, scaled to this launch.
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        try:
            ratio = json.loads(tp.read_text()).get("dram_bytes_over_algorithmic")
            traffic = int(round(ratio * bytes_)) if ratio else None
        except Exception:
            traffic = None
    return {"kernel": "mixed attention layer-call (aspire_attn_tc_kernel + aspire_attn_merge_kernel)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_source": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic, "ms_per_launch": round(ms, 4),
            "algorithmic_bytes_per_launch": int(bytes_)}


def graph_time(fn, reps: int, replays: int = 1) -> float:
    """Device milliseconds per call of `fn`, from `replays` replays of a CUDA
    graph that holds `reps` back-to-back calls (no host time in the interval)."""
    fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(replays):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (reps * replays)
    del g
    return ms


def breakdown(hp: HotPath) -> dict:
    """Device time of each call of the step: a CUDA graph of back-to-back calls
    of one kind, sized to run for tens of milliseconds like the step itself."""
    L = CFG["n_layer"]
    if not hasattr(hp, "refresh_nodump"):
        from aspire_b200.attention import HolisticAttentionWrapper
        full = hp.full
        hp.refresh_nodump = HolisticAttentionWrapper(torch.empty(1, device=hp.device))
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
        hp.refresh_nodump.set_page_tables(*hp.full_tables)
        hp.refresh_nodump.plan_host(t(full.qo_indptr), t(full.kv_indptr), t(full.kv_lens), None,
                                    full.num_qo_heads, full.num_kv_heads, 128, 16, causal=True)
    if not hasattr(hp, "prologue_args"):
        # The fused prologue (q/k norm + RoPE + append) on the step's q and new
        # K/V, Qwen3-8B settings (qk-norm, theta 1e6), RoPE positions at the
        # end of each row's context.
        from aspire_b200.kv_ops import qkv_prologue
        g = torch.Generator(device=hp.device)
        g.manual_seed(5)
        w = (1 + 0.1 * torch.randn(2, 128, generator=g, device=hp.device)).to(torch.bfloat16)
        offs = torch.from_numpy((hp.lay.kv_lens - hp.lay.q_lens).astype(np.int32)).to(hp.device)
        q_rot = torch.empty_like(hp.q[0])
        hp.prologue_args = (qkv_prologue, w, offs, q_rot)
    qkv_prologue, w, offs, q_rot = hp.prologue_args
    if not hasattr(hp, "mixed_random"):
        # The same batch with scattered physical pages (each row's pages a
        # random permutation of its own range of the same cache), as the draft
        # tables look after re-selection and block tables after reuse.
        from aspire_b200.attention import HolisticAttentionWrapper, first_last_dump_jit_args
        from aspire_b200.workloads import make_layout
        lay = hp.lay
        lay_r = make_layout(batch=lay.batch, ctx=CFG["ctx"], num_qo_heads=lay.num_qo_heads,
                            num_kv_heads=lay.num_kv_heads, draft_fraction=CFG["draft_fraction"],
                            budget_pages=CFG["budget_pages"], pages_per_row=CFG["pages_per_row"], seed=CFG["seed"],
                            block_table="random")
        assert np.array_equal(lay_r.kv_lens, lay.kv_lens) and np.array_equal(lay_r.q_lens, lay.q_lens)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(hp.device)  # noqa: E731
        counts = np.diff(lay_r.kv_indptr)
        draft_tab = np.zeros((lay.batch, max(1, int(counts.max()))), np.int32)
        for b in range(lay.batch):
            if lay_r.modes[b] == 0:
                draft_tab[b, :counts[b]] = lay_r.kv_indices[lay_r.kv_indptr[b]:lay_r.kv_indptr[b + 1]]
        hp.random_tables = (i32(draft_tab), i32(lay_r.block_table))
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
        hp.mixed_random = HolisticAttentionWrapper(torch.empty(1, device=hp.device))
        hp.mixed_random.set_page_tables(hp.mode_flags, *hp.random_tables)
        hp.mixed_random.plan_host(t(lay.qo_indptr), t(lay.kv_indptr), t(lay.kv_lens), None, lay.num_qo_heads,
                                  lay.num_kv_heads, 128, 16, causal=True)
        full = hp.full
        hp.refresh_random = HolisticAttentionWrapper(torch.empty(1, device=hp.device),
                                                     jit_args=first_last_dump_jit_args())
        hp.refresh_random.set_page_tables(hp.full_modes, *hp.random_tables)
        hp.refresh_random.plan_host(t(full.qo_indptr), t(full.kv_indptr), t(full.kv_lens), None,
                                    full.num_qo_heads, full.num_kv_heads, 128, 16, causal=True)
    calls = {
        "prologue": (lambda: qkv_prologue(hp.q[0], hp.k_new[0], hp.v_new[0], hp.qo_indptr, offs, hp.kv, None,
                                          hp.mixed_indptr, hp.mixed_last, 16, q_norm_weight=w[0],
                                          k_norm_weight=w[1], rope_theta=1e6, q_out=q_rot,
                                          page_tables=hp.mixed_tables), 200),
        "append": (lambda: hp.append_kv(hp.k_new[0], hp.v_new[0], hp.qo_indptr, hp.kv, None,
                                        hp.mixed_indptr, hp.mixed_last, 16, page_tables=hp.mixed_tables), 200),
        "mixed_attention": (lambda: hp.mixed.run(hp.q[0], hp.kv, out=hp.out[0]), 30),
        "mixed_attention_fused_append": (lambda: hp.mixed.run(hp.q[0], hp.kv, out=hp.out[0],
                                                              append=(hp.k_new[0], hp.v_new[0])), 30),
        "refresh_attention": (lambda: hp.refresh.run(hp.q[L - 2], hp.kv, hp.dump, hp.lay.num_qo_heads,
                                                     hp.kv_stride, out=hp.out[L - 2], lse=hp.lse), 15),
        "refresh_nodump": (lambda: hp.refresh_nodump.run(hp.q[L - 2], hp.kv, out=hp.out[L - 2], lse=hp.lse), 15),
        "select_pages": (lambda: hp.selector.select_into(hp.draft_table, hp.draft_counts, hp.dump, hp.lse,
                                                         hp.num_pages, hp.block_table, hp.qo_indptr), 100),
        "mixed_attention_random_tables": (lambda: hp.mixed_random.run(hp.q[0], hp.kv, out=hp.out[0]), 30),
        "refresh_attention_random_tables": (lambda: hp.refresh_random.run(hp.q[L - 2], hp.kv, hp.dump,
                                                                          hp.lay.num_qo_heads, hp.kv_stride,
                                                                          out=hp.out[L - 2], lse=hp.lse), 15),
    }
    res = {}
    for name, (fn, reps) in calls.items():
        res[name + "_ms"] = round(graph_time(fn, reps), 4)
    return res


def _torch_attention_row(q, kv, pages, kv_len: int, causal: bool = True):
    """Plain torch fp32 attention of one request row on the GPU (no library
    code): q [q_len, Hq, 128], pages the row's page ids; bottom-right causal
    mask, GQA head h -> KV head h // group.  Returns (out [q_len, Hq, 128],
    base-2 LSE [q_len, Hq])."""
    ql, hq, d = q.shape
    hkv = kv.shape[3]
    g = hq // hkv
    k = kv[pages, 0].reshape(-1, hkv, d)[:kv_len].float()
    v = kv[pages, 1].reshape(-1, hkv, d)[:kv_len].float()
    qg = q.float().view(ql, hkv, g, d)
    s = torch.einsum("qkgd,skd->kgqs", qg, k) / math.sqrt(d)
    if causal:
        i = torch.arange(ql, device=q.device)[:, None]
        j = torch.arange(kv_len, device=q.device)[None, :]
        s = s.masked_fill((j > kv_len - ql + i)[None, None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1) / math.log(2.0)
    o = torch.einsum("kgqs,skd->qkgd", torch.softmax(s, dim=-1), v)
    return o.reshape(ql, hq, d), lse.permute(2, 0, 1).reshape(ql, hq)


def check_step(hp: HotPath) -> dict:
    """Outside the timed region: recomputes a mixed layer and the refresh
    layer eagerly and compares one draft and one verify row of each with
    _torch_attention_row (max-abs <= 2e-2, mean-abs <= 2e-3, LSE <= 2e-3),
    then checks the new draft table: counts = min(pages, budget); each row's
    ids ascending, from its own block-table prefix, including its last L
    pages; zeros past the count.  Returns a summary; raises on a mismatch."""
    lay, full = hp.lay, hp.full
    rows = [int(np.flatnonzero(lay.modes == 0)[0]), int(np.flatnonzero(lay.modes == 1)[0])]
    worst = {"max_abs": 0.0, "mean_abs": 0.0, "lse_abs": 0.0}
    R = CFG["refresh_layer"]
    for layer, src, want_lse in ((0, lay, False), (R, full, True)):
        hp.layer(layer)
        torch.cuda.synchronize()
        for r in rows:
            t0, t1 = int(src.qo_indptr[r]), int(src.qo_indptr[r + 1])
            pages = torch.from_numpy(src.kv_indices[src.kv_indptr[r]:src.kv_indptr[r + 1]].astype(np.int64))
            ref, ref_lse = _torch_attention_row(hp.q[layer][t0:t1], hp.kv, pages.to(hp.device), int(src.kv_lens[r]))
            err = (hp.out[layer][t0:t1].float() - ref).abs()
            worst["max_abs"] = max(worst["max_abs"], float(err.max().item()))
            worst["mean_abs"] = max(worst["mean_abs"], float(err.mean().item()))
            if want_lse:
                worst["lse_abs"] = max(worst["lse_abs"], float((hp.lse[t0:t1] - ref_lse).abs().max().item()))
    hp.select()
    torch.cuda.synchronize()
    tab, cnt = hp.draft_table.cpu().numpy(), hp.draft_counts.cpu().numpy()
    num_pages = hp.num_pages.cpu().numpy()
    k, L = hp.k_sel, CFG["L"]
    table_ok = bool(np.array_equal(cnt, np.minimum(num_pages, k)))
    for b in range(lay.batch):
        n = int(cnt[b])
        ids = tab[b, :n]
        own = lay.block_table[b, :num_pages[b]]
        table_ok &= bool(np.all(np.diff(ids) > 0)) and bool(np.all(tab[b, n:] == 0))
        table_ok &= bool(np.isin(ids, own).all()) and bool(np.isin(own[max(0, num_pages[b] - L):], ids).all())
    ok = worst["max_abs"] <= 2e-2 and worst["mean_abs"] <= 2e-3 and worst["lse_abs"] <= 2e-3 and table_ok
    summary = {"rows": rows, "layers": [0, R], **{k_: round(v, 6) for k_, v in worst.items()},
               "draft_table_ok": table_ok, "ok": ok,
               "reference": "plain torch fp32 attention on the GPU (mixed layer 0 and the refresh layer)"}
    if not ok:
        raise SystemExit(f"bench output check failed: {json.dumps(summary)}")
    return summary


def e2e_measure(hp: HotPath, steps: int, warmup: int, bytes_per_step: int):
    """Through the public API with host buffers, every step: host planning of
    both attention programs (plan upload included), H2D of every layer's q and
    new K/V from pinned memory, the step, D2H of every layer's attention output
    and of the new draft table and counts, then a host synchronisation.  The
    copies stream per layer on a second stream, as a serving loop would issue
    them: layer L's inputs land while earlier layers compute (the layer waits
    for its own copy), and its output leaves once the layer is done; the
    timed region ends when the last copy of the step has reached the host."""
    q_h = hp.q.cpu().pin_memory()
    k_h = hp.k_new.cpu().pin_memory()
    v_h = hp.v_new.cpu().pin_memory()
    out_h = torch.empty(hp.out.shape, dtype=hp.out.dtype, pin_memory=True)
    tab_h = torch.empty(hp.draft_table.shape, dtype=torch.int32, pin_memory=True)
    cnt_h = torch.empty(hp.draft_counts.shape, dtype=torch.int32, pin_memory=True)
    n_layer = CFG["n_layer"]
    copy = torch.cuda.Stream()

    def streamed_step():
        main = torch.cuda.current_stream()
        ev_in = [torch.cuda.Event() for _ in range(n_layer)]
        ev_out = [torch.cuda.Event() for _ in range(n_layer)]
        copy.wait_stream(main)
        with torch.cuda.stream(copy):
            for layer in range(n_layer):
                hp.q[layer].copy_(q_h[layer], non_blocking=True)
                hp.k_new[layer].copy_(k_h[layer], non_blocking=True)
                hp.v_new[layer].copy_(v_h[layer], non_blocking=True)
                ev_in[layer].record(copy)
        for layer in range(n_layer):
            main.wait_event(ev_in[layer])
            hp.layer(layer)
            ev_out[layer].record(main)
        with torch.cuda.stream(copy):
            for layer in range(n_layer):
                copy.wait_event(ev_out[layer])
                out_h[layer].copy_(hp.out[layer], non_blocking=True)
        hp.select()
        tab_h.copy_(hp.draft_table, non_blocking=True)
        cnt_h.copy_(hp.draft_counts, non_blocking=True)
        main.wait_stream(copy)

    # One CUDA graph of the streamed step (copies included); the host plans
    # both programs before every replay.
    streamed_step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        streamed_step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        streamed_step()
    torch.cuda.synchronize()

    def one():
        hp.plan()
        g.replay()
        torch.cuda.current_stream().synchronize()

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = (time.perf_counter() - t0) / steps
    del g
    h2d = q_h.numel() * 2 + k_h.numel() * 2 + v_h.numel() * 2
    d2h = out_h.numel() * 2 + tab_h.numel() * 4 + cnt_h.numel() * 4
    return dt, h2d, d2h


# ----------------------------------------------------------------------------- CPU baseline
def cpu_baseline(lay, full, budget_s: float = 12.0, max_rows: int | None = None):
    """The oracle (fp32 torch on all the host cores) on a bounded sample of the
    workload: the mixed attention of whole rows of the bench batch, draft and
    verify rows alternating, one row per call, until about `budget_s` seconds
    of CPU work (or `max_rows` rows) are done."""
    from oracle import attention as oracle_attn

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    draft = [int(r) for r in np.flatnonzero(lay.modes == 0)]
    verify = [int(r) for r in np.flatnonzero(lay.modes == 1)]
    order = [r for pair in zip(draft, verify) for r in pair] + draft[len(verify):] + verify[len(draft):]
    if max_rows is not None:
        order = order[:max_rows]
    g = torch.Generator().manual_seed(1)
    oracle_attn.paged_attention(torch.zeros(1, lay.num_qo_heads, 128), torch.zeros(1, 2, 16, lay.num_kv_heads, 128),
                                [0, 1], [0, 1], [0], [16])  # warm
    elapsed, nbytes, done = 0.0, 0, {"draft": 0, "verify": 0}
    for r in order:
        pages = lay.kv_indices[lay.kv_indptr[r]:lay.kv_indptr[r + 1]]
        P = len(pages)
        kv = torch.randn(P, 2, 16, lay.num_kv_heads, 128, generator=g).to(torch.bfloat16).float()
        ql = int(lay.q_lens[r])
        q = torch.randn(ql, lay.num_qo_heads, 128, generator=g).to(torch.bfloat16).float()
        kvl = int(lay.kv_lens[r])
        t0 = time.perf_counter()
        oracle_attn.paged_attention(q, kv, [0, ql], [0, P], np.arange(P, dtype=np.int32), [kvl], causal=True)
        elapsed += time.perf_counter() - t0
        # Algorithmic bytes of the row: its K/V tokens, Q in and O out, page ids.
        nbytes += kvl * lay.num_kv_heads * 128 * 2 * 2 + ql * lay.num_qo_heads * 128 * 2 * 2 + P * 4
        done["draft" if lay.modes[r] == 0 else "verify"] += 1
        if elapsed >= budget_s:
            break
    return {"value": round(nbytes / elapsed / 1e9, 3), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"oracle fp32 mixed attention, one row per call, of {done['draft']} draft + {done['verify']} "
                      f"verify rows of the bench batch ({nbytes / 1e9:.3f} GB algorithmic) in {elapsed:.1f} s"}


def reference_arm(args, rank, world):
    """The reference's attention path has no CPU implementation (its ops are CUDA
    only); the oracle port, run on the host cores, stands in for it."""
    if rank != 0:
        return
    from aspire_b200.workloads import full_context_layout
    hq, hkv = local_head_counts(CFG["num_qo_heads"], CFG["num_kv_heads"], 0, world)
    from aspire_b200.workloads import make_layout
    lay = make_layout(batch=CFG["batch"], ctx=CFG["ctx"], num_qo_heads=hq, num_kv_heads=hkv,
                      draft_fraction=CFG["draft_fraction"], budget_pages=CFG["budget_pages"],
                      pages_per_row=CFG["pages_per_row"], seed=CFG["seed"])
    full = full_context_layout(lay)
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(lay, full, budget_s=1.0, max_rows=1)
    for _ in range(max(1, args.steps)):
        vals.append(cpu_baseline(lay, full, budget_s=4.0, max_rows=4))
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "mixed draft/verify attention layer-call, Qwen3-8B heads, B=64, 32k ctx (sample)",
                       "sample_rows": "up to 4 whole rows per step, about 4 s"},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def prefill_bench(args):
    """Prefill chunks through HolisticAttentionWrapper (prefill phase of the
    tcgen05 kernel): device time per call from CUDA-graph replays, TFLOP/s over
    the visible causal (query, key) pairs, and the same inputs through
    FlashInfer's prefill wrapper when it is installed (library code: the
    comparison the reference's own prefill path would give)."""
    from aspire_b200.attention import HolisticAttentionWrapper
    dev = torch.device("cuda", 0)
    hq, hkv, d = CFG["num_qo_heads"], CFG["num_kv_heads"], 128
    try:
        import flashinfer
    except Exception:  # noqa: BLE001
        flashinfer = None
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    cases = []
    for spec in args.prefill_cases.split(","):
        rows_s, rest = spec.split("x")
        qlen_s, prefix_s = rest.split("+")
        rows, qlen, prefix = int(rows_s), int(qlen_s), int(prefix_s)
        kvl = prefix + qlen
        pages = (kvl + 15) // 16
        qo = np.arange(rows + 1, dtype=np.int32) * qlen
        kvp = np.arange(rows + 1, dtype=np.int32) * pages
        idx = np.arange(rows * pages, dtype=np.int32)
        g = torch.Generator(device=dev)
        g.manual_seed(CFG["seed"])
        q = torch.randn(rows * qlen, hq, d, generator=g, device=dev).to(torch.bfloat16)
        kv = torch.randn(rows * pages, 2, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
        t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
        w = HolisticAttentionWrapper(torch.empty(1, device=dev))
        w.plan_host(torch.from_numpy(qo), torch.from_numpy(kvp), torch.from_numpy(np.full(rows, kvl, np.int32)),
                    t(idx), hq, hkv, d, 16, causal=True)
        out = torch.empty_like(q)
        for _ in range(max(args.warmup, 1)):
            w.run(q, kv, out=out)
        torch.cuda.synchronize()
        ms = graph_time(lambda: w.run(q, kv, out=out), max(args.steps, 1), replays=3)
        # causal (bottom-right): query i of a row sees prefix + i + 1 keys; QK^T and PV, 2 flops per MAC
        pairs = rows * (qlen * prefix + qlen * (qlen + 1) / 2)
        flops = pairs * hq * d * 2 * 2
        case = {"case": spec, "ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                "frac_of_bf16_peak": round(flops / (ms * 1e-3) / 1e12 / peak, 4),
                "items": int(w.plan_info.num_items_prefill), "status": int(w.device_status())}
        if flashinfer is not None:
            ws = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
            fw = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD")
            last = np.full(rows, (kvl - 1) % 16 + 1, np.int32)
            fw.plan(t(qo), t(kvp), t(idx), t(last), hq, hkv, d, 16, causal=True, q_data_type=torch.bfloat16,
                    kv_data_type=torch.bfloat16)
            fo = fw.run(q, kv)
            torch.cuda.synchronize()
            try:
                ms_fi = graph_time(lambda: fw.run(q, kv), max(args.steps, 1), replays=3)
            except Exception:  # noqa: BLE001  (a library call that cannot be captured: time it eagerly)
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(max(args.steps, 1)):
                    fw.run(q, kv)
                b.record()
                torch.cuda.synchronize()
                ms_fi = a.elapsed_time(b) / max(args.steps, 1)
            case.update({"flashinfer_ms": round(ms_fi, 4),
                         "flashinfer_tflops": round(flops / (ms_fi * 1e-3) / 1e12, 1),
                         "max_abs_diff_vs_flashinfer": float((fo.float() - out.float()).abs().max().item())})
            del ws, fw
        cases.append(case)
        del q, kv, out, w
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "prefill", "metric": "prefill attention TFLOP/s (causal visible pairs)",
                      "unit": "TFLOP/s", "dtype": "bf16", "data": "synthetic", "heads": [hq, hkv, d],
                      "peak_bf16_tflops": peak, "cases": cases}), flush=True)


# The reference's end-to-end configs (BASELINE configs[1..3]).  Config 3's
# 4 sink pages (config 2) have no counterpart in ASPIRE's selector and are
# left out; config 4 names no draft length, so it drafts 4 like config 2.
DECODE_CFGS = {
    2: dict(model="qwen3-1.7b", batch=32, prompt=16384, new=256, draft_len=4, budget_pages=128, recent_pages=8,
            refresh_layer=2, seed=0),
    3: dict(model="qwen3-8b", batch=64, prompt=32768, new=512, draft_len=(2, 8), budget_pages=128, recent_pages=8,
            refresh_layer=-2, seed=0),
    4: dict(model="llama-3.1-8b", batch=16, prompt=81920, new=256, draft_len=4, budget_pages=256, recent_pages=8,
            refresh_layer=-2, seed=0),
}


def decode_bench(args, device, world: int, dist_on: bool) -> dict:
    """End-to-end accepted tokens/s (the metric's second half) on one of the
    reference's end-to-end configs (DECODE_CFGS; config 2 by default:
    Qwen3-1.7B shapes with random-init bf16 weights, batch 32, synthetic
    16384-token prompts, 256 generated tokens per request, fixed draft length
    4, sparse budget 128 pages + 8 recent pages, refresh layer 2), TP = the
    number of ranks (aspire_b200.spec_decode).  The prompts are prefilled,
    one decode run warms up (and captures the CUDA graphs of the step
    shapes), then a second run from the same prefill state is timed: tokens
    produced by the decode loop / its wall time with the device synchronised
    at both ends, max over ranks."""
    from aspire_b200.spec_decode import PRESETS, DenseModel, SpecDecoder, synthetic_prompts, token_sha256
    c = dict(DECODE_CFGS[args.decode_config])
    for key, arg in (("batch", args.decode_batch), ("prompt", args.decode_prompt), ("new", args.decode_new)):
        if arg is not None:
            c[key] = arg
    cfg = PRESETS[c["model"]]
    model = DenseModel(cfg, device, seed=c["seed"])
    prompts = synthetic_prompts(c["batch"], c["prompt"], cfg.vocab, seed=c["seed"])
    dec = SpecDecoder(model, batch=c["batch"], prompt_len=c["prompt"], max_new=c["new"],
                      draft_len=c["draft_len"], budget_pages=c["budget_pages"], recent_pages=c["recent_pages"],
                      refresh_layer=c["refresh_layer"], draft_seed=c["seed"])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g0 = dec.prefill(prompts)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    warm = dec.generate()
    dec.restart(g0)
    r = dec.generate()
    same = bool(np.array_equal(warm["tokens"], r["tokens"]))
    secs = torch.tensor([r["seconds"], prefill_s], device=device)
    if dist_on:
        torch.distributed.all_reduce(secs, op=torch.distributed.ReduceOp.MAX)
    dec_s, pre_s = float(secs[0].item()), float(secs[1].item())
    steps = sum(r["steps"].values())
    out = {"config": args.decode_config, "model": c["model"] + " shapes, random-init bf16 weights",
           "batch": c["batch"], "prompt_tokens": c["prompt"], "new_tokens": c["new"],
           "draft_len": list(c["draft_len"]) if isinstance(c["draft_len"], tuple) else c["draft_len"],
           "budget_pages": c["budget_pages"], "recent_pages": c["recent_pages"], "refresh_layer": c["refresh_layer"],
           "tp": world, "accepted_tokens_per_s": round(r["decoded_tokens"] / dec_s, 1),
           "decode_s": round(dec_s, 3), "prefill_s": round(pre_s, 2),
           "prefill_tokens_per_s": round(c["batch"] * c["prompt"] / pre_s, 1),
           "steps": r["steps"], "ms_per_step": round(1e3 * dec_s / max(steps, 1), 3),
           "device_ms_per_step": r["device_ms_per_step"],
           "mean_accepted_drafts_per_verify": round(r["accepted_drafts"] / max(r["verify_rows"], 1), 3),
           "tokens_per_row_per_step": round(r["decoded_tokens"] / max(steps, 1) / c["batch"], 3),
           "repeat_identical": same, "token_sha256": token_sha256(r["tokens"]),
           "cuda_graphs": dec.use_graphs, "data": "synthetic uniform tokens in [100, vocab), no EOS"}
    del dec, model
    torch.cuda.empty_cache()
    return out


def sweep_bench(args):
    """The reference's config-5 sweep: mixed attention
    plus top-k page selection alone at Qwen3-8B heads (32 / 8 / 128).

    Grid: context in --sweep-ctx x batch in --sweep-batch x drafting fraction
    {0, 0.5, 1} x verify q_len {1, 5, 9} (when some rows verify) x budget
    {64, 512} pages (when some rows draft; capped at the context's pages).
    Every point plans its batch, then times a CUDA graph of back-to-back
    attention calls in page-table mode (arange block tables as the reference
    engine lays them out; draft rows' selected pages scattered over their
    context).  A point whose KV bytes are below 256 MB cycles through copies
    of its page tables shifted to disjoint page ranges of one large cache, so
    that consecutive calls read different memory and nothing is served from
    L2.  The selection is the top-k stage (aspire_select_pages on fp32 page
    scores) over the same batch, with page scores from mean-pooled keys:
    score[b, p] = max_h q_last[b, h] . mean_t K[b, p, t, kv(h)] (fp32,
    computed once per point outside the timing).  Reported per point:
    attention ms and GB/s (algorithmic bytes: KV read once, Q in, O out, page
    ids), selection ms, attention + selection GB/s, fraction of the measured
    HBM peak."""
    from aspire_b200.attention import HolisticAttentionWrapper
    from aspire_b200.page_selector import PageSelectorFirstLastAvg
    from aspire_b200.workloads import make_layout

    dev = torch.device("cuda", 0)
    hq, hkv = CFG["num_qo_heads"], CFG["num_kv_heads"]
    peak, peak_kind = measured_peaks()
    ctxs = [int(x) for x in args.sweep_ctx.split(",")]
    batches = [int(x) for x in args.sweep_batch.split(",")]
    ppr_of = lambda ctx: (ctx + 512 + 15) // 16  # noqa: E731  (context plus generation headroom)
    max_pages = max(b * ppr_of(c) for b in batches for c in ctxs)
    target = 256 << 20  # bytes cycled per call at least (2x the L2)
    page_bytes = 2 * 16 * hkv * 128 * 2
    total_pages = max(max_pages, (2 * target) // page_bytes + 1)
    kv = torch.empty(total_pages, 2, 16, hkv, 128, dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(CFG["seed"])
    step = 1 << 14
    for p0 in range(0, total_pages, step):
        p1 = min(total_pages, p0 + step)
        kv[p0:p1] = torch.randn(p1 - p0, 2, 16, hkv, 128, generator=gen, device=dev).to(torch.bfloat16)
    ws = torch.empty(1, device=dev)
    w = HolisticAttentionWrapper(ws)
    points = []
    t_start = time.perf_counter()
    for ctx in ctxs:
        ppr = ppr_of(ctx)
        ctx_pages = (ctx + 15) // 16
        budgets = sorted({min(b, ctx_pages) for b in (64, 512)})
        for B in batches:
            for frac in (0.0, 0.5, 1.0):
                qls = (1, 5, 9) if frac < 1.0 else (None,)
                buds = budgets if frac > 0.0 else (None,)
                for ql in qls:
                    for bud in buds:
                        lay = make_layout(batch=B, ctx=ctx, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=frac,
                                          verify_q_len=ql if ql is not None else 1,
                                          budget_pages=bud if bud is not None else 64, pages_per_row=ppr,
                                          seed=CFG["seed"], block_table="arange")
                        points.append(_sweep_point(w, kv, lay, ctx, B, frac, ql, bud, total_pages, target, peak,
                                                   PageSelectorFirstLastAvg, args))
    worst = sorted(points, key=lambda p: p["attn_frac"])[:8]
    fr = [p["attn_frac"] for p in points]
    print(json.dumps({"workload": "sweep", "metric": "mixed attention + page selection HBM GB/s per point",
                      "unit": "GB/s", "peak": peak, "peak_source": peak_kind, "dtype": "bf16", "data": "synthetic",
                      "heads": [hq, hkv, 128], "n_points": len(points),
                      "attn_frac_median": round(statistics.median(fr), 4), "attn_frac_min": round(min(fr), 4),
                      "wall_s": round(time.perf_counter() - t_start, 1), "worst": worst, "points": points}),
          flush=True)


def _sweep_point(w, kv, lay, ctx, B, frac, ql, bud, total_pages, target, peak, selector_cls, args):
    dev = kv.device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
    nbytes = lay.algorithmic_bytes()
    span = lay.batch * lay.pages_per_row  # pages one copy of the tables addresses
    copies = int(max(1, min(math.ceil(target / max(nbytes, 1)), total_pages // span, 64)))
    counts = np.diff(lay.kv_indptr)
    draft_tab = np.zeros((lay.batch, max(1, int(counts.max()))), np.int32)
    for b in range(lay.batch):
        if lay.modes[b] == 0:
            draft_tab[b, :counts[b]] = lay.kv_indices[lay.kv_indptr[b]:lay.kv_indptr[b + 1]]
    modes = t(lay.modes).to(dev)
    tables = [(modes, (t(draft_tab) + c * span).to(dev), (t(lay.block_table) + c * span).to(dev))
              for c in range(copies)]
    q = torch.randn(lay.total_q, lay.num_qo_heads, 128, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    w.set_page_tables(*tables[0])
    w.plan_host(t(lay.qo_indptr), t(lay.kv_indptr), t(lay.kv_lens), None, lay.num_qo_heads, lay.num_kv_heads, 128, 16,
                causal=True)
    # Page scores from mean-pooled keys (fp32), then the top-k stage alone.
    pages = torch.from_numpy(lay.block_table.astype(np.int64)).to(dev)          # [B, ppr]
    last_q = q[torch.from_numpy(lay.qo_indptr[1:] - 1).long().to(dev)].float()  # [B, Hq, 128]
    g = lay.num_qo_heads // lay.num_kv_heads
    scores = torch.empty(lay.batch, lay.pages_per_row, dtype=torch.float32, device=dev)
    for b in range(lay.batch):  # one row at a time keeps the fp32 temporary small
        kmean = kv[pages[b], 0].float().mean(dim=1)                             # [ppr, Hkv, 128]
        sc = torch.einsum("kgd,pkd->kgp", last_q[b].view(lay.num_kv_heads, g, 128), kmean)
        scores[b] = sc.amax(dim=(0, 1))
    del kmean, sc
    k_sel = int(bud) if bud is not None else 64
    sel = selector_cls(max_batch_size=lay.batch, pages_per_slot=lay.pages_per_row, subset_cache_size=k_sel,
                       L=CFG["L"], n_heads=lay.num_qo_heads, page_size=16, max_seq_length=lay.pages_per_row * 16,
                       device=dev, bsz=lay.batch, dec_len=9, kv_stride=lay.pages_per_row * 16, draft_percent=None,
                       min_draft_pages=k_sel)
    num_pages = t((lay.ctx_lens + 15) // 16).to(dev)
    table_out = torch.zeros(lay.batch, k_sel, dtype=torch.int32, device=dev)
    counts_out = torch.zeros(lay.batch, dtype=torch.int32, device=dev)
    bt = t(lay.block_table).to(dev)
    state = {"i": 0}

    def attn():
        i = state["i"] % copies
        state["i"] += 1
        w.set_page_tables(*tables[i])
        w.run(q, kv, out=out)

    def select():
        sel.finalize_scores_into(table_out, counts_out, scores, num_pages, bt)

    reps = int(max(copies, min(200, math.ceil(2.0e9 / max(nbytes, 1)))))
    reps = (reps + copies - 1) // copies * copies
    attn_ms = graph_time(attn, reps, replays=2)
    sel_ms = graph_time(select, 100, replays=2)
    status = int(w.device_status())
    sel_bytes = lay.batch * lay.pages_per_row * 4 + lay.batch * k_sel * 4 * 2
    gbps = nbytes / (attn_ms * 1e-3) / 1e9
    both = (nbytes + sel_bytes) / ((attn_ms + sel_ms) * 1e-3) / 1e9
    return {"ctx": ctx, "batch": B, "draft_fraction": frac, "verify_q_len": ql, "budget_pages": bud,
            "attn_bytes": int(nbytes), "attn_ms": round(attn_ms, 5), "attn_GBps": round(gbps, 1),
            "attn_frac": round(gbps / peak, 4), "select_ms": round(sel_ms, 5), "attn_select_GBps": round(both, 1),
            "attn_select_frac": round(both / peak, 4), "items": int(w.plan_info.num_items_tc),
            "chunk": int(w.plan_info.chunk_tokens), "copies": copies, "status": status}


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.workload == "decode":
        dist_on = world > 1
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
        if dist_on:
            import datetime
            torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
        from aspire_b200 import load_library
        load_library()
        res = decode_bench(args, device, world, dist_on)
        if rank == 0:
            print(json.dumps({"workload": "decode", "metric": "accepted tokens/s per box", **res}), flush=True)
        if dist_on:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    if args.workload in ("prefill", "sweep"):
        from aspire_b200 import load_library
        load_library()
        torch.cuda.set_device(0)
        (prefill_bench if args.workload == "prefill" else sweep_bench)(args)
        return
    dist_on = world > 1
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if dist_on:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))

    from aspire_b200 import load_library
    load_library()
    lay, full, lpl_m, lpl_f = build_workload(device, rank, world)
    hp = HotPath(device, lay, full, lpl_m, lpl_f, fused_append=not args.separate_append)
    hp.plan()
    hp.capture()
    sb = step_bytes(lay, full, CFG["n_layer"], hp.kv_stride, hp.k_sel)

    peak, peak_kind = measured_peaks()
    with ClockSampler(device) as clocks:
        ms = time_device(hp.graph.replay, args.steps, args.warmup, dist_on)
    t = torch.tensor([ms], device=device)
    tot_bytes = torch.tensor([float(sb["total"])], device=device)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(tot_bytes, op=torch.distributed.ReduceOp.SUM)
    ms_max = float(t.item())
    value = float(tot_bytes.item()) / (ms_max * 1e-3) / 1e9

    roof = kernel_roofline(hp, args.steps, peak, peak_kind)
    parts = breakdown(hp)
    parts["refresh_attention_GBps"] = round(sb["refresh"] / (parts["refresh_attention_ms"] * 1e-3) / 1e9, 1)
    parts["mixed_attention_GBps"] = round(sb["mixed"] / (parts["mixed_attention_ms"] * 1e-3) / 1e9, 1)
    parts["mixed_attention_random_tables_GBps"] = round(
        sb["mixed"] / (parts["mixed_attention_random_tables_ms"] * 1e-3) / 1e9, 1)
    parts["refresh_attention_random_tables_GBps"] = round(
        sb["refresh"] / (parts["refresh_attention_random_tables_ms"] * 1e-3) / 1e9, 1)
    parts["tc_items"] = [hp.mixed.plan_info.num_items_tc, hp.refresh.plan_info.num_items_tc]
    parts["gather_items"] = [hp.mixed.plan_info.num_items_gather, hp.refresh.plan_info.num_items_gather]
    check = check_step(hp)
    e2e = None
    if not args.no_e2e:
        dt, h2d, d2h = e2e_measure(hp, max(2, args.steps // 2), 1, sb["total"])
        tt = torch.tensor([dt], device=device)
        if dist_on:
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e = {"value": round(float(tot_bytes.item()) / float(tt.item()) / 1e9, 1), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(float(tt.item()) * 1e3, 3)}
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(lay, full, budget_s=12.0)
    launches = hp.launches_per_step() * args.steps
    decode = None
    if not args.no_decode:
        hp.graph = None
        del hp
        torch.cuda.empty_cache()
        decode = decode_bench(args, device, world, dist_on)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "one decode step of the attention hot path: 35 x (append + mixed draft/verify "
                                   "attention) + refresh layer (append + full attention + first/last dump) + page "
                                   "selection; Qwen3-8B heads 32/8/128, 36 layers, B=64, 32k ctx, draft fraction 0.5, "
                                   "verify q_len U{3..9}, budget 128 pages, one resident layer cache; pages read "
                                   "straight from the draft / block tables (page-list build absorbed); "
                                   + ("append as its own kernel" if args.separate_append
                                      else "append inside the attention launch"),
                       "batch": CFG["batch"], "ctx": CFG["ctx"], "tp": world, "heads_per_rank": [lay.num_qo_heads, lay.num_kv_heads],
                       "l2": "inputs larger than L2 (8.7 GB cache at TP1)", "bytes_per_step": sb},
            "roofline": roof, "breakdown": parts, "clocks": clocks.summary(), "e2e": e2e, "check": check,
            "gpu_launches": launches,
            "cpu_baseline": cb, "decode": decode,
        }
        print(json.dumps(line), flush=True)
    if dist_on:
        if args.no_decode:
            hp.graph = None
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
