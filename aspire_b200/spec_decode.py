"""Self-speculative decoding over the hot-path ops: accepted tokens/s and the
greedy-identity check, end to end.

This is the measurement harness the hot path is judged by, not a rebuild of
ASPIRE's engine.  It drives a dense decoder with random-init bf16 weights of
the reference's model shapes (Qwen3-1.7B / Qwen3-8B / Llama-3.1-8B geometry)
through exactly the calls the engine makes on the path:

* per layer: ``qkv_prologue`` (q/k RMSNorm + interleaved RoPE + paged append,
  the engine's ``q_norm``/``k_norm``, ``mylib::rope`` and
  ``mylib::update_kv_padded``) and ``HolisticAttentionWrapper.run``: the mixed
  draft/verify attention, or at the refresh layer the full-context attention
  with the first/last logit dump;
* per step, ahead of the forward: page re-selection for every row from the
  previous step's dump (``PageSelectorFirstLastAvg.select_into``, as
  ``LMBackendBase._prepare_replan_state`` runs it every step,
  aspire/backends/base.py:708-716) and the draft-page spill
  (``draft_page_spill``, base.py:1222-1236);
* after prefill: recent-page seeding of the draft tables
  (``seed_recent_into``, base.py:1522-1556).

The step loop follows the reference runtime's greedy path
(aspire/engine/runtime.py:579-866) under the fixed-draft policy
(``--method aspire-fixed --fixed-draft D``): a row drafts one token per step
(q_len 1, sparse attention over its draft table) until it holds D drafted
tokens, then verifies them (q_len D + 1, full causal attention); it accepts
the longest prefix of drafts equal to the target's greedy outputs and
commits it plus the target's next token (runtime.py:765-783:
``accepted = matches.cumprod(dim=1).sum(dim=1)``).  Every row of the batch
is in the one mixed forward.  The KV cache uses the engine's layout
(``[pages, 2, 16, Hkv, 128]`` per layer, row r owning pages
[r * pps, (r + 1) * pps)), page size 16.

Everything outside the path (GEMMs, norms, SwiGLU, embedding, argmax,
NCCL all-reduces of the tensor-parallel model) is plain torch; the mixed
forward of each step shape is replayed as one CUDA graph, as the reference
runs it.  Under torch.distributed each rank holds its tensor-parallel shard
(KV-head ranges as aspire/tp.py:35-51 shards wqkv, row-parallel wo / w2,
column-parallel w13, vocab-parallel output) and the per-layer all-reduces
run over NCCL (sparse_draft_transformer.py:177, transformer.py:501); the
argmax across vocabulary shards follows sparse_draft_transformer.py:268-281.

Synthetic data: prompts of uniform random tokens in [100, vocab) (the
semantics of aspire.data.synthetic_dataset), no EOS (every row generates
exactly ``max_new`` tokens), weights N(0, 0.02), norm weights 1.
"""

from __future__ import annotations

import hashlib
import json
import math
import time
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from .attention import HolisticAttentionWrapper, first_last_dump_jit_args
from .kv_ops import draft_page_spill, qkv_prologue
from .page_selector import PageSelectorFirstLastAvg
from .tp import tp_heads

PAGE = 16
HEAD_DIM = 128


@dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layer: int
    dim: int
    n_head: int
    n_kv_head: int
    intermediate: int
    vocab: int
    rope_theta: float
    qk_norm: bool
    norm_eps: float = 1e-6
    rope_scale: float = 1.0
    llama31: Optional[tuple] = None  # (low_freq_factor, high_freq_factor, old_context_len)


PRESETS = {
    "qwen3-1.7b": ModelConfig("qwen3-1.7b", 28, 2048, 16, 8, 6144, 151936, 1e6, True),
    "qwen3-8b": ModelConfig("qwen3-8b", 36, 4096, 32, 8, 12288, 151936, 1e6, True),
    "llama-3.1-8b": ModelConfig("llama-3.1-8b", 32, 4096, 32, 8, 14336, 128256, 5e5, False, 1e-5, 8.0,
                                (1.0, 4.0, 8192.0)),
}


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm as one fused torch kernel.  The reference normalises in fp32,
    casts back and then scales by the weight; the fused kernel scales in fp32
    before the cast, which gives the same values for the unit weights this
    harness uses."""
    return torch.rms_norm(x, (x.shape[-1],), w, eps)


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


class DenseModel:
    """Random-init decoder of a preset's shapes, holding this rank's shard."""

    def __init__(self, cfg: ModelConfig, device: torch.device, *, seed: int = 0, n_layer: Optional[int] = None):
        self.cfg = cfg
        self.device = device
        d = _dist()
        self.rank = d.get_rank() if d else 0
        self.world = d.get_world_size() if d else 1
        self.n_layer = n_layer or cfg.n_layer
        kv = tp_heads(cfg.n_kv_head, self.rank, self.world)
        g = cfg.n_head // cfg.n_kv_head
        self.hkv = len(kv)
        self.hq = self.hkv * g
        qcols = slice(kv.start * g * HEAD_DIM, kv.stop * g * HEAD_DIM)
        kvcols = slice(kv.start * HEAD_DIM, kv.stop * HEAD_DIM)
        inter = tp_heads(cfg.intermediate, self.rank, self.world)
        self.inter_local = len(inter)
        voc = tp_heads(cfg.vocab, self.rank, self.world)
        self.vocab_start = voc.start
        self.vocab_local = len(voc)

        def randn(shape, s):  # the full tensor, identical on every rank
            gen = torch.Generator(device=device)
            gen.manual_seed(seed * 1_000_003 + s)
            return (torch.randn(shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)

        D, I, Hq, Hkv = cfg.dim, cfg.intermediate, cfg.n_head, cfg.n_kv_head
        self.emb = randn((cfg.vocab, D), 1)
        self.w_out = randn((D, cfg.vocab), 2)[:, voc.start:voc.stop].contiguous()
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)  # noqa: E731
        self.final_norm = ones(D)
        self.layers = []
        for l in range(self.n_layer):
            s = 100 + 16 * l
            wq = randn((D, Hq * HEAD_DIM), s)[:, qcols]
            wk = randn((D, Hkv * HEAD_DIM), s + 1)[:, kvcols]
            wv = randn((D, Hkv * HEAD_DIM), s + 2)[:, kvcols]
            wo = randn((Hq * HEAD_DIM, D), s + 3)[qcols, :]
            w1 = randn((D, I), s + 4)[:, inter.start:inter.stop]
            w3 = randn((D, I), s + 5)[:, inter.start:inter.stop]
            w2 = randn((I, D), s + 6)[inter.start:inter.stop, :]
            self.layers.append(dict(
                wqkv=torch.cat([wq, wk, wv], dim=1).contiguous(), wo=wo.contiguous(),
                w13=torch.cat([w1, w3], dim=1).contiguous(), w2=w2.contiguous(),
                attn_norm=ones(D), ffn_norm=ones(D),
                q_norm=ones(HEAD_DIM) if cfg.qk_norm else None, k_norm=ones(HEAD_DIM) if cfg.qk_norm else None))
            del wq, wk, wv, wo, w1, w3, w2

    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        d = _dist()
        if d is not None and self.world > 1:
            d.all_reduce(t)
        return t

    def forward(self, tokens: torch.Tensor, attn) -> torch.Tensor:
        """Hidden states after the final norm; `attn(layer, q, k, v)` returns
        the attention output [T, hq, 128] (and does the prologue / append)."""
        cfg = self.cfg
        T = tokens.shape[0]
        hq, hkv = self.hq, self.hkv
        x = F.embedding(tokens, self.emb)
        for l, w in enumerate(self.layers):
            h = rms_norm(x, w["attn_norm"], cfg.norm_eps)
            qkv = h @ w["wqkv"]
            q = qkv[:, :hq * HEAD_DIM].view(T, hq, HEAD_DIM)
            k = qkv[:, hq * HEAD_DIM:(hq + hkv) * HEAD_DIM].view(T, hkv, HEAD_DIM)
            v = qkv[:, (hq + hkv) * HEAD_DIM:].view(T, hkv, HEAD_DIM)
            o = attn(l, q, k, v).reshape(T, hq * HEAD_DIM)
            # One GEMM with the residual add in its epilogue on one GPU; with
            # shards the partial products are summed first.
            x = torch.addmm(x, o, w["wo"]) if self.world == 1 else x + self._all_reduce(o @ w["wo"])
            h = rms_norm(x, w["ffn_norm"], cfg.norm_eps)
            gu = h @ w["w13"]
            a = F.silu(gu[:, :self.inter_local]).mul_(gu[:, self.inter_local:])
            x = torch.addmm(x, a, w["w2"]) if self.world == 1 else x + self._all_reduce(a @ w["w2"])
        return rms_norm(x, self.final_norm, cfg.norm_eps)

    def greedy(self, x: torch.Tensor) -> torch.Tensor:
        """Greedy ids [T] over the whole vocabulary: a local max per rank,
        then the rank with the largest value (lowest rank on ties), as
        sparse_draft_transformer.py:268-281 merges the shards."""
        logits = x @ self.w_out
        vals, ids = logits.max(dim=-1)
        ids = ids + self.vocab_start
        if self.world == 1:
            return ids
        T = x.shape[0]
        all_v = torch.zeros(T, self.world, dtype=vals.dtype, device=x.device)
        all_i = torch.zeros(T, self.world, dtype=torch.long, device=x.device)
        all_v[:, self.rank] = vals
        all_i[:, self.rank] = ids
        self._all_reduce(all_v)
        self._all_reduce(all_i)
        sel = torch.argmax(all_v, dim=-1, keepdim=True)
        return torch.gather(all_i, 1, sel).squeeze(1)

    def token_logit_stats(self, x: torch.Tensor, emitted: torch.Tensor):
        """(top-1 id, top-1 logit, top-2 logit, logit of `emitted`) per row of
        x, over the whole vocabulary (fp32; shards merged by all-reduce)."""
        logits = (x @ self.w_out).float()
        top = logits.topk(2, dim=-1)
        T = x.shape[0]
        vals = torch.zeros(T, self.world, 2, device=x.device)
        ids = torch.zeros(T, self.world, dtype=torch.long, device=x.device)
        vals[:, self.rank] = top.values
        ids[:, self.rank] = top.indices[:, 0] + self.vocab_start
        local = emitted - self.vocab_start
        own = (local >= 0) & (local < self.vocab_local)
        e = torch.where(own, logits.gather(1, local.clamp(0, self.vocab_local - 1)[:, None])[:, 0],
                        torch.zeros(T, device=x.device))
        if self.world > 1:
            self._all_reduce(vals)
            self._all_reduce(ids)
            self._all_reduce(e)
        flat = vals.reshape(T, -1)
        best = flat.topk(2, dim=-1).values
        r = torch.argmax(vals[:, :, 0], dim=-1, keepdim=True)
        return torch.gather(ids, 1, r)[:, 0], best[:, 0], best[:, 1], e


def step_shape(n: np.ndarray, dcnt: np.ndarray, active: np.ndarray, draft_len, budget_pages: int) -> dict:
    """Per-row shape of one fixed-draft step (host arrays).

    n: committed tokens in the cache; dcnt: drafted tokens pending; active:
    rows still generating.  A row verifies when it holds draft_len drafts
    (one length for every row, or an array of per-row lengths)
    (q_len dcnt + 1 at positions n..), else drafts one token at position
    n + dcnt.  ``end`` is the row's length once this step's tokens are
    appended.  Draft rows attend their draft table: after the step's
    re-selection it lists min(ceil(end / 16), budget) pages ending with the
    page of position end - 1 (the forced recent pages), so their mixed
    length is (count - 1) * 16 + last_page_len; verify rows attend their
    block-table prefix.  Finished rows take part with q_len 0."""
    verify = active & (dcnt == draft_len)
    draft = active & ~verify
    qlen = np.where(verify, dcnt + 1, np.where(draft, 1, 0))
    start = np.where(draft, n + dcnt, n)
    end = np.where(active, n + dcnt + 1, n)
    full_pages = (end + PAGE - 1) // PAGE
    counts = np.minimum(full_pages, budget_pages)
    last = np.where(end > 0, (end - 1) % PAGE + 1, 0)
    return dict(verify=verify, draft=draft, qlen=qlen, start=start, end=end, full_pages=full_pages,
                last=last, mixed_pages=np.where(draft, counts, full_pages),
                mixed_len=np.where(draft, (counts - 1) * PAGE + last, end),
                qo=np.concatenate([[0], np.cumsum(qlen)]))


def accept(drafts: np.ndarray, target: np.ndarray) -> int:
    """Length of the longest prefix of `drafts` equal to the target's greedy
    outputs (runtime.py:765-783)."""
    acc = 0
    while acc < len(drafts) and drafts[acc] == target[acc]:
        acc += 1
    return acc


class SpecDecoder:
    """Batched self-speculative decoding of one batch of equal-length prompts.
    ``draft_len`` is the fixed draft length of every row (``0`` gives plain
    greedy decoding: every step a q_len-1 full-attention step through the
    same ops), or a ``(lo, hi)`` range: each row draws its next draft length
    uniformly from it after every verification (seeded by ``draft_seed``), so
    the rows drift apart and steps mix drafting and verifying rows, as the
    reference's asynchronous scheduling interleaves them."""

    def __init__(self, model: DenseModel, *, batch: int, prompt_len: int, max_new: int, draft_len,
                 budget_pages: int, recent_pages: int = 8, refresh_layer: int = -2, use_graphs: bool = True,
                 prefill_chunk: int = 8192, draft_seed: int = 0):
        cfg = model.cfg
        dev = model.device
        self.model, self.dev = model, dev
        self.draft_range = tuple(draft_len) if isinstance(draft_len, (tuple, list)) else None
        self.draft_seed = draft_seed
        draft_len = self.draft_range[1] if self.draft_range else int(draft_len)
        self.B, self.P, self.G, self.D = batch, prompt_len, max_new, draft_len
        self.pps = (prompt_len + max_new + draft_len + 2 * PAGE - 1) // PAGE
        self.kv_stride = self.pps * PAGE
        self.k_sel = budget_pages
        self.L = recent_pages
        self.refresh_layer = refresh_layer % model.n_layer
        self.use_graphs = use_graphs
        self.prefill_chunk = prefill_chunk
        hq, hkv, B = model.hq, model.hkv, batch
        i32 = dict(dtype=torch.int32, device=dev)
        self.caches = [torch.zeros(B * self.pps, 2, PAGE, hkv, HEAD_DIM, dtype=torch.bfloat16, device=dev)
                       for _ in range(model.n_layer)]
        self.block_table = torch.arange(B * self.pps, **i32).view(B, self.pps)
        self.draft_table = torch.zeros(B, budget_pages + 8, **i32)
        self.draft_counts = torch.zeros(B, **i32)
        self.full_modes = torch.ones(B, **i32)
        self.t_max = B * (draft_len + 1)
        # Tokens stay on the device: tok_dev[b * (D + 1) + j] is row b's last
        # committed token (j = 0) or its j-th draft; the last element is a
        # sink for the outputs of tokens that store nothing.
        self.tok_dev = torch.zeros(B * (draft_len + 1) + 1, **i32)
        self.sink = B * (draft_len + 1)
        # Per-step host metadata, uploaded with one copy into views of one
        # device buffer, from a ring of pinned staging buffers (the host plans
        # a step while earlier ones still run).
        fields = [("tok_src", self.t_max), ("tok_dst", self.t_max), ("tok0", B), ("qo", B + 1), ("qo_prev", B + 1),
                  ("rope", B), ("mixed_indptr", B + 1), ("mixed_last", B), ("modes", B), ("num_pages", B),
                  ("dec_lens", B), ("draft_lens", B)]
        self._fields = fields
        n = sum(s for _, s in fields)
        self._stage = [torch.zeros(n, dtype=torch.int32, pin_memory=True) for _ in range(8)]
        self._stage_ev = [None] * len(self._stage)
        self._stage_slot = 0
        self._dev = torch.zeros(n, **i32)
        self.d = {}
        off = 0
        for name, size in fields:
            self.d[name] = self._dev[off:off + size]
            off += size
        self.dump = torch.full((B * hq * 2 * self.kv_stride,), float("-inf"), dtype=torch.float16, device=dev)
        self.lse = torch.zeros(self.t_max, hq, dtype=torch.float32, device=dev)
        self.q_rot = torch.zeros(self.t_max, hq, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self.attn_out = torch.zeros(self.t_max, hq, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self.out_ids = torch.zeros(self.t_max, dtype=torch.long, device=dev)
        ws = torch.empty(1, device=dev)
        self.mixed = HolisticAttentionWrapper(ws)
        self.mixed.set_page_tables(self.d["modes"], self.draft_table, self.block_table)
        self.refresh = HolisticAttentionWrapper(ws, jit_args=first_last_dump_jit_args())
        self.refresh.set_page_tables(self.full_modes, self.draft_table, self.block_table)
        self.prefill_w = HolisticAttentionWrapper(ws)
        self.selector = PageSelectorFirstLastAvg(
            max_batch_size=B, pages_per_slot=self.pps, subset_cache_size=budget_pages, L=recent_pages, n_heads=hq,
            page_size=PAGE, max_seq_length=self.kv_stride, device=dev, bsz=B, dec_len=draft_len + 1,
            kv_stride=self.kv_stride, draft_percent=None, min_draft_pages=budget_pages)
        self.graphs: dict = {}
        self.rope_kw = dict(rope_theta=cfg.rope_theta, rope_scale=cfg.rope_scale, llama31=cfg.llama31,
                            norm_eps=cfg.norm_eps)

    # ---------------------------------------------------------------- prefill
    def _prefill_attn(self, slot: int, c0: int, c1: int):
        """Attention callback of one prefill chunk of `slot`: positions [c0, c1)
        after a prefix of c0 tokens, causal, through the block table."""
        t = lambda a: torch.tensor(a, dtype=torch.int32)  # noqa: E731
        pages = (c1 + PAGE - 1) // PAGE
        qo, kvp, kvl = t([0, c1 - c0]), t([0, pages]), t([c1])
        dev = lambda a: a.to(self.dev)  # noqa: E731
        qo_d, kvp_d, last_d, rope_d = dev(qo), dev(kvp), dev(t([(c1 - 1) % PAGE + 1])), dev(t([c0]))
        tables = (self.full_modes[slot:slot + 1], self.draft_table[slot:slot + 1], self.block_table[slot:slot + 1])
        self.prefill_w.set_page_tables(*tables)
        m = self.model
        self.prefill_w.plan_host(qo, kvp, kvl, None, m.hq, m.hkv, HEAD_DIM, PAGE, causal=True)

        def attn(l, q, k, v):
            w = m.layers[l]
            q_rot = qkv_prologue(q, k, v, qo_d, rope_d, self.caches[l], None, kvp_d, last_d, PAGE,
                                 q_norm_weight=w["q_norm"], k_norm_weight=w["k_norm"], page_tables=tables,
                                 **self.rope_kw)
            return self.prefill_w.run(q_rot, self.caches[l])
        return attn

    def _run_slot(self, slot: int, tokens: torch.Tensor, start: int):
        """Forward of `tokens` of one slot at positions [start, start + len),
        chunked; returns the final hidden states."""
        outs = []
        for c0 in range(0, tokens.shape[0], self.prefill_chunk):
            c1 = min(tokens.shape[0], c0 + self.prefill_chunk)
            attn = self._prefill_attn(slot, start + c0, start + c1)
            outs.append(self.model.forward(tokens[c0:c1], attn))
        return torch.cat(outs)

    def prefill(self, prompts: torch.Tensor) -> np.ndarray:
        """Chunked prefill of every slot (prompts [B, P] int); returns the
        first generated token of each row (the target's greedy choice after
        the prompt) and seeds the draft tables with recent pages."""
        firsts = []
        for s in range(self.B):
            x = self._run_slot(s, prompts[s].to(self.dev, torch.int32), 0)
            firsts.append(self.model.greedy(x[-1:]))
        g0 = torch.cat(firsts).cpu().numpy()
        self._reset_decode_state(g0)
        return g0

    def restart(self, g0: np.ndarray) -> None:
        """Back to the state right after prefill (the prompt's cache is kept;
        positions past the prompt are rewritten before they are attended)."""
        self._reset_decode_state(g0)

    def _reset_decode_state(self, g0: np.ndarray):
        B, D = self.B, self.D
        self.n = np.full(B, self.P, np.int64)      # committed tokens in the cache
        self.dcnt = np.zeros(B, np.int64)          # drafted tokens pending verification
        self.tok0 = np.asarray(g0, np.int64).copy()  # last committed token of each row (not yet in the cache)
        self._rng = np.random.default_rng(self.draft_seed)
        self.dtarget = self._draw_targets(B)      # drafts each row makes before verifying
        self.out = [[int(g0[b])] for b in range(B)]
        self.tok_dev.zero_()
        self.step_no = 0
        self.prev_qo = None
        self.dump.fill_(float("-inf"))
        self.lse.zero_()
        num_pages = torch.from_numpy(((self.n + 1 + PAGE - 1) // PAGE).astype(np.int32)).to(self.dev)
        self.draft_table.zero_()
        self.selector.seed_recent_into(self.draft_table, self.draft_counts, num_pages, self.block_table)

    def _draw_targets(self, n: int) -> np.ndarray:
        if self.draft_range is None:
            return np.full(n, self.D, np.int64)
        lo, hi = self.draft_range
        return self._rng.integers(lo, hi + 1, size=n).astype(np.int64)

    # ------------------------------------------------------------------ steps
    def _attn_step(self, l, q, k, v):
        m = self.model
        T = q.shape[0]
        w = m.layers[l]
        tables = (self.d["modes"], self.draft_table, self.block_table)
        q_rot = qkv_prologue(q, k, v, self.d["qo"], self.d["rope"], self.caches[l], None, self.d["mixed_indptr"],
                             self.d["mixed_last"], PAGE, q_norm_weight=w["q_norm"], k_norm_weight=w["k_norm"],
                             q_out=self.q_rot[:T], page_tables=tables, **self.rope_kw)
        out = self.attn_out[:T]
        if l == self.refresh_layer:
            self.refresh.run(q_rot, self.caches[l], self.dump, m.hq, self.kv_stride, out=out, lse=self.lse[:T])
        else:
            self.mixed.run(q_rot, self.caches[l], out=out)
        return out

    def _body(self, T: int, select: bool):
        if select:
            self.selector.select_into(self.draft_table, self.draft_counts, self.dump, self.lse, self.d["num_pages"],
                                      self.block_table, self.d["qo_prev"])
            draft_page_spill(self.d["modes"], self.d["dec_lens"], self.d["draft_lens"], self.draft_table,
                             self.draft_counts, self.block_table)
        D1 = self.D + 1
        self.tok_dev[:self.sink].view(self.B, D1)[:, 0].copy_(self.d["tok0"])
        tokens = self.tok_dev.index_select(0, self.d["tok_src"][:T])
        x = self.model.forward(tokens, self._attn_step)
        ids = self.model.greedy(x)
        self.out_ids[:T].copy_(ids)
        # A draft row's proposal becomes its next draft token on the device.
        self.tok_dev.index_copy_(0, self.d["tok_dst"][:T].long(), ids.to(torch.int32))

    def _schedule(self):
        """Host side of one step: modes, lengths, plans and uploads (no sync)."""
        B = self.B
        active = np.array([len(o) < self.G for o in self.out])
        s = step_shape(self.n, self.dcnt, active, self.dtarget, self.k_sel)
        verify, draft, qlen, start, end = s["verify"], s["draft"], s["qlen"], s["start"], s["end"]
        full_pages, last, mixed_pages, mixed_len, qo = (s["full_pages"], s["last"], s["mixed_pages"],
                                                        s["mixed_len"], s["qo"])
        T = int(qo[-1])
        slot = self._stage_slot
        if self._stage_ev[slot] is not None:
            self._stage_ev[slot].synchronize()
        h, off = {}, 0
        for name, size in self._fields:
            h[name] = self._stage[slot][off:off + size].numpy()
            off += size
        D1 = self.D + 1
        src, dst = [], []
        for b in range(B):
            if verify[b]:
                src.extend(b * D1 + j for j in range(int(self.dcnt[b]) + 1))
                dst.extend([self.sink] * (int(self.dcnt[b]) + 1))
            elif draft[b]:
                src.append(b * D1 + int(self.dcnt[b]))
                dst.append(b * D1 + int(self.dcnt[b]) + 1)
        h["tok_src"][:] = self.sink
        h["tok_src"][:T] = src
        h["tok_dst"][:] = self.sink
        h["tok_dst"][:T] = dst
        h["tok0"][:] = self.tok0
        h["qo"][:] = qo
        h["qo_prev"][:] = self.prev_qo if self.prev_qo is not None else qo
        h["rope"][:] = start
        h["mixed_indptr"][:] = np.concatenate([[0], np.cumsum(mixed_pages)])
        h["mixed_last"][:] = last
        h["modes"][:] = np.where(draft, 0, 1)
        h["num_pages"][:] = full_pages
        h["dec_lens"][:] = qlen
        h["draft_lens"][:] = np.where(draft, end, 0)
        self._dev.copy_(self._stage[slot], non_blocking=True)
        ev = self._stage_ev[slot] or torch.cuda.Event()
        ev.record()
        self._stage_ev[slot] = ev
        self._stage_slot = (slot + 1) % len(self._stage)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32))  # noqa: E731
        m = self.model
        self.mixed.plan_host(t(qo), t(h["mixed_indptr"]), t(mixed_len), None, m.hq, m.hkv, HEAD_DIM, PAGE,
                             causal=True)
        self.refresh.plan_host(t(qo), t(np.concatenate([[0], np.cumsum(full_pages)])), t(end), None, m.hq, m.hkv,
                               HEAD_DIM, PAGE, causal=True)
        self.prev_qo = qo.copy()
        return dict(T=T, verify=verify, draft=draft, qlen=qlen)

    def _bucket(self, T: int) -> int:
        return self.B if T <= self.B else self.t_max

    def step(self) -> dict:
        s = self._schedule()
        T = s["T"]
        select = self.step_no > 0
        bucket = self._bucket(T)
        key = (bucket, select)
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        timed = True
        if not self.use_graphs:
            self._body(bucket, select)
        elif key in self.graphs:
            self.graphs[key].replay()
        else:
            timed = False
            # This step runs eagerly on a side stream (the warm-up a capture
            # needs); the graph captured after it serves later steps.
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._body(bucket, select)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._body(bucket, select)
            self.graphs[key] = g
        ev[1].record()
        if timed:
            s["events"] = ev
        # Draft rows advance without a readback (their proposals stay on the
        # device); a step with verify rows is read back to accept drafts.
        self.dcnt[s["draft"]] += 1
        if s["verify"].any():
            self._commit(s, self.out_ids[:T].cpu().numpy(), self.tok_dev[:self.sink].view(self.B, -1).cpu().numpy())
        self.step_no += 1
        return s

    def _commit(self, s: dict, ids: np.ndarray, drafts: np.ndarray):
        """Verify rows accept the longest prefix of their drafts that equals
        the target's greedy outputs and commit it plus the target's next token
        (runtime.py:755-783), capped at the row's remaining budget."""
        qo = np.concatenate([[0], np.cumsum(s["qlen"])])
        for b in np.flatnonzero(s["verify"]):
            out_b = ids[qo[b]:qo[b + 1]]
            d = int(self.dcnt[b])
            acc = accept(drafts[b, 1:d + 1], out_b)
            commit = [int(t) for t in drafts[b, 1:acc + 1]] + [int(out_b[acc])]
            commit = commit[:self.G - len(self.out[b])]
            self.out[b].extend(commit)
            self.n[b] += acc + 1
            self.tok0[b] = out_b[acc]
            self.dcnt[b] = 0
            self.dtarget[b] = self._draw_targets(1)[0]
            self.accepted_total += acc
            self.verify_rows += 1

    def generate(self) -> dict:
        """Runs the decode loop after prefill() until every row has max_new
        tokens; returns the tokens and counters (wall time with the device
        synchronised at both ends)."""
        self.accepted_total = 0
        self.verify_rows = 0
        steps = {"draft": 0, "verify": 0, "mixed": 0}
        events = {"draft": [], "verify": [], "mixed": []}
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while any(len(o) < self.G for o in self.out):
            s = self.step()
            kind = "mixed" if s["verify"].any() and s["draft"].any() else ("verify" if s["verify"].any() else "draft")
            steps[kind] += 1
            if "events" in s:
                events[kind].append(s["events"])
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        # Device time of the step's forward (selection, spill, layers, argmax), per kind.
        device_ms = {k: round(float(np.mean([a.elapsed_time(b) for a, b in v])), 4) for k, v in events.items() if v}
        tokens = np.array([o[:self.G] for o in self.out], np.int64)
        decoded = int(tokens.shape[0] * (self.G - 1))  # tokens produced by the loop (the first came from prefill)
        return {"tokens": tokens, "seconds": dt, "steps": steps, "decoded_tokens": decoded, "device_ms_per_step": device_ms,
                "accepted_drafts": int(self.accepted_total), "verify_rows": int(self.verify_rows)}

    # ------------------------------------------------------ greedy identity
    def teacher_forced_check(self, prompts_len: int, tokens: np.ndarray):
        """Feeds each row's generated tokens back through full causal
        attention (one chunk per row, positions P.., the prompt's cache
        unchanged) and returns, per emitted token after the first, the
        target's greedy choice and the logit gap between that choice and the
        emitted token (0 where they agree)."""
        gaps, agree = [], []
        for b in range(self.B):
            seq = torch.from_numpy(tokens[b]).to(self.dev, torch.int32)
            x = self._run_slot(b, seq[:-1], prompts_len)
            top_id, top1, _, e = self.model.token_logit_stats(x, seq[1:].long())
            agree.append((top_id == seq[1:].long()).cpu().numpy())
            gaps.append((top1 - e).clamp(min=0).cpu().numpy())
        return np.stack(agree), np.stack(gaps)


def synthetic_prompts(batch: int, length: int, vocab: int, seed: int = 0) -> torch.Tensor:
    """Uniform random tokens in [100, vocab) (aspire.data.synthetic_dataset semantics)."""
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.integers(100, vocab, size=(batch, length)).astype(np.int32))


def token_sha256(tokens: np.ndarray) -> str:
    return hashlib.sha256(json.dumps(tokens.tolist()).encode()).hexdigest()


def compare_sequences(spec: np.ndarray, ar: np.ndarray) -> dict:
    """Rows identical, and the first divergence position of the others."""
    same = [bool(np.array_equal(a, b)) for a, b in zip(spec, ar)]
    first = [int(np.flatnonzero(a != b)[0]) if not s else -1 for a, b, s in zip(spec, ar, same)]
    return {"rows_identical": int(sum(same)), "rows": len(same), "first_divergence": first}
