"""Tensor-parallel head sharding of the hot path, on CPU gloo ranks.

Each of two ranks owns a contiguous KV-head range (and the query heads of its
groups), runs the mixed attention of its shard, and the shards are
all-gathered along the head dimension.  The result must equal the attention
over all heads: the path is rank-local, no collective is needed on it.
Ranks use 127.0.0.1 for the rendezvous.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aspire_b200.tp import local_head_counts, local_qo_heads, tp_heads
from aspire_b200.workloads import make_layout

WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import attention as oracle_attn

        hq, hkv = 8, 4
        lay = make_layout(batch=3, ctx=300, num_qo_heads=hq, num_kv_heads=hkv, draft_fraction=0.34,
                          budget_pages=6, seed=7)
        g = torch.Generator().manual_seed(1)
        q = torch.randn(lay.total_q, hq, 128, generator=g)
        kv = torch.randn(lay.num_pages_total, 2, 16, hkv, 128, generator=g)
        kv_r = tp_heads(hkv, rank, world)
        q_r = local_qo_heads(hq, hkv, rank, world)
        out, lse = oracle_attn.paged_attention(q[:, q_r.start:q_r.stop].contiguous(),
                                               kv[:, :, :, kv_r.start:kv_r.stop].contiguous(), lay.qo_indptr,
                                               lay.kv_indptr, lay.kv_indices, lay.kv_lens)
        outs = [torch.empty(lay.total_q, len(local_qo_heads(hq, hkv, r, world)), 128) for r in range(world)]
        dist.all_gather(outs, out.contiguous())
        if rank == 0:
            full, _ = oracle_attn.paged_attention(q, kv, lay.qo_indptr, lay.kv_indptr, lay.kv_indices, lay.kv_lens)
            torch.save({"gathered": torch.cat(outs, dim=1), "full": full}, os.path.join(result_dir, "tp.pt"))
    finally:
        dist.destroy_process_group()


def test_head_ranges_partition():
    for n in (1, 2, 3, 8, 32):
        for world in (1, 2, 4, 8):
            if world > n:
                continue
            ranges = [tp_heads(n, r, world) for r in range(world)]
            assert ranges[0].start == 0 and ranges[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(ranges, ranges[1:]))
            sizes = [len(r) for r in ranges]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    assert local_head_counts(32, 8, 1, 8) == (4, 1)


def test_sharded_attention_equals_full(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(WORLD, port, str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    res = torch.load(tmp_path / "tp.pt")
    assert torch.allclose(res["gathered"], res["full"], atol=1e-5, rtol=1e-5)
