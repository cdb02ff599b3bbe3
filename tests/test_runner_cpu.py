"""Parallel layout and paged KV-cache allocation (engine/runner.py), on the CPU.

The block budget follows the reference's formula (nanovllm/engine/model_runner.py:
387-416) with the KV heads sharded over the TP ranks instead of replicated; the layout
never puts more TP ranks on a layer than it has KV heads (the rest is data parallel).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from layerbatch_b200.engine.runner import (KVCachePlan, ParallelLayout, agree_on_blocks,
                                           allocate_kv_cache, count_attention_layers,
                                           kv_cache_plan)
from layerbatch_b200.layers.attention import Attention, store_kvcache

GiB = 1 << 30


def test_layout_shards_whole_kv_heads():
    lay = ParallelLayout.plan(8, 2, rank=5)
    assert (lay.tp, lay.dp, lay.tp_rank, lay.dp_rank) == (2, 4, 1, 2)
    assert lay.all_tp_groups() == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert lay.kv_heads(2) == slice(1, 2)
    assert (lay.ep_size, lay.ep_rank) == (8, 5)
    assert ParallelLayout.plan(8, 4).tp == 4
    assert ParallelLayout.plan(6, 4).tp == 2
    assert ParallelLayout.plan(1, 2).tp == 1
    assert ParallelLayout.plan(8, 8, max_tp=2).tp == 2
    with pytest.raises(ValueError):
        ParallelLayout(8, 4, 0).kv_heads(2)       # would need replicated KV heads
    with pytest.raises(ValueError):
        ParallelLayout(8, 3, 0)


def test_plan_matches_the_reference_budget_formula():
    total, free = 183 * GiB, 150 * GiB
    peak, current, reserved = 12 * GiB, 10 * GiB, 1 * GiB
    L, Hkv, D, bs, util = 12, 2, 256, 256, 0.9
    for world in (1, 2, 8):
        lay = ParallelLayout.plan(world, Hkv, rank=world - 1)
        p = kv_cache_plan(Hkv, D, L, lay, block_size=bs, gpu_memory_utilization=util,
                          reserved_bytes=reserved, mem_info=(free, total),
                          allocator_peak=peak, allocator_current=current)
        used = total - free
        budget = int(total * util - used - peak + current) - reserved
        block_bytes = 2 * L * bs * (Hkv // lay.tp) * D * 2
        assert p.block_bytes == block_bytes
        assert p.num_blocks == budget // block_bytes
        assert p.num_kv_heads == Hkv // lay.tp
        assert p.shape == (2, L, budget // block_bytes, bs, Hkv // lay.tp, D)
    with pytest.raises(RuntimeError):
        kv_cache_plan(Hkv, D, L, ParallelLayout(1, 1, 0), mem_info=(1 * GiB, 183 * GiB),
                      allocator_peak=0, allocator_current=0)


class _Block(nn.Module):
    def __init__(self, hq, hkv, d):
        super().__init__()
        self.proj = nn.Linear(8, 8)
        self.attn = Attention(hq, d, d ** -0.5, hkv)


class _Model(nn.Module):
    def __init__(self, n, hq, hkv, d):
        super().__init__()
        self.layers = nn.ModuleList([_Block(hq, hkv, d) for _ in range(n)])
        self.norm = nn.LayerNorm(8)


def test_allocate_assigns_per_layer_views():
    Hq, Hkv, D = 16, 2, 64
    lay = ParallelLayout.plan(2, Hkv, rank=1)
    m = _Model(3, Hq // lay.tp, Hkv // lay.tp, D)
    L = count_attention_layers(m)
    assert L == 3
    plan = KVCachePlan(L, 256, Hkv // lay.tp, D, 2, 2 * L * 256 * (Hkv // lay.tp) * D * 2,
                       0, 5)
    kv = allocate_kv_cache(m, plan, dtype=torch.bfloat16)
    assert kv.shape == (2, 3, 5, 256, 1, D)
    for i, blk in enumerate(m.layers):
        a = blk.attn
        assert a.k_cache.shape == (5, 256, 1, D)
        assert a.k_cache.data_ptr() == kv[0, i].data_ptr()
        assert a.v_cache.data_ptr() == kv[1, i].data_ptr()
        # the stride store_kvcache requires of the per-layer views
        assert a.k_cache.stride(1) == (Hkv // lay.tp) * D
    with pytest.raises(ValueError):
        allocate_kv_cache(_Model(4, 8, 1, D), plan)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _agree_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        lay = ParallelLayout.plan(world, 2, rank=rank)
        # the ranks see different free memory; the group must agree on the smaller count
        free = (150 - 10 * rank) * GiB
        p = kv_cache_plan(2, 256, 12, lay, mem_info=(free, 183 * GiB), allocator_peak=0,
                          allocator_current=0)
        q.put((rank, p.num_blocks, agree_on_blocks(p).num_blocks))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), None))


def test_tp_group_agrees_on_block_count():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    own = [r[1] for r in res]
    assert all(isinstance(n, int) for n in own), res
    assert own[1] < own[0]
    assert res[0][2] == res[1][2] == min(own)
