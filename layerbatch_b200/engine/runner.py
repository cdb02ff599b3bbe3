"""Parallel layout and paged KV-cache allocation for the hot path (the ModelRunner side).

The reference runner puts every rank in one tensor-parallel group, replicates the KV heads
when ``num_key_value_heads < world_size`` and sizes one cache tensor
``[2, layers, blocks, block_size, kv_heads, head_dim]`` from the free device memory
(nanovllm/engine/model_runner.py:387-416); when ``Hkv < tp`` the attention layer also
expands K/V to the TP head count (qwen3_5.py:623-633, 718-726), and the stored rows then
no longer match the cache's per-token stride that ``store_kvcache`` asserts (read from
the source, not run).

Here attention is sharded by whole KV heads and the remaining factor is data parallel:

* ``ParallelLayout.plan(world, num_kv_heads)``: ``tp`` = the largest divisor of
  ``num_kv_heads`` that also divides ``world``; ``dp = world / tp`` groups of ``tp``
  consecutive ranks, each with its own batch and its own paged cache; experts are split
  over all ``world`` ranks (``ep = world``).  No KV head is ever replicated.
* ``kv_cache_plan``: the reference's budget formula (device total x utilisation, minus
  what is in use outside the allocator's current tensors, minus the allocator's peak over
  its current bytes, minus reserved bytes), divided by the bytes of one block on this rank
  (``2 x layers x block_size x Hkv/tp x head_dim x itemsize``).  A rank of a TP group
  holds its KV heads of the group's blocks, so every rank of the group gets the same block
  count and the scheduler of the group hands out block ids once.
* ``agree_on_blocks``: the smallest block count over the TP group (the ranks' free
  memory can differ).
* ``allocate_kv_cache``: one tensor per rank, per-layer views assigned to every module
  that has ``k_cache`` and ``v_cache`` attributes, in module order (model_runner.py:
  409-416).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import nn


@dataclass(frozen=True)
class ParallelLayout:
    world: int
    tp: int
    rank: int

    def __post_init__(self):
        if self.world < 1 or self.tp < 1 or self.world % self.tp:
            raise ValueError(f"tp={self.tp} must divide world={self.world}")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside [0, {self.world})")

    @classmethod
    def plan(cls, world: int, num_kv_heads: int, rank: int = 0, max_tp: int | None = None):
        """Largest tensor-parallel degree that shards whole KV heads (divides both
        ``num_kv_heads`` and ``world``, at most ``max_tp``); the rest is data parallel."""
        cap = min(num_kv_heads, world, max_tp or world)
        tp = max(t for t in range(1, cap + 1) if num_kv_heads % t == 0 and world % t == 0)
        return cls(world, tp, rank)

    @property
    def dp(self) -> int:
        return self.world // self.tp

    @property
    def tp_rank(self) -> int:
        return self.rank % self.tp

    @property
    def dp_rank(self) -> int:
        return self.rank // self.tp

    @property
    def ep_size(self) -> int:
        return self.world

    @property
    def ep_rank(self) -> int:
        return self.rank

    def tp_group_ranks(self, dp_rank: int | None = None) -> list[int]:
        g = self.dp_rank if dp_rank is None else dp_rank
        return list(range(g * self.tp, (g + 1) * self.tp))

    def all_tp_groups(self) -> list[list[int]]:
        return [self.tp_group_ranks(g) for g in range(self.dp)]

    def kv_heads(self, num_kv_heads: int) -> slice:
        if num_kv_heads % self.tp:
            raise ValueError(f"tp={self.tp} does not divide num_kv_heads={num_kv_heads}; "
                             "KV heads are sharded, never replicated")
        n = num_kv_heads // self.tp
        return slice(self.tp_rank * n, (self.tp_rank + 1) * n)


@dataclass(frozen=True)
class KVCachePlan:
    num_layers: int
    block_size: int
    num_kv_heads: int        # on this rank
    head_dim: int
    itemsize: int
    block_bytes: int         # one block of every layer, K and V, on this rank
    budget_bytes: int
    num_blocks: int

    @property
    def shape(self) -> tuple:
        return (2, self.num_layers, self.num_blocks, self.block_size, self.num_kv_heads,
                self.head_dim)


def count_attention_layers(model: nn.Module) -> int:
    """Modules that own a paged cache (``k_cache`` and ``v_cache`` attributes)."""
    return sum(1 for m in model.modules() if hasattr(m, "k_cache") and hasattr(m, "v_cache"))


def kv_cache_plan(num_kv_heads: int, head_dim: int, num_layers: int, layout: ParallelLayout,
                  block_size: int = 256, dtype: torch.dtype = torch.bfloat16,
                  gpu_memory_utilization: float = 0.9, reserved_bytes: int = 0,
                  mem_info: tuple[int, int] | None = None,
                  allocator_peak: int | None = None,
                  allocator_current: int | None = None) -> KVCachePlan:
    """Blocks of paged KV cache this rank can hold.

    ``mem_info`` = (free, total) bytes of the device and ``allocator_peak`` /
    ``allocator_current`` the caching allocator's peak and current bytes; by default they
    are read from the current CUDA device (``torch.cuda.mem_get_info`` and
    ``torch.cuda.memory_stats``), as the reference does."""
    if num_layers <= 0:
        raise ValueError("no attention layer holds a KV cache")
    if mem_info is None:
        mem_info = torch.cuda.mem_get_info()
    free, total = mem_info
    if allocator_peak is None or allocator_current is None:
        stats = torch.cuda.memory_stats()
        allocator_peak = stats.get("allocated_bytes.all.peak", 0)
        allocator_current = stats.get("allocated_bytes.all.current", 0)
    used = total - free
    kv_local = layout.kv_heads(num_kv_heads).stop - layout.kv_heads(num_kv_heads).start
    itemsize = torch.empty((), dtype=dtype).element_size()
    block_bytes = 2 * num_layers * block_size * kv_local * head_dim * itemsize
    budget = int(total * gpu_memory_utilization - used - allocator_peak + allocator_current)
    budget -= int(reserved_bytes)
    blocks = budget // block_bytes
    if blocks <= 0:
        raise RuntimeError(f"no room for a KV block: budget {budget} B, block {block_bytes} B")
    return KVCachePlan(num_layers, block_size, kv_local, head_dim, itemsize, block_bytes,
                       budget, int(blocks))


def agree_on_blocks(plan: KVCachePlan, group=None) -> KVCachePlan:
    """The ranks of a TP group share block ids (each holds its KV heads of every block),
    so they all take the smallest block count any of them can hold."""
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([plan.num_blocks], dtype=torch.int64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return dataclasses.replace(plan, num_blocks=int(t.item()))


def allocate_kv_cache(model: nn.Module, plan: KVCachePlan, device=None,
                      dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """One cache tensor ``plan.shape`` on ``device``; layer i's modules get the views
    ``[0, i]`` (K) and ``[1, i]`` (V), ``[blocks, block_size, Hkv/tp, head_dim]``."""
    kv = torch.empty(plan.shape, dtype=dtype, device=device)
    layer = 0
    for m in model.modules():
        if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
            if layer >= plan.num_layers:
                raise ValueError(f"model has more cache-owning modules than the plan's "
                                 f"{plan.num_layers} layers")
            m.k_cache = kv[0, layer]
            m.v_cache = kv[1, layer]
            layer += 1
    if layer != plan.num_layers:
        raise ValueError(f"plan has {plan.num_layers} layers, the model {layer}")
    return kv
