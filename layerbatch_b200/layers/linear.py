"""Drop-in tensor-parallel linears (nanovllm/layers/linear.py:12-159) on the sm_100a GEMM:
``ReplicatedLinear``, ``ColumnParallelLinear``, ``MergedColumnParallelLinear``,
``QKVParallelLinear`` and ``RowParallelLinear``.

Same constructor signatures, parameter names and ``weight_loader`` sharding hooks as the
reference.  Forward passes run ``lb_gemm_bf16`` (tcgen05 tensor cores, fp32 accumulate).
``RowParallelLinear`` at tp > 1 keeps the reference's numerics (linear.py:149-157): the
partial product is produced in fp32 (split-K reductions on the device, no bf16 rounding)
and summed across ranks with an fp32 NCCL all-reduce before the cast back.  Biases are
not on the hot path (the reference's attention projections have none) and are added with
a plain tensor add.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .. import ops


def divide(numerator, denominator):
    assert numerator % denominator == 0
    return numerator // denominator


def _tp():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _linear(x, w, b):
    shp = x.shape
    y = ops.gemm(x.reshape(-1, shp[-1]).contiguous(), w)
    y = y.view(*shp[:-1], w.shape[0])
    return y if b is None else y + b


class LinearBase(nn.Module):

    def __init__(self, input_size, output_size, bias=False, tp_dim=None):
        super().__init__()
        self.tp_dim = tp_dim
        self.tp_rank, self.tp_size = _tp()
        self.weight = nn.Parameter(torch.empty(output_size, input_size))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)


class ReplicatedLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False):
        super().__init__(input_size, output_size, bias)

    def weight_loader(self, param, loaded_weight):
        param.data.copy_(loaded_weight)

    def forward(self, x):
        return _linear(x, self.weight, self.bias)


class ColumnParallelLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False):
        _, tp_size = _tp()
        super().__init__(input_size, divide(output_size, tp_size), bias, 0)

    def weight_loader(self, param, loaded_weight):
        shard = param.data.size(self.tp_dim)
        param.data.copy_(loaded_weight.narrow(self.tp_dim, self.tp_rank * shard, shard))

    def forward(self, x):
        return _linear(x, self.weight, self.bias)


class MergedColumnParallelLinear(ColumnParallelLinear):
    """Several column-parallel outputs in one weight (linear.py:76-95): the loader writes
    shard ``loaded_shard_id`` of ``output_sizes`` into its rows; one GEMM computes all."""

    def __init__(self, input_size, output_sizes, bias=False):
        self.output_sizes = list(output_sizes)
        super().__init__(input_size, sum(self.output_sizes), bias)

    def weight_loader(self, param, loaded_weight, loaded_shard_id: int):
        off = sum(self.output_sizes[:loaded_shard_id]) // self.tp_size
        size = self.output_sizes[loaded_shard_id] // self.tp_size
        dst = param.data.narrow(self.tp_dim, off, size)
        dst.copy_(loaded_weight.chunk(self.tp_size, self.tp_dim)[self.tp_rank])


class QKVParallelLinear(ColumnParallelLinear):
    """Query, key and value projections in one weight (linear.py:98-130): rows
    ``[q | k | v]`` of this rank's heads, written by the loader per shard id "q" / "k" /
    "v"; one GEMM computes all three (the merged projection ``ops.gated_attention_layer``
    takes)."""

    def __init__(self, hidden_size, head_size, total_num_heads, total_num_kv_heads=None,
                 bias=False):
        _, tp_size = _tp()
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.head_size = head_size
        self.num_heads = divide(total_num_heads, tp_size)
        self.num_kv_heads = divide(total_num_kv_heads, tp_size)
        super().__init__(hidden_size, (total_num_heads + 2 * total_num_kv_heads) * head_size,
                         bias)

    def weight_loader(self, param, loaded_weight, loaded_shard_id: str):
        assert loaded_shard_id in ("q", "k", "v")
        q = self.num_heads * self.head_size
        kv = self.num_kv_heads * self.head_size
        off, size = {"q": (0, q), "k": (q, kv), "v": (q + kv, kv)}[loaded_shard_id]
        dst = param.data.narrow(self.tp_dim, off, size)
        dst.copy_(loaded_weight.chunk(self.tp_size, self.tp_dim)[self.tp_rank])


class RowParallelLinear(LinearBase):

    def __init__(self, input_size, output_size, bias=False):
        _, tp_size = _tp()
        super().__init__(divide(input_size, tp_size), output_size, bias, 1)

    def weight_loader(self, param, loaded_weight):
        shard = param.data.size(self.tp_dim)
        param.data.copy_(loaded_weight.narrow(self.tp_dim, self.tp_rank * shard, shard))

    def forward(self, x):
        if self.tp_size == 1:
            return _linear(x, self.weight, self.bias)
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).contiguous()
        y = torch.zeros(x2.shape[0], self.weight.shape[0], dtype=torch.float32, device=x.device)
        ops.gemm(x2, self.weight, out=y, accumulate_fp32=True, splits=_splits(x2.shape[0], x2.shape[1]))
        if self.bias is not None and self.tp_rank == 0:
            y += self.bias.float()
        dist.all_reduce(y)
        return y.to(x.dtype).view(*shp[:-1], self.weight.shape[0])


def _splits(M, K):
    """Split-K factor for an fp32-accumulated GEMM with few 128-row tiles."""
    kb = K // 64
    s = 1
    while s * 2 <= kb and kb % (s * 2) == 0 and ((M + 127) // 128) * s * 2 <= 16:
        s *= 2
    return s
