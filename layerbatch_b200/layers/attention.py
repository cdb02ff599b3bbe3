"""Drop-in for the reference's attention operator module (nanovllm/layers/attention.py and
the POD entry points of nanovllm/layers/pod_kernels.py), backed by the sm_100a library.

* ``store_kvcache`` (attention.py:71-80) -> ``lb_store_kvcache``.
* ``Attention(num_heads, head_dim, scale, num_kv_heads).forward(q, k, v)``
  (attention.py:83-226): stores the new K/V, then runs the POD kernel over the paged
  cache for prefill, decode or mixed batches; returns ``[N, Hq, D]`` for prefill and
  ``[B, 1, Hq, D]`` for decode, like the reference.
* ``gated_attention_oproj`` replaces ``o = attn(q,k,v); o * sigmoid(gate); o_proj(o)``
  (nanovllm/models/qwen3_5.py:739-746) with one fused call.
* ``pod_fused_attn_gemm`` / ``pod_attn_only`` keep the POD signatures
  (pod_kernels.py:237-354).
* ``set_use_pod_decode`` / ``set_pod_runtime_cfg`` (attention.py:36-46) are kept for API
  compatibility; the B200 path always runs its own kernel and sizes its own tiles.

There is no flash-attn, flashinfer, Triton or SDPA fallback: without the CUDA library the
calls raise.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..utils.context import get_context

_USE_POD_DECODE = True
_POD_RUNTIME_CFG = dict(num_kv_splits=0)


def set_use_pod_decode(flag: bool):
    global _USE_POD_DECODE
    _USE_POD_DECODE = bool(flag)


def get_use_pod_decode() -> bool:
    return _USE_POD_DECODE


def set_pod_runtime_cfg(cfg: dict):
    """Accepts the reference's keys; only ``num_kv_splits`` (0 = automatic) is used."""
    _POD_RUNTIME_CFG.update({k: v for k, v in cfg.items() if v is not None})


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor):
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    ops.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


def _split_pages(block_tables: torch.Tensor) -> int:
    n = int(_POD_RUNTIME_CFG.get("num_kv_splits", 0) or 0)
    if n <= 0:
        return 0
    return max(1, -(-block_tables.shape[1] // n))


def _tables_from_slots(slot_mapping, cu_seqlens_q, max_seqlen_q, page_size):
    """Block tables of sequences that were just stored whole (prefill without a prefix
    cache, where the reference passes no block tables): page m of sequence b is the page
    holding its token 256*m."""
    B = cu_seqlens_q.numel() - 1
    nblk = max(1, -(-max_seqlen_q // page_size))
    m = torch.arange(nblk, device=slot_mapping.device, dtype=torch.int64)
    start = cu_seqlens_q[:-1].to(torch.int64).view(B, 1)
    ln = (cu_seqlens_q[1:] - cu_seqlens_q[:-1]).to(torch.int64).view(B, 1)
    pos = m.view(1, nblk) * page_size
    idx = torch.clamp(start + pos, max=slot_mapping.numel() - 1)
    bt = torch.div(slot_mapping.to(torch.int64)[idx], page_size, rounding_mode="floor")
    bt = torch.where(pos < ln, bt, torch.full_like(bt, -1))
    return bt.to(torch.int32), ln.view(B).to(torch.int32)


def _batch_meta(q, context, decode):
    """(block_tables, context_lens, cu_seqlens_q, max_q_len) for the current context."""
    if decode:
        B = q.shape[0]
        cu = torch.arange(B + 1, dtype=torch.int32, device=q.device)
        return context.block_tables, context.context_lens, cu, 1
    cu = context.cu_seqlens_q
    if context.block_tables is not None:
        # prefix-cached prefill: context length = cu_seqlens_k span
        lens = (context.cu_seqlens_k[1:] - context.cu_seqlens_k[:-1]).to(torch.int32)
        return context.block_tables, lens, cu, context.max_seqlen_q
    return None, None, cu, context.max_seqlen_q


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def _run(self, q, gate=None, w_o=None, out=None):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        decode = not context.is_prefill
        bt, lens, cu, max_q = _batch_meta(q, context, decode)
        if bt is None:
            bt, lens = _tables_from_slots(context.slot_mapping, cu, max_q, k_cache.shape[1])
        return ops.pod_attn_oproj(q, gate, k_cache, v_cache, bt, lens, cu, w_o, self.scale,
                                  out=out, max_q_len=max_q, kv_split_pages=_split_pages(bt))

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = get_context()
        if not (self.k_cache.numel() and self.v_cache.numel()):
            raise RuntimeError("Attention needs its paged k_cache/v_cache assigned by the runner")
        store_kvcache(k, v, self.k_cache, self.v_cache, context.slot_mapping)
        o = self._run(q)
        o = o.view(q.shape[0], self.num_heads, self.head_dim)
        return o if context.is_prefill else o.unsqueeze(1)

    def forward_gated_oproj(self, q, k, v, gate, w_o, out=None):
        """store K/V, attention, ``* sigmoid(gate)`` and o_proj in one library call."""
        context = get_context()
        store_kvcache(k, v, self.k_cache, self.v_cache, context.slot_mapping)
        return self._run(q, gate=gate, w_o=w_o, out=out)


def gated_attention_oproj(attn: Attention, q, k, v, gate, w_o, out=None):
    """Fused replacement of qwen3_5.py:739-746 (``gate`` is ``[N, Hq, D]`` or its flat view)."""
    if gate.dim() == 2:
        gate = gate.view(gate.shape[0], attn.num_heads, attn.head_dim)
    return attn.forward_gated_oproj(q, k, v, gate, w_o, out=out)


def pod_fused_attn_gemm(q, k_cache, v_cache, block_table, context_lens, sm_scale, A, B, C_out,
                        num_kv_splits: int = 16, block_n: int = 64, block_h: int = 16,
                        mid_o=None, out=None):
    """Decode attention over the paged cache plus a piggy-back ``C_out = A @ B``
    (pod_kernels.py:237-326).  ``mid_o``, ``block_n`` and ``block_h`` are accepted for
    compatibility; the split length follows ``num_kv_splits``.  Returns ``[B, Hq, D]``."""
    Bsz, Hq, D = q.shape
    cu = torch.arange(Bsz + 1, dtype=torch.int32, device=q.device)
    split = max(1, -(-block_table.shape[1] // max(1, num_kv_splits)))
    flat = None if out is None else out.view(Bsz, Hq * D)
    o = ops.pod_attn_oproj(q, None, k_cache, v_cache, block_table, context_lens, cu, None,
                           sm_scale, attn_out=flat, max_q_len=1, kv_split_pages=split)
    if A is not None and A.numel() and B is not None and B.numel():
        ops.gemm(A, B.t().contiguous(), out=C_out)
    return o.view(Bsz, Hq, D)


def pod_attn_only(q, k_cache, v_cache, block_table, context_lens, sm_scale,
                  num_kv_splits: int = 16, block_n: int = 64, block_h: int = 16,
                  mid_o=None, out=None):
    """pod_kernels.py:329-354: the decode attention alone."""
    return pod_fused_attn_gemm(q, k_cache, v_cache, block_table, context_lens, sm_scale, None,
                               None, None, num_kv_splits, block_n, block_h, mid_o, out)
