"""Drop-in for the reference's gated full-attention layer ``Qwen3_5FullAttention``
(nanovllm/models/qwen3_5.py:587-746) at tensor-parallel size 1, on the sm_100a library.

Same constructor arguments and parameter names (``q_proj``, ``k_proj``, ``v_proj``,
``o_proj``, ``q_norm``, ``k_norm``, ``rotary_emb.cos_sin_cache``), same
``forward(positions, hidden_states)``.  One call runs:

1. the q / k / v projections (``lb_gemm_bf16``: tcgen05, fp32 accumulate, bf16 out);
2. ``lb_attn_prologue``: (1+w) RMSNorm of query and key, partial RoPE of both, and the
   K/V store into the paged cache, in one launch; the gate stays in place as the second
   half of each head of q_proj's output (qwen3_5.py:710-713) and is read strided;
3. ``lb_pod_attn_oproj``: POD attention over the paged cache for any mix of prefill and
   decode sequences, sigmoid gate and o_proj.  (The prologue can also run inside this
   call's attention kernel, ``ops.gated_attention_layer(fuse_prologue=True)``.)

The rotary cache is built with the same torch operations as the reference
(rotary_embedding.py:26-33), so the kernel reads bit-identical cos/sin values.  Tensor
parallel attention goes through ``engine.sharding.tp_attention_oproj``.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..utils.context import get_context
from .attention import Attention, _batch_meta, _split_pages, _tables_from_slots
from .linear import ReplicatedLinear


class Qwen3_5RMSNorm(nn.Module):
    """Holds the (1 + weight) RMSNorm parameters (qwen3_5.py:39-55); the normalisation
    itself runs fused inside ``lb_attn_prologue``."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(dim))


class RotaryEmbedding(nn.Module):
    """Partial rotary embedding parameters (rotary_embedding.py:17-33): the fp32
    ``cos_sin_cache [max_position, 1, rotary_dim]`` read by ``lb_attn_prologue``."""

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int,
                 base: float):
        super().__init__()
        self.head_size = head_size
        self.rotary_dim = rotary_dim
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def _apply(self, fn, recurse=True):
        # device moves apply; dtype casts (module.to(bf16)) must not round the fp32 cache
        cache = self.cos_sin_cache
        super()._apply(fn, recurse)
        self.cos_sin_cache = cache.to(self.cos_sin_cache.device)
        return self


class Qwen3_5FullAttention(nn.Module):

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 max_position: int, rms_norm_eps: float, rope_theta: float,
                 partial_rotary_factor: float = 0.25):
        super().__init__()
        self.total_num_heads = self.num_heads = num_heads
        self.total_num_kv_heads = self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.q_size = num_heads * head_dim
        self.kv_size = num_kv_heads * head_dim
        self.scaling = head_dim ** -0.5
        self.q_proj = ReplicatedLinear(hidden_size, num_heads * head_dim * 2)
        self.k_proj = ReplicatedLinear(hidden_size, self.kv_size)
        self.v_proj = ReplicatedLinear(hidden_size, self.kv_size)
        self.o_proj = ReplicatedLinear(num_heads * head_dim, hidden_size)
        self.rotary_dim = int(head_dim * partial_rotary_factor)
        self.rotary_emb = RotaryEmbedding(head_dim, self.rotary_dim, max_position, rope_theta)
        self.q_norm = Qwen3_5RMSNorm(head_dim, eps=rms_norm_eps)
        self.k_norm = Qwen3_5RMSNorm(head_dim, eps=rms_norm_eps)
        self.attn = Attention(num_heads, head_dim, self.scaling, num_kv_heads)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        context = get_context()
        attn = self.attn
        if not (attn.k_cache.numel() and attn.v_cache.numel()):
            raise RuntimeError("attention needs its paged k_cache/v_cache assigned by the runner")
        x = hidden_states.reshape(-1, hidden_states.shape[-1]).contiguous()
        N, Hq, Hkv, D = x.shape[0], self.num_heads, self.num_kv_heads, self.head_dim
        q_out = ops.gemm(x, self.q_proj.weight).view(N, Hq, 2 * D)
        k = ops.gemm(x, self.k_proj.weight).view(N, Hkv, D)
        v = ops.gemm(x, self.v_proj.weight).view(N, Hkv, D)
        query = ops.attn_prologue(q_out[..., :D], k, v, self.q_norm.weight, self.k_norm.weight,
                                  self.rotary_emb.cos_sin_cache, positions,
                                  context.slot_mapping, attn.k_cache, attn.v_cache,
                                  self.q_norm.eps)
        gate = q_out[..., D:]
        decode = not context.is_prefill
        bt, lens, cu, max_q = _batch_meta(query, context, decode)
        if bt is None:
            bt, lens = _tables_from_slots(context.slot_mapping, cu, max_q, attn.k_cache.shape[1])
        return ops.pod_attn_oproj(query, gate, attn.k_cache, attn.v_cache, bt, lens, cu,
                                  self.o_proj.weight, self.scaling, out=out, max_q_len=max_q,
                                  kv_split_pages=_split_pages(bt))
