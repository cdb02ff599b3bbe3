"""Per-step forward context, the same side channel as the reference engine's
``nanovllm/utils/context.py:5-53``: the model runner sets it before a forward pass and
every attention layer reads the KV metadata from it.

Fields keep the reference's names and meaning:
``slot_mapping`` [N] int32 (cache slot of each new token, -1 = skip),
``block_tables`` [B, max_blocks] int32 (-1 padded), ``context_lens`` [B] int32 (cached +
new tokens), ``cu_seqlens_q``/``cu_seqlens_k`` [B+1] int32.  ``is_prefill`` selects the
reference's prefill or decode dispatch; the B200 path handles both, and mixed batches,
in one launch, so it only needs ``cu_seqlens_q`` to know each sequence's query rows.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    seq_ids: list = field(default_factory=list)
    linear_attn_slot_indices: torch.Tensor | None = None
    max_ctx_len: int = 0
    total_tokens: int = 0
    pod_gemm: tuple | None = None
    fi_slot: str = "default"
    la_chunk_continuation: bool = False


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None, seq_ids=None,
                linear_attn_slot_indices=None, max_ctx_len=0, total_tokens=0,
                fi_slot="default", la_chunk_continuation=False):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                       slot_mapping, context_lens, block_tables, seq_ids or [],
                       linear_attn_slot_indices, max_ctx_len, total_tokens, pod_gemm=None,
                       fi_slot=fi_slot, la_chunk_continuation=la_chunk_continuation)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
