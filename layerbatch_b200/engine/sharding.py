"""Tensor- and expert-parallel sharding of the hot path (the ModelRunner side).

The reference engine shards attention heads Megatron-style over ``tensor_parallel_size``
ranks and replicates every expert on every rank (nanovllm/engine/model_runner.py:37-74,
387-416; nanovllm/models/qwen3_5.py:605-633, 795-800).  Here:

* **Attention, tensor parallel by KV head.**  Rank r of a TP group of size tp holds KV
  heads ``[r*Hkv/tp, (r+1)*Hkv/tp)``, the query / gate heads of their GQA groups, its
  slice of the paged cache ``[num_blocks, 256, Hkv/tp, D]`` and the matching column slice
  of o_proj ``W_o[:, heads]``.  The fused attention call writes fp32 o_proj partials and
  an fp32 all-reduce sums them (the reference's RowParallelLinear numerics,
  nanovllm/layers/linear.py:149-157).  With Hkv = 2, tp <= 2; larger GPU counts add
  data-parallel TP groups.
* **MoE, expert parallel with all-to-all.**  Experts are split in contiguous ranges of
  E/P over the P ranks.  Each rank routes its own tokens, sends every (token, slot) pair
  to the rank owning the chosen expert (``all_to_all_single`` with split sizes), the owner
  runs its local experts on the rows it received (routing given, no shared expert), the
  weighted rows travel back, and the source adds them to its shared-expert output in the
  library's combine.  Pairs routed to the source's own experts go through the same path
  (NCCL copies them locally).

The exchange helpers work on any device: the multi-process CPU tests run them over gloo
with the CPU oracle as the expert compute.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


# ------------------------------------------------------------------------------ expert parallel
@dataclass
class EPPlan:
    """Routing table of one expert-parallel exchange on one rank."""
    order: torch.Tensor        # [T*k] flat pair index (t*k + j) in send order (by dest rank)
    pair_pos: torch.Tensor     # [T, k] int32 position of pair (t, j) in the send order
    send_counts: list          # pairs sent to each rank
    recv_counts: list          # pairs received from each rank
    top_k: int


def ep_plan(ids: torch.Tensor, num_experts: int, group=None) -> EPPlan:
    """Destination of every pair = owner of its expert; stable order by destination."""
    P = dist.get_world_size(group)
    nl = num_experts // P
    T, k = ids.shape
    dest = (ids.long() // nl).reshape(-1)
    order = torch.argsort(dest, stable=True)
    send = torch.bincount(dest, minlength=P)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    pair_pos = torch.empty(T * k, dtype=torch.int32, device=ids.device)
    pair_pos[order] = torch.arange(T * k, dtype=torch.int32, device=ids.device)
    return EPPlan(order, pair_pos.view(T, k), send.tolist(), recv.tolist(), k)


def _a2a(x: torch.Tensor, out_rows: int, out_split, in_split, group):
    """all_to_all_single of rows; bf16 rows travel bit-exactly as int32 pairs."""
    bf16 = x.dtype == torch.bfloat16
    flat = x.contiguous().view(torch.int32) if bf16 else x.contiguous()
    out = torch.empty((out_rows,) + tuple(flat.shape[1:]), dtype=flat.dtype, device=x.device)
    dist.all_to_all_single(out, flat, out_split, in_split, group=group)
    return out.view(torch.bfloat16) if bf16 else out


def ep_dispatch(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, plan: EPPlan, group=None):
    """Send each pair's token row, global expert id and weight to the expert's owner."""
    k = plan.top_k
    rows = x[plan.order // k]
    n_in = sum(plan.recv_counts)
    rx = _a2a(rows, n_in, plan.recv_counts, plan.send_counts, group)
    rid = _a2a(ids.reshape(-1)[plan.order].to(torch.int32), n_in, plan.recv_counts,
               plan.send_counts, group)
    rw = _a2a(w.reshape(-1)[plan.order].to(torch.float32), n_in, plan.recv_counts,
              plan.send_counts, group)
    return rx, rid, rw


def ep_return(y_recv: torch.Tensor, plan: EPPlan, group=None) -> torch.Tensor:
    """Send the owners' weighted expert rows back; result is in the source's send order."""
    return _a2a(y_recv, sum(plan.send_counts), plan.send_counts, plan.recv_counts, group)


def ep_moe_forward(block, x: torch.Tensor, group=None) -> torch.Tensor:
    """Expert-parallel ``Qwen3_5SparseMoeBlock`` forward on this rank's tokens."""
    from .. import ops
    k = block.top_k
    E = block.num_experts
    logits = ops.gemm(x.contiguous(), block.gate.weight)
    ids, wf, _ = ops.router_topk(logits, k)
    plan = ep_plan(ids, E, group)
    rx, rid, rw = ep_dispatch(x, ids, wf, plan, group)
    n = rx.shape[0]
    if n:
        y_recv = ops.moe_forward(rx.contiguous(), None, block.experts.gate_up_proj,
                                 block.experts.down_proj, None, None, None, None, 1,
                                 expert_base=block.expert_base, topk_ids=rid.view(n, 1),
                                 topk_weights=rw.view(n, 1), num_experts=E, ws_tag="ep_owner")
    else:
        y_recv = torch.empty(0, x.shape[1], dtype=x.dtype, device=x.device)
    y_send = ep_return(y_recv, plan, group)
    se = block.shared_expert
    return ops.moe_forward(x.contiguous(), None, None, None, se.gate_proj.weight,
                           se.up_proj.weight, se.down_proj.weight,
                           block.shared_expert_gate.weight, k, topk_ids=ids, topk_weights=wf,
                           num_experts=E, pair_rows=y_send, pair_index=plan.pair_pos,
                           ws_tag="ep_source")


# ------------------------------------------------------------------------------ tensor parallel
@dataclass
class TPShard:
    """KV-head shard of one full-attention layer on one TP rank."""
    q_heads: slice
    kv_heads: slice
    tp_rank: int
    tp_size: int


def attention_shard(num_heads: int, num_kv_heads: int, tp_rank: int, tp_size: int) -> TPShard:
    """Heads owned by ``tp_rank``: whole GQA groups, so no KV head is replicated.

    The reference replicates and expands the KV head when ``Hkv < tp``
    (qwen3_5.py:623-633, 718-726); here tp must divide Hkv and larger GPU counts use
    several data-parallel TP groups instead.
    """
    if num_kv_heads % tp_size or num_heads % num_kv_heads:
        raise ValueError(f"tp={tp_size} must divide num_kv_heads={num_kv_heads}")
    kv = num_kv_heads // tp_size
    g = num_heads // num_kv_heads
    return TPShard(slice(tp_rank * kv * g, (tp_rank + 1) * kv * g),
                   slice(tp_rank * kv, (tp_rank + 1) * kv), tp_rank, tp_size)


def shard_attention_tensors(shard: TPShard, q, gate, k_cache, v_cache, w_o, head_dim):
    """Slice full-model tensors to one rank (q/gate [N, Hq, D], caches [nb, 256, Hkv, D],
    W_o [H, Hq*D])."""
    hs = shard.q_heads
    return (q[:, hs].contiguous(), gate[:, hs].contiguous(),
            k_cache[:, :, shard.kv_heads].contiguous(), v_cache[:, :, shard.kv_heads].contiguous(),
            w_o[:, hs.start * head_dim:hs.stop * head_dim].contiguous())


def tp_attention_oproj(shard: TPShard, q, gate, k_cache, v_cache, block_tables, context_lens,
                       cu_seqlens_q, w_o, scale, group=None, max_q_len=None, events=None,
                       out=None, work_hint=None, exchange=None, tp_phases=0):
    """This rank's heads -> fp32 o_proj partial -> all-reduce -> bf16 ``[N, H]``.

    With ``exchange`` (an ``engine.peer.TPExchange`` of the TP group) the reduction runs
    inside the library call: the o_proj GEMM stores each fp32 tile into the inbox of the
    rank owning it over NVLink, owners sum in rank order and send the bf16 rows back (no
    NCCL).  Without it, an fp32 NCCL all-reduce of the partials, like the reference."""
    from .. import ops
    N = q.shape[0]
    if exchange is not None and shard.tp_size > 1:
        if out is None:
            out = torch.empty(N, w_o.shape[0], dtype=torch.bfloat16, device=q.device)
        return ops.pod_attn_oproj(q, gate, k_cache, v_cache, block_tables, context_lens,
                                  cu_seqlens_q, w_o, scale, out=out, max_q_len=max_q_len,
                                  ws_tag=f"tp_attn{exchange.rank}", events=events,
                                  work_hint=work_hint, tp=exchange, tp_phases=tp_phases)
    partial = torch.empty(N, w_o.shape[0], dtype=torch.float32, device=q.device)
    ops.pod_attn_oproj(q, gate, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q,
                       w_o, scale, out=partial, max_q_len=max_q_len, ws_tag="tp_attn",
                       events=events, work_hint=work_hint)
    if shard.tp_size > 1:
        dist.all_reduce(partial, group=group)
    if out is None:
        return partial.to(torch.bfloat16)
    out.copy_(partial)
    return out
