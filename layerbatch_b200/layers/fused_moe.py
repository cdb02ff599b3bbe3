"""Drop-in MoE modules with the reference's constructor signatures and parameter names
(nanovllm/models/qwen3_5.py:754-917), computed by the sm_100a library.

* ``Qwen3_5TopKRouter`` (qwen3_5.py:754-774): router GEMM on tensor cores, then the
  top-k kernel (softmax fp32, lowest-index ties, renormalised, cast to the input dtype).
* ``Qwen3_5SparseMoeBlock`` (qwen3_5.py:881-905): the whole block in one library call,
  ``lb_moe_forward``: router, top-k, permutation, grouped SwiGLU GEMM of the routed and
  shared experts, grouped down GEMM with the routing weight and the sigmoid shared gate
  fused, and the combine.  The prefill/decode split of ``Qwen3_5Experts.forward``
  (qwen3_5.py:802-813) disappears: one path serves both.
* ``fused_moe`` is the functional form over borrowed parameter tensors.

Parameters are registered exactly as the reference loader expects (``gate.weight``,
``experts.gate_up_proj``, ``experts.down_proj``, ``shared_expert.{gate,up,down}_proj.weight``,
``shared_expert_gate.weight``), so a reference state dict loads unchanged.  With an
expert-parallel shard (``ep_rank``/``ep_size``) the module holds only its slice of the
expert tensors and ``layerbatch_b200.engine.sharding`` routes tokens between ranks.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops


def fused_moe(x, router_w, gate_up, down, sh_gate, sh_up, sh_down, sh_gate_w, top_k,
              out=None, expert_base=0):
    return ops.moe_forward(x.contiguous(), router_w, gate_up, down, sh_gate, sh_up, sh_down,
                           sh_gate_w, top_k, out=out, expert_base=expert_base)


class Qwen3_5TopKRouter(nn.Module):

    def __init__(self, num_experts: int, hidden_size: int, top_k: int):
        super().__init__()
        self.top_k = top_k
        self.num_experts = num_experts
        self.weight = nn.Parameter(torch.zeros(num_experts, hidden_size))

    def forward(self, hidden_states: torch.Tensor):
        logits = ops.gemm(hidden_states.contiguous(), self.weight)
        ids, _, wb = ops.router_topk(logits, self.top_k)
        return wb.to(hidden_states.dtype), ids.long()


class Qwen3_5Experts(nn.Module):
    """The routed experts (qwen3_5.py:776-874).  ``forward(hidden_states, top_k_indices,
    top_k_weights)`` returns ``sum_j w[t,j] * expert_{id[t,j]}(x[t])`` for the experts this
    module holds (global ids ``[expert_base, expert_base + num_experts)``; others add
    nothing) with one grouped GEMM pair; the reference's prefill (sparse) and decode
    (dense) dispatches (:808-813) are the same call here."""

    def __init__(self, num_experts: int, hidden_size: int, moe_intermediate_size: int):
        super().__init__()
        self.num_experts = num_experts
        self.hidden_size = hidden_size
        self.intermediate_size = moe_intermediate_size
        self.gate_up_proj = nn.Parameter(
            torch.empty(num_experts, 2 * moe_intermediate_size, hidden_size))
        self.down_proj = nn.Parameter(torch.empty(num_experts, hidden_size, moe_intermediate_size))
        self.expert_base = 0                 # first global id held (expert parallel)
        self.total_experts = num_experts     # router width

    def forward(self, hidden_states, top_k_indices, top_k_weights):
        x = hidden_states.reshape(-1, self.hidden_size).contiguous()
        k = top_k_indices.shape[-1]
        y = ops.moe_forward(x, None, self.gate_up_proj, self.down_proj, None, None, None, None,
                            k, expert_base=self.expert_base,
                            topk_ids=top_k_indices.reshape(-1, k).to(torch.int32),
                            topk_weights=top_k_weights.reshape(-1, k).float(),
                            num_experts=self.total_experts, ws_tag="experts")
        return y.view_as(hidden_states)


class Qwen3_5SharedExpertMLP(nn.Module):
    """The shared expert (qwen3_5.py:910-917): ``down(silu(gate(x)) * up(x))``, as the
    shared group of the library's grouped GEMM pair, ungated (the block's sigmoid gate is
    applied by the block)."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x):
        H = self.gate_proj.weight.shape[1]
        x2 = x.reshape(-1, H).contiguous()
        T = x2.shape[0]
        # no routed experts: every (token, slot) pair is dropped
        ids = torch.zeros(T, 1, dtype=torch.int32, device=x.device)
        w = torch.zeros(T, 1, dtype=torch.float32, device=x.device)
        y = ops.moe_forward(x2, None, None, None, self.gate_proj.weight, self.up_proj.weight,
                            self.down_proj.weight, None, 1, topk_ids=ids, topk_weights=w,
                            num_experts=1, ws_tag="shared_expert")
        return y.view_as(x)


class Qwen3_5SparseMoeBlock(nn.Module):

    def __init__(self, hidden_size: int, num_experts: int, num_experts_per_tok: int,
                 moe_intermediate_size: int, shared_expert_intermediate_size: int,
                 ep_rank: int = 0, ep_size: int = 1):
        super().__init__()
        if num_experts % ep_size:
            raise ValueError("num_experts must divide by ep_size")
        self.num_experts = num_experts
        self.top_k = num_experts_per_tok
        self.ep_rank, self.ep_size = ep_rank, ep_size
        self.local_experts = num_experts // ep_size
        self.expert_base = ep_rank * self.local_experts
        self.gate = Qwen3_5TopKRouter(num_experts, hidden_size, num_experts_per_tok)
        self.experts = Qwen3_5Experts(self.local_experts, hidden_size, moe_intermediate_size)
        self.experts.expert_base = self.expert_base
        self.experts.total_experts = num_experts
        self.shared_expert = Qwen3_5SharedExpertMLP(hidden_size, shared_expert_intermediate_size)
        self.shared_expert_gate = nn.Linear(hidden_size, 1, bias=False)
        self.ep_exchange = None
        self.expert_slot = None   # [E] int32 slot of every expert (custom placement)

    def attach_exchange(self, exchange) -> None:
        """Use the NVLink peer-memory exchange (``engine.ep.EPExchange``) for expert
        parallelism instead of the NCCL all-to-all path."""
        if exchange.world != self.ep_size or exchange.rank != self.ep_rank:
            raise ValueError("exchange group does not match ep_rank / ep_size")
        self.ep_exchange = exchange

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if self.ep_exchange is not None:
            from ..engine.ep import ep_moe_forward_nvlink
            return ep_moe_forward_nvlink(self, hidden_states, self.ep_exchange)
        if self.ep_size > 1:
            if getattr(self, "expert_slot", None) is not None:
                raise NotImplementedError("a custom expert placement needs the NVLink exchange "
                                          "(attach_exchange)")
            from ..engine.sharding import ep_moe_forward
            return ep_moe_forward(self, hidden_states)
        return fused_moe(hidden_states, self.gate.weight, self.experts.gate_up_proj,
                         self.experts.down_proj, self.shared_expert.gate_proj.weight,
                         self.shared_expert.up_proj.weight, self.shared_expert.down_proj.weight,
                         self.shared_expert_gate.weight, self.top_k)

    def load_expert_shard(self, gate_up_full: torch.Tensor, down_full: torch.Tensor,
                          placement=None):
        """Copy this rank's experts out of full ``[E, ...]`` expert tensors (expert
        parallel).  Without ``placement`` rank r holds experts [r*E/P, (r+1)*E/P); with it
        (global expert ids in slot order, e.g. ``engine.ep.placement_by_load``) rank r
        holds ``placement[r*E/P:(r+1)*E/P]``, which the NVLink exchange routes by."""
        s, e = self.expert_base, self.expert_base + self.local_experts
        with torch.no_grad():
            if placement is None:
                self.experts.gate_up_proj.copy_(gate_up_full[s:e])
                self.experts.down_proj.copy_(down_full[s:e])
                self.expert_slot = None
                return
            pl = torch.as_tensor(placement, dtype=torch.int64)
            if sorted(pl.tolist()) != list(range(self.num_experts)):
                raise ValueError("placement must be a permutation of the experts")
            idx = pl[s:e].to(gate_up_full.device)
            self.experts.gate_up_proj.copy_(gate_up_full[idx])
            self.experts.down_proj.copy_(down_full[idx])
            slot = torch.empty(self.num_experts, dtype=torch.int32)
            slot[pl] = torch.arange(self.num_experts, dtype=torch.int32)
            self.expert_slot = slot.to(self.experts.gate_up_proj.device)
