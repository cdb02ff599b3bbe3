"""Expert-parallel MoE over NVLink peer memory: the host side of ``lb_ep_moe_forward``.

``EPExchange`` owns this rank's exchange buffer (allocated by the library with
``cudaMalloc`` and exported as a CUDA IPC handle), all-gathers the handles over the
process group and maps every other rank's buffer, so the dispatch and return kernels can
store token rows straight into the owner's / source's memory over NVLink.  The reference
has no expert parallelism (every rank holds every expert, nanovllm/models/qwen3_5.py:
795-800); the result of one call equals ``Qwen3_5SparseMoeBlock.forward`` on this rank's
tokens (qwen3_5.py:899-905).

Exchange buffers are sized for ``capacity`` tokens per rank and call.  No host
synchronisation happens per call: routing tables, row counts and the epoch flags that
order the phases across GPUs all live on the devices.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .. import ops
from .._lib import LB_EP_MAX_RANKS, LbEpArgs, check, lib, ptr, stream_ptr
from .peer import PeerBuffers


class EPExchange(PeerBuffers):
    """This rank's mapping of the exchange buffers of one expert-parallel group, sized
    for ``capacity`` tokens per rank and call."""

    def __init__(self, capacity: int, hidden: int, top_k: int, group=None, device=None,
                 _local=None):
        self.capacity, self.hidden, self.top_k = capacity, hidden, top_k
        world = _local[1] if _local is not None else dist.get_world_size(group)
        if world > LB_EP_MAX_RANKS:
            raise ValueError(f"expert-parallel group of {world} > {LB_EP_MAX_RANKS} ranks")
        super().__init__(lib().lb_ep_buffer_size(world, capacity, hidden, top_k), group,
                         device, _local)

    @classmethod
    def emulated(cls, world: int, capacity: int, hidden: int, top_k: int, device=None):
        """``world`` ranks' exchanges in one process on one device (single-GPU tests):
        the phases of all ranks are then issued in order on one stream."""
        nbytes = lib().lb_ep_buffer_size(world, capacity, hidden, top_k)
        return cls._emulated(world, nbytes, device,
                             lambda _local: cls(capacity, hidden, top_k, device=device,
                                                _local=_local))


def ep_args(block, x: torch.Tensor, ex: EPExchange, out: torch.Tensor, phases: int = 0,
            events=None) -> LbEpArgs:
    T, H = x.shape
    a = LbEpArgs()
    a.num_tokens, a.capacity, a.hidden = T, ex.capacity, H
    a.num_experts, a.top_k = block.num_experts, block.top_k
    a.inter = block.experts.down_proj.shape[2]
    a.rank, a.world = ex.rank, ex.world
    a.x, a.out = ptr(x), ptr(out)
    a.w_router = ptr(block.gate.weight)
    a.w_gate_up = ptr(block.experts.gate_up_proj)
    a.w_down = ptr(block.experts.down_proj)
    se = block.shared_expert
    a.w_shared_gate, a.w_shared_up = ptr(se.gate_proj.weight), ptr(se.up_proj.weight)
    a.w_shared_down = ptr(se.down_proj.weight)
    a.w_shared_expert_gate = ptr(block.shared_expert_gate.weight)
    for r, p in enumerate(ex.peers):
        a.peer_bufs[r] = p
    a.phases = phases
    slot = getattr(block, "expert_slot", None)
    if slot is not None:
        a.expert_slot = slot.data_ptr()
    ops._events(a, events)
    return a


def placement_by_load(loads, world: int) -> torch.Tensor:
    """Experts of every rank by popularity: heaviest expert first, each to the rank with
    the least load so far that still has room (E/P experts per rank).  ``loads`` [E] are
    routed pairs per expert from a calibration batch (the same on every rank).  Returns the
    placement: global expert ids in slot order (rank r holds slots [r*E/P, (r+1)*E/P))."""
    loads = torch.as_tensor(loads, dtype=torch.float64).cpu()
    E = loads.numel()
    epr = E // world
    order = sorted(range(E), key=lambda e: (-float(loads[e]), e))
    acc = [0.0] * world
    held = [[] for _ in range(world)]
    for e in order:
        r = min((r for r in range(world) if len(held[r]) < epr), key=lambda r: (acc[r], r))
        held[r].append(e)
        acc[r] += float(loads[e])
    return torch.tensor([e for r in range(world) for e in sorted(held[r])], dtype=torch.int64)


def ep_moe_forward_nvlink(block, x: torch.Tensor, ex: EPExchange, out=None, phases: int = 0,
                          events=None, ws_tag: str | None = None) -> torch.Tensor:
    """One expert-parallel MoE block call on this rank's tokens ``x [T, H]`` (T <= the
    exchange capacity).  ``block`` holds this rank's expert shard
    (``Qwen3_5SparseMoeBlock(..., ep_rank, ep_size)``)."""
    x = x.contiguous()
    if x.shape[0] > ex.capacity:
        raise ValueError(f"{x.shape[0]} tokens exceed the exchange capacity {ex.capacity}")
    if out is None:
        out = torch.empty_like(x)
    a = ep_args(block, x, ex, out, phases, events)
    L = lib()
    n = C.c_size_t(0)
    check(L.lb_ep_workspace_size(C.byref(a), C.byref(n)), "lb_ep_workspace_size")
    ws = ops.workspace(n.value, x.device, ws_tag or f"ep{ex.rank}")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    check(L.lb_ep_moe_forward(C.byref(a), stream_ptr()), "lb_ep_moe_forward")
    return out
