"""Peer-mapped device buffers of one node's ranks (CUDA IPC through the library).

Each rank allocates one buffer with ``lb_ep_buffer_alloc`` (``cudaMalloc``, zeroed, IPC
handle exported), the 64-byte handles are all-gathered over the process group once, and
every rank maps every other rank's buffer (``lb_ep_buffer_open``).  The kernels that use
them (expert-parallel dispatch / return, the tensor-parallel o_proj reduction) store
straight into the peers' memory over NVLink and order their phases with epoch flags in
the buffers' headers.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .._lib import LB_EP_IPC_HANDLE_BYTES, LB_EP_MAX_RANKS, check, lib


def _alloc(nbytes):
    h = (C.c_uint8 * LB_EP_IPC_HANDLE_BYTES)()
    p = C.c_void_p()
    check(lib().lb_ep_buffer_alloc(nbytes, C.byref(p), h), "lb_ep_buffer_alloc")
    return p.value, h


class PeerBuffers:
    """This rank's view of one buffer per rank of a group: ``peers[r]`` is rank r's
    buffer as mapped in this process (``peers[rank]`` is its own)."""

    def __init__(self, nbytes: int, group=None, device=None, _local=None):
        self.nbytes = nbytes
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self._opened, self._owned = [], []
        if _local is not None:            # emulated ranks in one process (tests)
            self.rank, self.world, self.peers = _local
            return
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > LB_EP_MAX_RANKS:
            raise ValueError(f"peer group of {self.world} > {LB_EP_MAX_RANKS} ranks")
        L = lib()
        own, handle = _alloc(nbytes)
        self._owned.append(own)
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(every, mine, group=group)
        self.peers = []
        for r, h in enumerate(every):
            if r == self.rank:
                self.peers.append(own)
                continue
            hb = (C.c_uint8 * LB_EP_IPC_HANDLE_BYTES).from_buffer_copy(bytes(h.cpu().tolist()))
            p = C.c_void_p()
            check(L.lb_ep_buffer_open(hb, C.byref(p)), "lb_ep_buffer_open")
            self._opened.append(p.value)
            self.peers.append(p.value)
        dist.barrier(group=group)

    @classmethod
    def _emulated(cls, world: int, nbytes: int, device, make):
        bufs = [_alloc(nbytes)[0] for _ in range(world)]
        out = [make(_local=(r, world, list(bufs))) for r in range(world)]
        out[0]._owned = bufs
        return out

    def close(self):
        """Unmap the peers and free this rank's buffer (every rank must be done with it)."""
        torch.cuda.synchronize(self.device)
        L = lib()
        for p in self._opened:
            check(L.lb_ep_buffer_close(p), "lb_ep_buffer_close")
        for p in self._owned:
            check(L.lb_ep_buffer_free(p), "lb_ep_buffer_free")
        self._opened, self._owned = [], []


class TPExchange(PeerBuffers):
    """Buffers of the tensor-parallel o_proj reduction of ``lb_pod_attn_oproj``: up to
    ``capacity`` token rows of ``hidden`` outputs per call."""

    def __init__(self, capacity: int, hidden: int, group=None, device=None, _local=None):
        self.capacity, self.hidden = capacity, hidden
        world = _local[1] if _local is not None else dist.get_world_size(group)
        super().__init__(lib().lb_tp_buffer_size(world, capacity, hidden), group, device, _local)

    @classmethod
    def emulated(cls, world: int, capacity: int, hidden: int, device=None):
        nbytes = lib().lb_tp_buffer_size(world, capacity, hidden)
        return cls._emulated(world, nbytes, device,
                             lambda _local: cls(capacity, hidden, device=device, _local=_local))
