"""Multi-process CPU tests (gloo, world size 2) of the tensor/expert-parallel host logic.

The exchange code of ``layerbatch_b200.engine.sharding`` is device-agnostic; here the
expert and attention compute is the CPU oracle, so these tests check the routing tables,
the all-to-all split sizes and orders, the head / column slicing and the reductions
without a GPU.  One test injects a failure on the host: a rank raises before the
exchange and the other rank's collective must end with an error (short timeout).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _expert_rows_fp32(p, rows, eids, ws):
    """The expert math for single (row, expert, weight) pairs, fp32 -> bf16 row."""
    out = torch.empty(rows.shape[0], rows.shape[1], dtype=torch.bfloat16)
    for i in range(rows.shape[0]):
        e = int(eids[i])
        h = rows[i].float() @ p.gate_up[e].float().t()
        g, u = h.chunk(2)
        y = (F.silu(g) * u) @ p.down[e].float().t()
        out[i] = (y * float(ws[i])).to(torch.bfloat16)
    return out


def _ep_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from layerbatch_b200 import workloads as W
        from layerbatch_b200.engine import sharding as S
        from oracle import moe as OM
        _init(rank, world, port)
        T, H, E, I, k = 24, 256, 16, 128, 4
        p = W.make_moe_params(H, E, I, I, k, seed=0)
        x = W.make_moe_input(T, H, seed=10 + rank)
        w, ids = OM.topk_route(OM.router_logits(x, p.router), k)
        plan = S.ep_plan(ids, E)
        rx, rid, rw = S.ep_dispatch(x, ids, w, plan)
        nl = E // world
        assert bool(((rid >= rank * nl) & (rid < (rank + 1) * nl)).all()), "pair sent to wrong owner"
        # every pair routed to this rank arrives exactly once
        all_ids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(all_ids, ids)
        mine = sum(int(((a >= rank * nl) & (a < (rank + 1) * nl)).sum()) for a in all_ids)
        assert rx.shape[0] == mine == sum(plan.recv_counts)
        y_recv = _expert_rows_fp32(p, rx, rid, rw)
        y_send = S.ep_return(y_recv, plan)
        assert y_send.shape[0] == T * k
        xf = x.float()
        shared = (F.silu(xf @ p.sh_gate.float().t()) * (xf @ p.sh_up.float().t())) @ p.sh_down.float().t()
        out = torch.sigmoid(xf @ p.sh_gate_w.float().t()) * shared
        out = out + y_send.float()[plan.pair_pos.long()].sum(dim=1)
        ref = OM.moe_block_fp32(x, p, ids, w)
        err = OM.rel_err(out, ref)
        assert err < 1e-2, err
        dist.destroy_process_group()
        q.put((rank, "ok", err))
    except Exception as e:  # report to the parent
        q.put((rank, "fail", repr(e)))


def _tp_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from layerbatch_b200 import workloads as W
        from layerbatch_b200.engine import sharding as S
        from oracle import attention as OA
        from oracle import moe as OM
        _init(rank, world, port)
        b = W.make_attn_batch([300, 40], [(64, 80)], Hq=16, Hkv=2, D=64, H=128, seed=7)
        shard = S.attention_shard(16, 2, rank, world)
        qs, g, kc, vc, wo = S.shard_attention_tensors(shard, b.q, b.gate, b.k_cache, b.v_cache,
                                                      b.w_o, 64)
        o = OA.paged_attention(qs, kc, vc, b.block_tables, b.context_lens, b.cu_seqlens_q, b.scale)
        N = o.shape[0]
        partial = OA.gate_oproj_fp32(o.reshape(N, -1), g.reshape(N, -1), wo)
        dist.all_reduce(partial)
        ref, _ = OA.attn_oproj_fp32(b)
        err = OM.rel_err(partial, ref)
        assert err < 1e-5, err
        dist.destroy_process_group()
        q.put((rank, "ok", err))
    except Exception as e:
        q.put((rank, "fail", repr(e)))


def _fault_worker(rank, world, port, q):
    """Rank 1 raises before the exchange; rank 0's collective must fail, not hang."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from layerbatch_b200.engine import sharding as S
    _init(rank, world, port, timeout_s=5)
    ids = torch.randint(0, 8, (6, 2))
    if rank == 1:
        q.put((rank, "raised", "injected failure before dispatch"))
        q.close()
        q.join_thread()
        os._exit(0)  # leaves without joining the collective
    try:
        S.ep_plan(ids, 8)
        q.put((rank, "no error", ""))
    except Exception as e:
        q.put((rank, "error", type(e).__name__))


def _run(fn, world=2, timeout=150):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res)


def test_expert_parallel_exchange_gloo():
    res = _run(_ep_worker)
    assert all(r[1] == "ok" for r in res), res


def test_tensor_parallel_head_shards_gloo():
    res = _run(_tp_worker)
    assert all(r[1] == "ok" for r in res), res


def test_rank_failure_surfaces_as_collective_error():
    res = _run(_fault_worker)
    status = dict((r[0], r[1]) for r in res)
    assert status[1] == "raised"
    assert status[0] == "error", res
