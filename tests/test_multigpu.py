"""Tensor / expert parallel on 2 GPUs (skipped with fewer than 2 GPUs).

Each rank compares the sharded result with the single-GPU library call on the same
inputs: attention TP by KV head with the fp32 o_proj all-reduce and with the reduction
over peer memory, the whole gated attention layer (projections, prologue and K/V store of
each rank's heads, attention, o_proj reduced over peer memory), the MoE block with
experts split over the ranks and the NCCL all-to-all exchange, and the MoE block with the
NVLink peer-memory exchange (``lb_ep_moe_forward``).  NVLS is off (plain NCCL transport,
no multicast objects) and the process group has a short timeout.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch.distributed as dist
        from layerbatch_b200 import ops
        from layerbatch_b200 import workloads as W
        from layerbatch_b200.engine import sharding as S
        from layerbatch_b200.layers.fused_moe import Qwen3_5SparseMoeBlock
        from oracle import moe as OM
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        errs = {}
        # ---- attention, TP by KV head
        b = W.make_attn_batch([900, 2000, 64], [(128, 300)], seed=31).to(dev)
        full = ops.pod_attn_oproj(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables,
                                  b.context_lens, b.cu_seqlens_q, b.w_o, b.scale, max_q_len=300,
                                  ws_tag="full")
        shard = S.attention_shard(16, 2, rank, world)
        qs, gs, kc, vc, wo = S.shard_attention_tensors(shard, b.q, b.gate, b.k_cache, b.v_cache,
                                                       b.w_o, 256)
        tp = S.tp_attention_oproj(shard, qs, gs, kc, vc, b.block_tables, b.context_lens,
                                  b.cu_seqlens_q, wo, b.scale, max_q_len=300)
        errs["tp"] = OM.rel_err(tp.float(), full.float())
        # the same with the o_proj reduction fused over peer memory (no NCCL)
        from layerbatch_b200.engine.peer import TPExchange
        tpx = TPExchange(1024, 2048, device=dev)
        for _ in range(2):
            tp2 = S.tp_attention_oproj(shard, qs, gs, kc, vc, b.block_tables, b.context_lens,
                                       b.cu_seqlens_q, wo, b.scale, max_q_len=300, exchange=tpx)
        torch.cuda.synchronize()
        errs["tp_peer"] = OM.rel_err(tp2.float(), full.float())
        # ---- the whole gated attention layer, TP by KV head (the bench's sharded step):
        # each rank projects its own heads (its rows of the merged q/k/v weight), stores
        # its KV head's new rows into its cache slice and reduces o_proj over peer memory
        lp = W.make_attn_layer_params(seed=5, device=dev)
        pos, slots = W.layer_positions_slots(b)
        pos, slots = pos.to(dev), slots.to(dev)
        x_attn = W.make_layer_input(b.num_tokens, 2048, seed=6, device=dev)
        kc_full, vc_full = b.k_cache.clone(), b.v_cache.clone()
        full_l = ops.gated_attention_layer(
            x_attn, lp.w_qkv, 16, 2, lp.q_norm_w, lp.k_norm_w, lp.cos_sin_cache, lp.eps, pos,
            slots, kc_full, vc_full, b.block_tables, b.context_lens, b.cu_seqlens_q, b.w_o,
            b.scale, max_q_len=300, ws_tag="full_layer")
        D = 256
        hs, ks = shard.q_heads, shard.kv_heads
        w_loc = torch.cat([lp.w_qkv[hs.start * 2 * D:hs.stop * 2 * D],
                           lp.w_qkv[16 * 2 * D + ks.start * D:16 * 2 * D + ks.stop * D],
                           lp.w_qkv[16 * 2 * D + 2 * D + ks.start * D:
                                    16 * 2 * D + 2 * D + ks.stop * D]]).contiguous()
        kc_l = b.k_cache[:, :, ks].contiguous()
        vc_l = b.v_cache[:, :, ks].contiguous()
        tpx2 = TPExchange(1024, 2048, device=dev)
        for _ in range(2):
            tp_l = ops.gated_attention_layer(
                x_attn, w_loc, hs.stop - hs.start, ks.stop - ks.start, lp.q_norm_w,
                lp.k_norm_w, lp.cos_sin_cache, lp.eps, pos, slots, kc_l, vc_l, b.block_tables,
                b.context_lens, b.cu_seqlens_q, wo, b.scale, max_q_len=300,
                ws_tag=f"tp_layer{rank}", tp=tpx2)
        torch.cuda.synchronize()
        errs["tp_layer"] = OM.rel_err(tp_l.float(), full_l.float())
        # the K/V rows this rank stored equal the single-GPU layer's rows of its head
        errs["tp_layer_cache"] = float(not (torch.equal(kc_l, kc_full[:, :, ks]) and
                                            torch.equal(vc_l, vc_full[:, :, ks])))
        errs["tp_layer_status"] = float(ops.device_status(ops._WS[(rank, f"tp_layer{rank}")]))
        dist.barrier()
        tpx2.close()
        tpx.close()
        # ---- MoE, expert parallel with all-to-all
        H, E, I, k, T = 2048, 64, 512, 8, 96 + 32 * rank
        p = W.make_moe_params(H, E, I, I, k, seed=0).to(dev)
        x = W.make_moe_input(T, H, seed=40 + rank).to(dev)
        blk = Qwen3_5SparseMoeBlock(H, E, k, I, I, ep_rank=rank, ep_size=world).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            blk.gate.weight.copy_(p.router)
            blk.load_expert_shard(p.gate_up, p.down)
            blk.shared_expert.gate_proj.weight.copy_(p.sh_gate)
            blk.shared_expert.up_proj.weight.copy_(p.sh_up)
            blk.shared_expert.down_proj.weight.copy_(p.sh_down)
            blk.shared_expert_gate.weight.copy_(p.sh_gate_w)
            y_ep = blk(x)
        y_1 = ops.moe_forward(x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up, p.sh_down,
                              p.sh_gate_w, k, ws_tag="moe_full")
        torch.cuda.synchronize()
        errs["ep"] = OM.rel_err(y_ep.float(), y_1.float())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", errs))
    except Exception as e:
        q.put((rank, "fail", repr(e)))


def _nvlink_worker(rank, world, port, q):
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch.distributed as dist
        from layerbatch_b200 import ops
        from layerbatch_b200 import workloads as W
        from layerbatch_b200.engine.ep import EPExchange, ep_moe_forward_nvlink
        from layerbatch_b200.layers.fused_moe import Qwen3_5SparseMoeBlock
        from oracle import moe as OM
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        H, E, I, k, C = 2048, 512, 512, 10, 512
        p = W.make_moe_params(H, E, I, I, k, seed=0).to(dev)
        blk = Qwen3_5SparseMoeBlock(H, E, k, I, I, ep_rank=rank, ep_size=world).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            blk.gate.weight.copy_(p.router)
            blk.load_expert_shard(p.gate_up, p.down)
            blk.shared_expert.gate_proj.weight.copy_(p.sh_gate)
            blk.shared_expert.up_proj.weight.copy_(p.sh_up)
            blk.shared_expert.down_proj.weight.copy_(p.sh_down)
            blk.shared_expert_gate.weight.copy_(p.sh_gate_w)
        ex = EPExchange(C, H, k, device=dev)
        errs = {}
        for call, T in enumerate([384 + 64 * rank, 200 - 150 * rank, 512]):
            x = W.make_moe_input(T, H, seed=50 + 10 * call + rank).to(dev)
            y = ep_moe_forward_nvlink(blk, x, ex)
            y1 = ops.moe_forward(x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up, p.sh_down,
                                 p.sh_gate_w, k, ws_tag="moe_full")
            torch.cuda.synchronize()
            errs[f"call{call}"] = OM.rel_err(y.float(), y1.float())
        errs["status"] = ops.device_status(ops._WS[(rank, f"ep{rank}")])
        dist.barrier()
        ex.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", errs))
    except Exception as e:
        q.put((rank, "fail", repr(e)))


def _run2(fn):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    return res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_ep_moe_nvlink_exchange_on_two_gpus():
    res = _run2(_nvlink_worker)
    assert all(r[1] == "ok" for r in res), res
    for _, _, errs in res:
        assert errs.pop("status") == 0, errs
        assert all(v <= 2e-2 for v in errs.values()), errs


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_tp_attention_and_ep_moe_on_two_gpus():
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    assert all(r[1] == "ok" for r in res), res
    for _, _, errs in res:
        assert errs["tp"] <= 2e-2 and errs["ep"] <= 2e-2 and errs["tp_peer"] <= 2e-2, errs
        assert errs["tp_layer"] <= 2e-2, errs
        assert errs["tp_layer_cache"] == 0 and errs["tp_layer_status"] == 0, errs
