"""Tensor-parallel o_proj reduction over peer memory (``lb_pod_attn_oproj`` with
``tp_bufs``), emulated on one GPU.

Two or four ranks live in one process, each with its KV-head shard of the attention
(whole GQA groups), W_o's matching columns, its own exchange buffer mapping every
rank's, and its own workspace.  The three phases of a call (attention + o_proj GEMM whose
epilogue stores each fp32 tile into the owning rank's inbox; owner reduction and
broadcast; gather) are issued for all ranks in order on one stream, so every bounded
wait finds its flags set.  Each rank must end with the same bf16 rows, within 2e-2 of the
single-GPU fused call; two consecutive calls exercise the epochs.
"""
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from layerbatch_b200._lib import LB_TP_PHASE_ATTN, LB_TP_PHASE_GATHER, LB_TP_PHASE_REDUCE
from layerbatch_b200.engine import sharding as S
from layerbatch_b200.engine.peer import TPExchange
from oracle import moe as OM

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


@pytest.mark.parametrize("P,Hq,Hkv,decode,prefill", [
    (2, 16, 2, [900, 2000, 64], [(128, 300)]),    # 303 rows: tiles 0,2 -> rank 0, 1 -> rank 1
    (2, 16, 2, [700, 33], []),                     # 2 rows: rank 1 owns no tile
    (4, 16, 4, [300, 4000, 1500, 77, 2048], [(0, 520)]),
])
def test_tp_oproj_peer_reduction_emulated(cuda, P, Hq, Hkv, decode, prefill):
    exs = None
    try:
        for call in range(2):
            b = W.make_attn_batch(decode, prefill, Hq=Hq, Hkv=Hkv, seed=40 + call).to(cuda)
            mq = max(b.qlen_list)
            full = ops.pod_attn_oproj(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables,
                                      b.context_lens, b.cu_seqlens_q, b.w_o, b.scale,
                                      max_q_len=mq, ws_tag="tp_full")
            N, H = b.num_tokens, b.w_o.shape[0]
            if exs is None:
                exs = TPExchange.emulated(P, 1024, H, device=cuda)
            parts = []
            for r in range(P):
                sh = S.attention_shard(Hq, Hkv, r, P)
                parts.append(S.shard_attention_tensors(sh, b.q, b.gate, b.k_cache, b.v_cache,
                                                       b.w_o, 256))
            outs = [torch.full((N, H), float("nan"), dtype=torch.bfloat16, device=cuda)
                    for _ in range(P)]
            for ph in (LB_TP_PHASE_ATTN, LB_TP_PHASE_REDUCE, LB_TP_PHASE_GATHER):
                for r in range(P):
                    qs, gs, kc, vc, wo = parts[r]
                    ops.pod_attn_oproj(qs, gs, kc, vc, b.block_tables, b.context_lens,
                                       b.cu_seqlens_q, wo, b.scale, out=outs[r], max_q_len=mq,
                                       ws_tag=f"tp_emu{r}", tp=exs[r], tp_phases=ph)
            torch.cuda.synchronize()
            for r in range(P):
                assert ops.device_status(ops._WS[(torch.cuda.current_device(), f"tp_emu{r}")]) == 0
                assert torch.equal(outs[r], outs[0]), r
            assert OM.rel_err(outs[0].float(), full.float()) <= TOL
    finally:
        if exs is not None:
            exs[0].close()


def test_tp_reduce_wait_times_out_and_reports(cuda):
    """Rank 0 of an emulated TP pair reduces while rank 1 never computes its partials: the
    owner's wait gives up after its time limit with LB_DEV_TIMEOUT, and the context
    stays usable."""
    b = W.make_attn_batch([700, 900], [], seed=45).to(cuda)
    exs = TPExchange.emulated(2, 256, 2048, device=cuda)
    try:
        sh = S.attention_shard(16, 2, 0, 2)
        qs, gs, kc, vc, wo = S.shard_attention_tensors(sh, b.q, b.gate, b.k_cache, b.v_cache,
                                                       b.w_o, 256)
        ops.pod_attn_oproj(qs, gs, kc, vc, b.block_tables, b.context_lens, b.cu_seqlens_q, wo,
                           b.scale, max_q_len=1, ws_tag="tp_dead_peer", tp=exs[0])
        torch.cuda.synchronize()
        assert ops.device_status(ops._WS[(torch.cuda.current_device(), "tp_dead_peer")]) == 1
        full = ops.pod_attn_oproj(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables,
                                  b.context_lens, b.cu_seqlens_q, b.w_o, b.scale, max_q_len=1,
                                  ws_tag="tp_after_timeout")
        torch.cuda.synchronize()
        assert bool(torch.isfinite(full.float()).all())
    finally:
        exs[0].close()
