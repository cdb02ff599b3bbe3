"""GPU tests of the drop-in layer modules that mirror the reference's operator API:
``Attention`` driven by the forward context, the POD decode entry points, the MoE block
module with the reference's parameter names, and the tensor-parallel linears at tp = 1.
"""
import pytest
import torch

from layerbatch_b200 import workloads as W
from layerbatch_b200.layers import attention as LA
from layerbatch_b200.layers.fused_moe import (Qwen3_5Experts, Qwen3_5SharedExpertMLP,
                                               Qwen3_5SparseMoeBlock, Qwen3_5TopKRouter)
from layerbatch_b200.layers.linear import (MergedColumnParallelLinear, QKVParallelLinear,
                                           ReplicatedLinear)
from layerbatch_b200.utils.context import reset_context, set_context
from oracle import attention as OA
from oracle import moe as OM

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def test_attention_module_decode_and_prefill(cuda):
    """store_kvcache + attention through the context, as Qwen3_5FullAttention calls it."""
    Hq, Hkv, D = 16, 2, 256
    # decode: 3 sequences whose last token is new
    b = W.make_attn_batch([700, 33, 256], (), seed=21)
    k_new = torch.randn(3, Hkv, D).to(torch.bfloat16)
    v_new = torch.randn(3, Hkv, D).to(torch.bfloat16)
    slots = []
    for i, c in enumerate(b.ctx_list):
        blk = int(b.block_tables[i, (c - 1) // 256])
        slots.append(blk * 256 + (c - 1) % 256)
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    kc, vc = b.k_cache.clone(), b.v_cache.clone()
    OA.store_kvcache(k_new, v_new, kc, vc, slot_mapping)
    ref = OA.paged_attention(b.q, kc, vc, b.block_tables, b.context_lens, b.cu_seqlens_q, b.scale)
    attn = LA.Attention(Hq, D, b.scale, Hkv)
    attn.k_cache, attn.v_cache = b.k_cache.to(cuda), b.v_cache.to(cuda)
    set_context(False, slot_mapping=slot_mapping.to(cuda), context_lens=b.context_lens.to(cuda),
                block_tables=b.block_tables.to(cuda))
    o = attn(b.q.to(cuda), k_new.to(cuda), v_new.to(cuda))
    torch.cuda.synchronize()
    assert o.shape == (3, 1, Hq, D)
    assert OM.rel_err(o.squeeze(1).cpu(), ref) <= TOL
    # prefill without a prefix cache: no block tables in the context (reference path
    # attention.py:118-127); the tables are recovered from the slot mapping
    L = 300
    nb = 4
    perm = torch.randperm(nb).to(torch.int32)
    q = torch.randn(L, Hq, D).to(torch.bfloat16)
    k = torch.randn(L, Hkv, D).to(torch.bfloat16)
    v = torch.randn(L, Hkv, D).to(torch.bfloat16)
    slot = torch.tensor([int(perm[i // 256]) * 256 + i % 256 for i in range(L)], dtype=torch.int32)
    kc = torch.zeros(nb, 256, Hkv, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    attn.k_cache, attn.v_cache = kc.to(cuda), vc.to(cuda)
    cu = torch.tensor([0, L], dtype=torch.int32)
    set_context(True, cu_seqlens_q=cu.to(cuda), cu_seqlens_k=cu.to(cuda), max_seqlen_q=L,
                max_seqlen_k=L, slot_mapping=slot.to(cuda))
    o = attn(q.to(cuda), k.to(cuda), v.to(cuda))
    torch.cuda.synchronize()
    reset_context()
    OA.store_kvcache(k, v, kc, vc, slot)
    bt = torch.full((1, 2), -1, dtype=torch.int32)
    bt[0, :2] = perm[:2]
    ref = OA.paged_attention(q, kc, vc, bt, torch.tensor([L], dtype=torch.int32), cu, D ** -0.5)
    assert OM.rel_err(o.cpu(), ref) <= TOL


def test_pod_decode_entry_points(cuda):
    b = W.make_attn_batch([1200, 77, 4000], (), seed=22)
    g = b.to(cuda)
    o = LA.pod_attn_only(g.q, g.k_cache, g.v_cache, g.block_tables, g.context_lens, g.scale,
                         num_kv_splits=4)
    A = torch.randn(5, 64, device=cuda).to(torch.bfloat16)
    Bm = torch.randn(64, 96, device=cuda).to(torch.bfloat16)
    C = torch.empty(5, 96, dtype=torch.bfloat16, device=cuda)
    o2 = LA.pod_fused_attn_gemm(g.q, g.k_cache, g.v_cache, g.block_tables, g.context_lens,
                                g.scale, A, Bm, C)
    torch.cuda.synchronize()
    ref = OA.paged_attention(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                             b.cu_seqlens_q, b.scale)
    assert OM.rel_err(o.cpu(), ref) <= TOL and OM.rel_err(o2.cpu(), ref) <= TOL
    assert OM.rel_err(C.cpu(), A.cpu().float() @ Bm.cpu().float()) <= 1e-2


def test_moe_block_module_loads_reference_names(cuda):
    H, E, I, k, T = 2048, 64, 512, 8, 40
    p = W.make_moe_params(H, E, I, I, k, seed=5)
    blk = Qwen3_5SparseMoeBlock(H, E, k, I, I).to(torch.bfloat16)
    sd = {"gate.weight": p.router, "experts.gate_up_proj": p.gate_up,
          "experts.down_proj": p.down, "shared_expert.gate_proj.weight": p.sh_gate,
          "shared_expert.up_proj.weight": p.sh_up, "shared_expert.down_proj.weight": p.sh_down,
          "shared_expert_gate.weight": p.sh_gate_w}
    blk.load_state_dict(sd)
    blk = blk.to(cuda)
    x = W.make_moe_input(T, H, seed=6)
    y = blk(x.to(cuda))
    tw, ti = blk.gate(x.to(cuda))
    torch.cuda.synchronize()
    logits = OM.router_logits(x, p.router)
    w32, ids = OM.topk_route(logits, k)
    assert bool(OM.same_up_to_ties(ti.cpu(), ids, logits).all())
    y32 = OM.moe_block_fp32(x, p, ti.cpu(), w32)
    assert OM.rel_err(y.cpu(), y32) <= TOL
    assert isinstance(blk.gate, Qwen3_5TopKRouter) and tw.dtype == torch.bfloat16


def test_replicated_linear(cuda):
    lin = ReplicatedLinear(512, 256).to(torch.bfloat16).to(cuda)
    with torch.no_grad():
        lin.weight.normal_(0, 0.02)
    x = torch.randn(3, 7, 512, device=cuda).to(torch.bfloat16)
    y = lin(x)
    torch.cuda.synchronize()
    assert y.shape == (3, 7, 256)
    assert OM.rel_err(y, x.float() @ lin.weight.float().t()) <= 1e-2


def test_experts_and_shared_expert_modules(cuda):
    """``Qwen3_5Experts.forward(x, ids, w)`` and ``Qwen3_5SharedExpertMLP.forward(x)``, the
    block's two halves called on their own as the reference's block calls them
    (qwen3_5.py:899-905), against the fp32 oracle; their sum with the sigmoid gate is the
    block's output."""
    H, E, I, k, T = 2048, 64, 512, 8, 37
    p = W.make_moe_params(H, E, I, I, k, seed=15)
    x = W.make_moe_input(T, H, seed=16)
    w32, ids = OM.topk_route(OM.router_logits(x, p.router), k)
    ex = Qwen3_5Experts(E, H, I).to(torch.bfloat16)
    se = Qwen3_5SharedExpertMLP(H, I).to(torch.bfloat16)
    with torch.no_grad():
        ex.gate_up_proj.copy_(p.gate_up)
        ex.down_proj.copy_(p.down)
        se.gate_proj.weight.copy_(p.sh_gate)
        se.up_proj.weight.copy_(p.sh_up)
        se.down_proj.weight.copy_(p.sh_down)
    ex, se = ex.to(cuda), se.to(cuda)
    xd = x.to(cuda)
    y_e = ex(xd, ids.to(cuda), w32.to(torch.bfloat16).to(cuda))
    y_s = se(xd)
    torch.cuda.synchronize()
    assert OM.rel_err(y_e.cpu(), OM.experts_fp32(x, p.gate_up, p.down, ids, w32.to(torch.bfloat16))) <= TOL
    assert OM.rel_err(y_s.cpu(), OM.shared_expert_fp32(x, p.sh_gate, p.sh_up, p.sh_down)) <= TOL
    # an expert-parallel shard: only ids in [16, 48) contribute
    part = Qwen3_5Experts(32, H, I).to(torch.bfloat16)
    with torch.no_grad():
        part.gate_up_proj.copy_(p.gate_up[16:48])
        part.down_proj.copy_(p.down[16:48])
    part = part.to(cuda)
    part.expert_base, part.total_experts = 16, E
    y_p = part(xd, ids.to(cuda), w32.to(cuda))
    torch.cuda.synchronize()
    ref_p = OM.experts_fp32(x, p.gate_up[16:48], p.down[16:48], ids, w32, expert_base=16)
    assert OM.rel_err(y_p.cpu(), ref_p) <= TOL


def test_merged_and_qkv_linears_load_shards_and_compute_one_gemm(cuda):
    H = 512
    qkv = QKVParallelLinear(H, 64, 4, 2).to(torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    wq, wk, wv = (0.02 * torch.randn(n, H, generator=g) for n in (4 * 64, 2 * 64, 2 * 64))
    for wt, sid in ((wq, "q"), (wk, "k"), (wv, "v")):
        qkv.weight.weight_loader(qkv.weight, wt.to(torch.bfloat16), sid)
    mc = MergedColumnParallelLinear(H, [256, 256]).to(torch.bfloat16)
    wa, wb = (0.02 * torch.randn(256, H, generator=g) for _ in range(2))
    mc.weight.weight_loader(mc.weight, wa.to(torch.bfloat16), 0)
    mc.weight.weight_loader(mc.weight, wb.to(torch.bfloat16), 1)
    qkv, mc = qkv.to(cuda), mc.to(cuda)
    x = torch.randn(9, H, generator=g).to(torch.bfloat16)
    y, z = qkv(x.to(cuda)), mc(x.to(cuda))
    torch.cuda.synchronize()
    ref_y = x.float() @ torch.cat([wq, wk, wv]).to(torch.bfloat16).float().t()
    ref_z = x.float() @ torch.cat([wa, wb]).to(torch.bfloat16).float().t()
    assert OM.rel_err(y.cpu(), ref_y) <= 1e-2 and OM.rel_err(z.cpu(), ref_z) <= 1e-2
