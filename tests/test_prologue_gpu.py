"""Attention prologue on B200: ``lb_attn_prologue`` (fused (1+w) RMSNorm + partial RoPE of
query and key + K/V cache store) against the CPU oracle, and the drop-in
``Qwen3_5FullAttention`` layer (projections -> prologue -> POD attention + gate + o_proj)
against the oracle chain of the reference's forward (qwen3_5.py:707-746).
"""
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from layerbatch_b200.layers.full_attention import Qwen3_5FullAttention
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


def _bf16_close(a, b, min_exact=0.999):
    a, b = a.float().cpu(), b.float().cpu()
    exact = float((a == b).float().mean())
    # one bf16 ulp of |b| (2^-7 relative) where they differ
    ulp = torch.clamp(b.abs(), min=1e-30) * 2.0 ** -7
    assert exact >= min_exact, exact
    assert bool(((a - b).abs() <= ulp + 1e-30).all()), float((a - b).abs().max())


@pytest.mark.parametrize("rot", [64, 0, 256])
def test_attn_prologue_matches_oracle(cuda, rot):
    N, Hq, Hkv, D, max_pos = 37, 16, 2, 256, 40000
    g = torch.Generator().manual_seed(3)
    q_out = torch.randn(N, Hq * 2 * D, generator=g).to(torch.bfloat16)
    k_raw = (3 * torch.randn(N, Hkv * D, generator=g)).to(torch.bfloat16)
    v_raw = torch.randn(N, Hkv * D, generator=g).to(torch.bfloat16)
    qw = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    kw = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (N,), generator=g)
    pos[0], pos[1] = 0, max_pos - 1
    nb = 3
    slots = torch.randperm(nb * 256, generator=g)[:N].to(torch.int32)
    slots[5] = -1                                   # padding token: no store
    cache = OA.rope_cos_sin_cache(max(rot, 16), max_pos, 1.0e7)
    if rot == 0:
        cache = cache[..., :0]
    k_cache = torch.zeros(nb, 256, Hkv, D, dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    dk, dv = k_cache.to(cuda), v_cache.to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    qd = q_out.to(cuda).view(N, Hq, 2 * D)
    query = ops.attn_prologue(qd[..., :D], k_raw.to(cuda).view(N, Hkv, D),
                              v_raw.to(cuda).view(N, Hkv, D), qw.to(cuda), kw.to(cuda),
                              cache.contiguous().to(cuda), pos.to(cuda), slots.to(cuda), dk, dv,
                              1e-6, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    if rot == 0:   # no rotation: the norms alone
        rq = OA.rmsnorm_1pw(q_out.view(N, Hq, 2 * D)[..., :D], qw, 1e-6)
        rk = OA.rmsnorm_1pw(k_raw.view(N, Hkv, D), kw, 1e-6)
        rv = v_raw.view(N, Hkv, D)
    else:
        rq, _, rk, rv = OA.attn_prologue(q_out, k_raw, v_raw, qw, kw, cache, pos, 1e-6, Hq, D)
    _bf16_close(query, rq)
    OA.store_kvcache(rk, rv, k_cache, v_cache, slots)
    _bf16_close(dk, k_cache)
    assert torch.equal(dv.cpu(), v_cache)


def _module(cuda, seed=9):
    H, Hq, Hkv, D = 2048, 16, 2, 256
    m = Qwen3_5FullAttention(H, Hq, Hkv, D, max_position=40000, rms_norm_eps=1e-6,
                             rope_theta=1.0e7)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for lin in (m.q_proj, m.k_proj, m.v_proj, m.o_proj):
            lin.weight.copy_(0.02 * torch.randn(lin.weight.shape, generator=g))
        m.q_norm.weight.copy_(0.1 * torch.randn(D, generator=g))
        m.k_norm.weight.copy_(0.1 * torch.randn(D, generator=g))
    return m.to(torch.bfloat16).to(cuda)


def _oracle_layer(m, x, pos, k_cache, v_cache, slots, tables, ctx, cu):
    """The reference forward restated on the CPU: bf16 projections with fp32
    accumulation, prologue, K/V store, paged attention, gate and o_proj in fp32."""
    w = {n: getattr(m, n).weight.detach().cpu().float() for n in ("q_proj", "k_proj", "v_proj", "o_proj")}
    xf = x.float()
    q_out = (xf @ w["q_proj"].t()).to(torch.bfloat16)
    k_raw = (xf @ w["k_proj"].t()).to(torch.bfloat16)
    v_raw = (xf @ w["v_proj"].t()).to(torch.bfloat16)
    cache = m.rotary_emb.cos_sin_cache.cpu()
    q, gate, k, v = OA.attn_prologue(q_out, k_raw, v_raw, m.q_norm.weight.cpu(),
                                     m.k_norm.weight.cpu(), cache, pos, 1e-6, m.num_heads,
                                     m.head_dim)
    OA.store_kvcache(k, v, k_cache, v_cache, slots)
    o = OA.paged_attention(q, k_cache, v_cache, tables, ctx, cu, m.scaling)
    N = x.shape[0]
    return OA.gate_oproj_fp32(o.reshape(N, -1), gate, w["o_proj"].to(torch.bfloat16))


def test_full_attention_layer_decode(cuda):
    m = _module(cuda)
    b = W.make_attn_batch([700, 33, 256, 1900], (), seed=21)
    N = len(b.ctx_list)
    x = torch.randn(N, 2048, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    pos = torch.tensor([c - 1 for c in b.ctx_list], dtype=torch.long)
    slots = torch.tensor([int(b.block_tables[i, (c - 1) // 256]) * 256 + (c - 1) % 256
                          for i, c in enumerate(b.ctx_list)], dtype=torch.int32)
    kc, vc = b.k_cache.clone(), b.v_cache.clone()
    ref = _oracle_layer(m, x, pos, kc, vc, slots, b.block_tables, b.context_lens, b.cu_seqlens_q)
    m.attn.k_cache, m.attn.v_cache = b.k_cache.to(cuda), b.v_cache.to(cuda)
    set_context(False, slot_mapping=slots.to(cuda), context_lens=b.context_lens.to(cuda),
                block_tables=b.block_tables.to(cuda))
    try:
        y = m(pos.to(cuda), x.to(cuda))
        torch.cuda.synchronize()
    finally:
        reset_context()
    assert y.shape == (N, 2048)
    assert OM.rel_err(y.cpu(), ref) <= TOL
    # the new tokens' K/V landed in the cache as the oracle stored them
    _bf16_close(m.attn.k_cache.cpu()[:, :, :, :].reshape(-1, 512)[slots.long()],
                kc.reshape(-1, 512)[slots.long()], min_exact=0.99)


def test_full_attention_layer_prefill(cuda):
    m = _module(cuda, seed=10)
    L, nb = 300, 4
    g = torch.Generator().manual_seed(6)
    x = torch.randn(L, 2048, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    slots = torch.tensor([int(perm[i // 256]) * 256 + i % 256 for i in range(L)], dtype=torch.int32)
    pos = torch.arange(L, dtype=torch.long)
    kc = torch.zeros(nb, 256, 2, 256, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    bt = torch.full((1, 2), -1, dtype=torch.int32)
    bt[0, :2] = perm[:2]
    cu = torch.tensor([0, L], dtype=torch.int32)
    ref = _oracle_layer(m, x, pos, kc.clone(), vc.clone(), slots, bt,
                        torch.tensor([L], dtype=torch.int32), cu)
    m.attn.k_cache, m.attn.v_cache = kc.to(cuda), vc.to(cuda)
    set_context(True, cu_seqlens_q=cu.to(cuda), cu_seqlens_k=cu.to(cuda), max_seqlen_q=L,
                max_seqlen_k=L, slot_mapping=slots.to(cuda))
    try:
        y = m(pos.to(cuda), x.to(cuda))
        torch.cuda.synchronize()
    finally:
        reset_context()
    assert OM.rel_err(y.cpu(), ref) <= TOL


def test_full_attention_layer_mixed_step_from_scheduler(cuda):
    """One step of the mixed scheduler (a prompt chunk on its cached prefix plus decode
    tokens of finished prompts) through the layer in one POD launch."""
    from layerbatch_b200.engine.batch_builder import (MixedScheduler, Sequence, prepare_mixed,
                                                      set_mixed_context)
    m = _module(cuda, seed=12)
    sched = MixedScheduler(num_blocks=24, max_num_batched_tokens=700, chunk_size=600)
    seqs = [Sequence([0] * n, max_tokens=4) for n in (900, 130, 257)]
    for s in seqs:
        sched.add(s)
    for _ in range(2):                          # the three prompts, in chunks
        b = sched.schedule()
        sched.postprocess(b, {s.seq_id: 1 for s in seqs})
    late = Sequence([0] * 800, max_tokens=4)
    sched.add(late)
    b = sched.schedule()                        # 3 decodes + the first 600 of the late prompt
    sched.postprocess(b, {s.seq_id: 1 for s in seqs + [late]})
    step = sched.schedule()                     # 3 decodes + its last 200 on a 600 prefix
    assert [(i.start, i.length) for i in step.prefill] == [(600, 200)]
    assert step.prefill and step.decode, "expected a mixed step"
    meta = prepare_mixed(step)
    N = int(meta["cu_seqlens_q"][-1])
    g = torch.Generator().manual_seed(13)
    x = torch.randn(N, 2048, generator=g).to(torch.bfloat16)
    # cache: earlier steps' K/V stand in as random values; this step overwrites its slots
    kc = torch.randn(24, 256, 2, 256, generator=g).to(torch.bfloat16)
    vc = torch.randn(24, 256, 2, 256, generator=g).to(torch.bfloat16)
    ref = _oracle_layer(m, x, meta["positions"], kc.clone(), vc.clone(), meta["slot_mapping"],
                        meta["block_tables"], meta["context_lens"], meta["cu_seqlens_q"])
    m.attn.k_cache, m.attn.v_cache = kc.to(cuda), vc.to(cuda)
    dmeta = prepare_mixed(step, device=cuda)
    set_mixed_context(dmeta)
    try:
        y = m(dmeta["positions"], x.to(cuda))
        torch.cuda.synchronize()
    finally:
        reset_context()
    assert OM.rel_err(y.cpu(), ref) <= TOL


def test_fused_prologue_equals_the_separate_launch(cuda):
    """The prologue fused into the attention kernel (its CTAs normalise, rotate and store
    the batch's rows first; each item waits for its sequence) and fused into the q/k/v
    projection GEMM's epilogue (lb_qkv_prologue_gemm) give bit for bit what the separate
    lb_attn_prologue launch gives: the query rows, the stored K/V rows, the layer output.
    Two prefill chunks (one on a prefix) and decode steps, one token a padding token
    (slot -1: its K/V are not stored)."""
    b = W.make_attn_batch([700, 33, 1900, 256, 2], [(300, 200), (0, 129)], seed=41)
    N = b.num_tokens
    lp = W.make_attn_layer_params(seed=42, device=cuda)
    pos, slots = W.layer_positions_slots(b)
    slots[N - 1] = -1
    x = W.make_layer_input(N, 2048, seed=43, device=cuda)
    g = b.to(cuda)
    outs = {}
    for mode in ("kernel", "pod", "gemm"):
        kc, vc = g.k_cache.clone(), g.v_cache.clone()
        q = torch.empty(N, 16, 256, dtype=torch.bfloat16, device=cuda)
        attn = torch.empty(N, 16 * 256, dtype=torch.bfloat16, device=cuda)
        y = ops.gated_attention_layer(
            x, lp.w_qkv, 16, 2, lp.q_norm_w, lp.k_norm_w, lp.cos_sin_cache, lp.eps,
            pos.to(cuda), slots.to(cuda), kc, vc, g.block_tables, g.context_lens,
            g.cu_seqlens_q, g.w_o, g.scale, max_q_len=200, q=q, attn_out=attn,
            ws_tag=f"fused_{mode}", prologue=mode)
        torch.cuda.synchronize()
        assert ops.device_status(ops.workspace(0, cuda, f"fused_{mode}")) == 0
        assert ops.device_status(ops.workspace(0, cuda, f"fused_{mode}_prologue")) == 0
        assert ops.device_status(ops.workspace(0, cuda, "gemm")) == 0
        outs[mode] = (y, q, attn, kc, vc)
    for mode in ("pod", "gemm"):
        for a, r in zip(outs[mode], outs["kernel"]):
            assert torch.equal(a, r), mode
    # and the padding token's slot was left alone
    last = int(b.block_tables[b.num_seqs - 1, 0]) * 256 + 1
    for mode in outs:
        assert torch.equal(outs[mode][3].view(-1, 2, 256)[last], g.k_cache.view(-1, 2, 256)[last])


def test_qkv_prologue_gemm_reports_bad_positions_and_slots(cuda):
    """lb_qkv_prologue_gemm checks each token's position and slot like lb_attn_prologue:
    a position outside the rotary table and a slot past the cache are reported in the
    status word (and skipped or clamped), never read or written out of bounds."""
    b = W.make_attn_batch([300, 40], [(0, 64)], seed=51)
    N = b.num_tokens
    lp = W.make_attn_layer_params(seed=52, device=cuda)
    pos, slots = W.layer_positions_slots(b)
    g = b.to(cuda)
    x = W.make_layer_input(N, 2048, seed=53, device=cuda)
    for bad_pos, bad_slot in ((True, False), (False, True)):
        p2, s2 = pos.clone(), slots.clone()
        if bad_pos:
            p2[3] = lp.cos_sin_cache.shape[0] + 5
        if bad_slot:
            s2[5] = g.k_cache.shape[0] * 256 + 7
        kc, vc = g.k_cache.clone(), g.v_cache.clone()
        tag = f"qkvbad{int(bad_pos)}{int(bad_slot)}"
        ops.gated_attention_layer(
            x, lp.w_qkv, 16, 2, lp.q_norm_w, lp.k_norm_w, lp.cos_sin_cache, lp.eps,
            p2.to(cuda), s2.to(cuda), kc, vc, g.block_tables, g.context_lens, g.cu_seqlens_q,
            g.w_o, g.scale, max_q_len=64, ws_tag=tag, prologue="gemm")
        torch.cuda.synchronize()
        assert ops.device_status(ops.workspace(0, cuda, tag + "_prologue")) == 2   # LB_DEV_BAD_INDEX


def test_qkv_prologue_gemm_rejects_other_rotary_dims(cuda):
    """The GEMM-epilogue prologue handles head_dim 256 with 64 rotated dims; another
    rotary_dim is refused with LB_ERR_UNSUPPORTED before anything is launched, and the layer
    call falls back to the separate prologue launch (same results as prologue="kernel")."""
    import ctypes as C
    from layerbatch_b200._lib import lib
    b = W.make_attn_batch([300, 40], [(0, 64)], seed=61)
    N = b.num_tokens
    lp = W.make_attn_layer_params(seed=62, device=cuda)
    cs32 = lp.cos_sin_cache[:, :32].contiguous()   # a 32-dim rotary table
    pos, slots = W.layer_positions_slots(b)
    g = b.to(cuda)
    x = W.make_layer_input(N, 2048, seed=63, device=cuda)
    qkv = torch.empty(N, lp.w_qkv.shape[0], dtype=torch.bfloat16, device=cuda)
    q = torch.empty(N, 16, 256, dtype=torch.bfloat16, device=cuda)
    q3 = qkv[:, :16 * 512].view(N, 16, 512)
    k_in = qkv[:, 16 * 512:16 * 512 + 512].view(N, 2, 256)
    v_in = qkv[:, 16 * 512 + 512:].view(N, 2, 256)
    a, keep = ops.prologue_args(q3[..., :256], k_in, v_in, lp.q_norm_w, lp.k_norm_w, cs32,
                                pos.to(cuda), slots.to(cuda), g.k_cache, g.v_cache, lp.eps, q)
    ws = ops.workspace(256, cuda, "gemm")
    n0 = ops.launch_count()
    rc = lib().lb_qkv_prologue_gemm(x.data_ptr(), x.stride(0), lp.w_qkv.data_ptr(),
                                    lp.w_qkv.stride(0), qkv.data_ptr(), qkv.stride(0),
                                    x.shape[1], C.byref(a), ws.data_ptr(), None)
    assert rc == 2 and ops.launch_count() == n0
    outs = {}
    for mode in ("gemm", "kernel"):
        kc, vc = g.k_cache.clone(), g.v_cache.clone()
        outs[mode] = ops.gated_attention_layer(
            x, lp.w_qkv, 16, 2, lp.q_norm_w, lp.k_norm_w, cs32, lp.eps, pos.to(cuda),
            slots.to(cuda), kc, vc, g.block_tables, g.context_lens, g.cu_seqlens_q, g.w_o,
            g.scale, max_q_len=64, ws_tag=f"rot32_{mode}", prologue=mode)
    torch.cuda.synchronize()
    assert torch.equal(outs["gemm"], outs["kernel"])
