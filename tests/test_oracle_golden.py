"""Pin the CPU oracle against golden vectors produced by the reference's own modules.

CPU only.  Inputs are regenerated from seeds; their SHA-256 must match the fixture.
"""
import numpy as np
import pytest
import torch

from layerbatch_b200 import workloads as W
from oracle import attention as OA
from oracle import moe as OM
from tests.golden.make_golden import (MOE_CASES, DECODE_CASES, PREFILL_CASES, PROLOGUE_CASES,
                                     moe_inputs, prologue_inputs, sha, tie_inputs)


def assert_bf16_match(a, b, min_exact=0.99, rel=1e-2):
    """Same torch ops on the same inputs: expect (near) bitwise equality.

    A different CPU may pick different oneDNN kernels, so allow rare last-bit changes.
    """
    a = a.float()
    b = b.float()
    exact = float((a == b).float().mean())
    err = OM.rel_err(a, b)
    assert exact >= min_exact and err <= rel, (exact, err)


@pytest.mark.parametrize("name", list(MOE_CASES))
def test_moe_oracle_matches_reference(golden, name):
    g = golden[name]
    T, H, E, I, Is, k, zipf = MOE_CASES[name]
    p, x = moe_inputs(T, H, E, I, Is, k, zipf)
    assert sha(x) == g["x_sha"]
    logits = OM.router_logits(x, p.router)
    assert_bf16_match(logits, g["logits"])
    w, ids = OM.topk_route(g["logits"], k)
    assert bool(OM.same_up_to_ties(ids, g["topk_ids"], g["logits"]).all())
    # the oracle's expert math on the reference's own routing reproduces its output
    y = OM.moe_block_bf16(x, p, "sparse", ids=g["topk_ids"], w=g["topk_w"])
    assert_bf16_match(y, g["y_sparse"])
    if "y_dense" in g:
        y = OM.moe_block_bf16(x, p, "dense", ids=g["topk_ids"], w=g["topk_w"])
        assert_bf16_match(y, g["y_dense"])
    # fp32 oracle agrees with the bf16 reference within the parity tolerance
    w32, ids32 = OM.topk_route_reference(g["logits"], k, torch.float32)
    assert torch.equal(ids32, g["topk_ids"])
    y32 = OM.moe_block_fp32(x, p, ids32, w32)
    assert OM.rel_err(g["y_sparse"], y32) < 2e-2


def test_router_ties(golden):
    g = golden["router_ties"]
    x, w, k = tie_inputs()
    assert sha(x) == g["x_sha"]
    logits = OM.router_logits(x, w)
    assert torch.equal(logits, g["logits"])
    vals, ids = OM.topk_route(logits, k)
    # the fixture must actually contain ties inside the selection or across its boundary
    srt = torch.sort(logits.float(), 1, descending=True).values
    assert bool((srt[:, :k] == srt[:, 1:k + 1]).any())
    assert bool(OM.same_up_to_ties(ids, g["topk_ids"], logits).all())
    # lowest-index tie-break: equal logits appear in ascending expert order
    for r in range(ids.shape[0]):
        lr = logits[r, ids[r]].float()
        for j in range(k - 1):
            if lr[j] == lr[j + 1]:
                assert ids[r, j] < ids[r, j + 1]
    ref_w, _ = OM.topk_route_reference(logits, k)
    assert torch.allclose(vals.to(torch.bfloat16).float().sort(1).values,
                          ref_w.float().sort(1).values)


def test_permutation_matches_reference_order():
    """Order inside an expert equals torch.where(expert_mask[e]) (qwen3_5.py:823-831)."""
    T, E, k = 50, 12, 3
    g = torch.Generator().manual_seed(7)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    counts, offsets, ptok, pslot, row_of = OM.permutation(ids.numpy(), E)
    mask = torch.nn.functional.one_hot(ids, E).permute(2, 1, 0)
    for e in range(E):
        pos, tok = torch.where(mask[e])
        s, t = offsets[e], offsets[e + 1]
        assert counts[e] == tok.numel()
        assert np.array_equal(ptok[s:t], tok.numpy())
        assert np.array_equal(pslot[s:t], pos.numpy())
    for t in range(T):
        for j in range(k):
            r = row_of[t, j]
            assert ptok[r] == t and pslot[r] == j
    # ids outside [0, G) are dropped (expert owned by another rank)
    c2, o2, pt2, ps2, r2 = OM.permutation(ids.numpy(), E // 2)
    assert c2.sum() == int((ids < E // 2).sum())
    assert (r2[ids.numpy() >= E // 2] == -1).all()


@pytest.mark.parametrize("name", list(DECODE_CASES))
def test_decode_oracle_matches_reference(golden, name):
    g = golden[name]
    b = W.make_attn_batch(DECODE_CASES[name], (), seed=3)
    assert sha(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.w_o) == g["in_sha"]
    o = OA.paged_decode_bf16(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens, b.scale)
    assert_bf16_match(o, g["attn"])
    y = OA.gate_oproj_bf16(o.flatten(1, -1), b.gate.reshape(b.num_tokens, -1), b.w_o)
    assert_bf16_match(y, g["y"])
    o32 = OA.paged_attention(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                             b.cu_seqlens_q, b.scale)
    assert OM.rel_err(g["attn"].squeeze(1), o32) < 1e-2
    y32 = OA.gate_oproj_fp32(o32.reshape(b.num_tokens, -1), b.gate.reshape(b.num_tokens, -1), b.w_o)
    assert OM.rel_err(g["y"], y32) < 2e-2
    for splits in (1, 3, 16):
        osplit = OA.split_kv_decode_fp32(b.q, b.k_cache, b.v_cache, b.block_tables,
                                         b.context_lens, b.scale, splits)
        assert OM.rel_err(osplit, o32) < 1e-5


@pytest.mark.parametrize("name", list(PREFILL_CASES))
def test_prefill_oracle_matches_reference(golden, name):
    g = golden[name]
    b = W.make_attn_batch([], PREFILL_CASES[name], seed=4)
    assert sha(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.w_o) == g["in_sha"]
    o32 = OA.paged_attention(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                             b.cu_seqlens_q, b.scale)
    assert OM.rel_err(g["attn"], o32) < 1e-2


def test_prefix_prefill_is_bottom_right_causal():
    """With a cached prefix, query i of the chunk sees keys [0, prefix + i]."""
    b = W.make_attn_batch([], [(300, 20)], seed=9, Hq=4, Hkv=2, D=64, H=64)
    o = OA.paged_attention(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                           b.cu_seqlens_q, b.scale)
    # last query row == a decode step over the full context
    last = OA.paged_attention(b.q[-1:], b.k_cache, b.v_cache, b.block_tables,
                              b.context_lens, torch.tensor([0, 1], dtype=torch.int32), b.scale)
    assert torch.allclose(o[-1], last[0], atol=1e-5)
    # first query row sees exactly prefix + 1 keys
    first_ctx = torch.tensor([301], dtype=torch.int32)
    first = OA.paged_attention(b.q[:1], b.k_cache, b.v_cache, b.block_tables, first_ctx,
                               torch.tensor([0, 1], dtype=torch.int32), b.scale)
    assert torch.allclose(o[0], first[0], atol=1e-5)


@pytest.mark.parametrize("name", list(PROLOGUE_CASES))
def test_prologue_oracle_matches_reference(golden, name):
    """(query, gate) split, (1+w) RMSNorm and partial RoPE of the full-attention prologue."""
    g = golden[name]
    N, Hq, Hkv, D, rot, max_pos, theta, seed = PROLOGUE_CASES[name]
    q_out, k_raw, v_raw, q_w, k_w, pos = prologue_inputs(N, Hq, Hkv, D, max_pos, seed)
    assert sha(q_out, k_raw, v_raw, q_w, k_w, pos) == g["in_sha"]
    cache = OA.rope_cos_sin_cache(rot, max_pos, theta)
    assert torch.equal(cache[pos], g["cos_sin_rows"])
    query, gate, k, _ = OA.attn_prologue(q_out, k_raw, v_raw, q_w, k_w, cache, pos, 1e-6, Hq, D)
    assert torch.equal(gate, g["gate"])
    assert_bf16_match(query, g["query"], min_exact=0.999, rel=1e-2)
    assert_bf16_match(k, g["key"], min_exact=0.999, rel=1e-2)
