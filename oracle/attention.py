"""CPU oracle of the paged attention + output gate + o_proj tail.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates:

* ``store_kvcache`` (nanovllm/layers/attention.py:50-80): scatter of new K/V rows into
  ``[num_blocks, 256, Hkv, D]`` by ``slot_mapping``, skipping slot -1;
* ``sdpa_decode_paged`` (nanovllm/layers/sdpa_fallback.py:121-159): one query per sequence
  over its pages;
* prefill over a cached prefix (attention.py:104-141): causal attention where query i of
  a chunk of length L on a sequence of context C sits at absolute position C-L+i and sees
  keys [0, C-L+i].  This is flash-attn's bottom-right causal alignment, the reference's
  default GPU path (attention.py:124-127).  The reference's SDPA fallback
  (sdpa_fallback.py:108 via ``_sdpa_one_seq``) passes ``is_causal=True`` to
  ``F.scaled_dot_product_attention``, which aligns top-left when Sq != Sk; for Sq == Sk
  (no prefix) both agree, and the golden vectors pin that case;
* the split-KV online softmax with LSE merge of the POD kernel
  (nanovllm/layers/pod_kernels.py:102-159 and 205-231), in fp32;
* ``o * sigmoid(gate)`` then o_proj (nanovllm/models/qwen3_5.py:742-746);
* the full-attention prologue (qwen3_5.py:707-736): the per-head (query, gate) split of the
  q_proj output, the (1 + w) RMSNorm of query and key (qwen3_5.py:39-55) and the partial
  rotary embedding of their first ``rotary_dim`` dims with the fp32 cos/sin cache
  (nanovllm/layers/rotary_embedding.py:5-54).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def store_kvcache(k, v, k_cache, v_cache, slot_mapping):
    """attention.py:50-80: ``cache.flat[slot] = row`` for slot != -1 (one indexed copy of
    the kept rows, the index-assignment form of attention.py:62-70)."""
    nb, bs, hkv, d = k_cache.shape
    kc = k_cache.view(nb * bs, hkv, d)
    vc = v_cache.view(nb * bs, hkv, d)
    keep = slot_mapping.long() != -1
    s = slot_mapping.long()[keep]
    kc[s] = k[keep].to(kc.dtype)
    vc[s] = v[keep].to(vc.dtype)


def gather_pages(cache, table_row, n):
    """Concatenate the first ``n`` token rows of a sequence's pages -> [n, Hkv, D]."""
    bs = cache.shape[1]
    pieces, rem = [], n
    for blk in table_row[: (n + bs - 1) // bs]:
        take = min(bs, rem)
        pieces.append(cache[int(blk), :take])
        rem -= take
    return torch.cat(pieces, 0)


def _sdpa_one_seq(q, k, v, scale, causal):
    """sdpa_fallback.py:34-58 restated: [Sq,Hq,D] x [Sk,Hkv,D] -> [Sq,Hq,D]."""
    hq, hkv = q.shape[1], k.shape[1]
    qq = q.transpose(0, 1).unsqueeze(0)
    kk = k.transpose(0, 1).unsqueeze(0)
    vv = v.transpose(0, 1).unsqueeze(0)
    if hkv != hq:
        kk = kk.repeat_interleave(hq // hkv, dim=1)
        vv = vv.repeat_interleave(hq // hkv, dim=1)
    o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal, scale=scale)
    return o.squeeze(0).transpose(0, 1)


def paged_decode_bf16(q, k_cache, v_cache, block_tables, context_lens, scale):
    """sdpa_decode_paged restated (sdpa_fallback.py:121-159); returns [B, 1, Hq, D]."""
    outs = []
    for i, n in enumerate(context_lens.tolist()):
        row = block_tables[i].tolist()
        k = gather_pages(k_cache, row, n)
        v = gather_pages(v_cache, row, n)
        outs.append(_sdpa_one_seq(q[i].unsqueeze(0), k, v, scale, causal=False))
    return torch.stack(outs, 0)


def paged_prefill_bf16(q, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, scale):
    """``sdpa_prefill_varlen`` with block tables restated (sdpa_fallback.py:61-118), bf16.

    The reference gathers each sequence's pages and calls SDPA with ``is_causal=True``;
    here the mask is given explicitly in bottom-right form so that a chunk on a cached
    prefix sees the prefix (identical to the reference when there is no prefix).
    """
    cu = cu_seqlens_q.tolist()
    out = torch.empty_like(q)
    for b, c in enumerate(context_lens.tolist()):
        s, e = cu[b], cu[b + 1]
        L = e - s
        if L == 0:
            continue
        row = block_tables[b].tolist()
        k = gather_pages(k_cache, row, c)
        v = gather_pages(v_cache, row, c)
        hq, hkv = q.shape[1], k.shape[1]
        qq = q[s:e].transpose(0, 1).unsqueeze(0)
        kk = k.transpose(0, 1).unsqueeze(0).repeat_interleave(hq // hkv, dim=1)
        vv = v.transpose(0, 1).unsqueeze(0).repeat_interleave(hq // hkv, dim=1)
        mask = torch.arange(c).view(1, c) <= torch.arange(c - L, c).view(L, 1)
        o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=scale)
        out[s:e] = o.squeeze(0).transpose(0, 1)
    return out


def paged_attention(q, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, scale,
                    dtype=torch.float32):
    """Mixed prefill + decode attention over paged KV, bottom-right causal.

    ``q`` is ``[N, Hq, D]`` packed by ``cu_seqlens_q``; sequence b owns query rows
    ``cu[b]:cu[b+1]`` which are its last ``L_b`` positions of ``context_lens[b]``.
    Computed in ``dtype`` (fp32 by default) with an explicit mask.  Returns ``[N, Hq, D]``.
    """
    cu = cu_seqlens_q.tolist()
    out = torch.empty(q.shape, dtype=dtype, device=q.device)
    hq = q.shape[1]
    for b, c in enumerate(context_lens.tolist()):
        s, e = cu[b], cu[b + 1]
        L = e - s
        if L == 0:
            continue
        row = block_tables[b].tolist()
        k = gather_pages(k_cache, row, c).to(dtype)
        v = gather_pages(v_cache, row, c).to(dtype)
        hkv = k.shape[1]
        k = k.repeat_interleave(hq // hkv, dim=1)       # [C, Hq, D]
        v = v.repeat_interleave(hq // hkv, dim=1)
        qq = q[s:e].to(dtype)                            # [L, Hq, D]
        sc = torch.einsum("lhd,chd->hlc", qq, k) * scale
        qpos = torch.arange(c - L, c, device=q.device).view(L, 1)
        kpos = torch.arange(c, device=q.device).view(1, c)
        sc = sc.masked_fill((kpos > qpos).unsqueeze(0), float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s:e] = torch.einsum("hlc,chd->lhd", p, v)
    return out


def attention_rows_fp32(q_rows, positions, k, v, scale):
    """Attention of selected query rows of ONE sequence over its gathered keys, in fp32.

    Row i sits at absolute position ``positions[i]`` and sees keys ``[0, positions[i]]``:
    the bottom-right causal rule of a chunk on a cached prefix (attention.py:104-141,
    flash-attn varlen) and, for the last position, the decode query
    (sdpa_fallback.py:121-159).  ``q_rows [R, Hq, D]``, ``k``/``v`` ``[C, Hkv, D]``;
    returns ``[R, Hq, D]`` fp32.  Lets a check cover a sample of a long chunk's rows
    without the whole ``[L, C]`` score matrix.
    """
    hq, hkv = q_rows.shape[1], k.shape[1]
    kk = k.float().repeat_interleave(hq // hkv, dim=1)
    vv = v.float().repeat_interleave(hq // hkv, dim=1)
    sc = torch.einsum("rhd,chd->hrc", q_rows.float(), kk) * scale
    kpos = torch.arange(k.shape[0], device=k.device).view(1, -1)
    mask = kpos > positions.to(k.device).view(-1, 1)
    sc = sc.masked_fill(mask.unsqueeze(0), float("-inf"))
    p = torch.softmax(sc, dim=-1)
    return torch.einsum("hrc,chd->rhd", p, vv)


def split_kv_decode_fp32(q, k_cache, v_cache, block_tables, context_lens, scale, num_splits):
    """POD split-KV decode + LSE merge restated in fp32 (pod_kernels.py:102-159, 205-231).

    Split s of a sequence of length n covers ``[s*ceil(n/S), min((s+1)*ceil(n/S), n))``.
    Returns ``[B, Hq, D]`` fp32.
    """
    B, hq, d = q.shape
    out = torch.zeros(B, hq, d)
    for b, n in enumerate(context_lens.tolist()):
        row = block_tables[b].tolist()
        k = gather_pages(k_cache, row, n).float()
        v = gather_pages(v_cache, row, n).float()
        hkv = k.shape[1]
        k = k.repeat_interleave(hq // hkv, dim=1)
        v = v.repeat_interleave(hq // hkv, dim=1)
        per = -(-n // num_splits)
        acc = torch.zeros(hq, d)
        e_sum = torch.zeros(hq)
        e_max = torch.full((hq,), float("-inf"))
        for s in range(num_splits):
            lo, hi = per * s, min(per * (s + 1), n)
            if hi <= lo:
                continue
            qk = torch.einsum("hd,chd->hc", q[b].float(), k[lo:hi]) * scale
            m = qk.max(-1).values
            p = torch.exp(qk - m[:, None])
            l = p.sum(-1)
            o = torch.einsum("hc,chd->hd", p, v[lo:hi]) / l[:, None]
            lse = m + torch.log(l)
            n_max = torch.maximum(lse, e_max)
            old = torch.exp(e_max - n_max)
            new = torch.exp(lse - n_max)
            acc = acc * old[:, None] + new[:, None] * o
            e_sum = e_sum * old + new
            e_max = n_max
        out[b] = acc / e_sum[:, None]
    return out


def gate_oproj_bf16(o_flat, gate_flat, w_o):
    """qwen3_5.py:742-746 at tp=1: ``F.linear(o * sigmoid(gate), W_o)`` in bf16."""
    return F.linear(o_flat * torch.sigmoid(gate_flat), w_o)


def gate_oproj_fp32(o_flat, gate_flat, w_o):
    return (o_flat.float() * torch.sigmoid(gate_flat.float())) @ w_o.float().t()


def attn_oproj_fp32(batch):
    """The full fused op in fp32 on an ``AttnBatch``: attention -> gate -> o_proj."""
    o = paged_attention(batch.q, batch.k_cache, batch.v_cache, batch.block_tables,
                        batch.context_lens, batch.cu_seqlens_q, batch.scale)
    N = o.shape[0]
    return gate_oproj_fp32(o.reshape(N, -1), batch.gate.reshape(N, -1), batch.w_o), o


def default_scale(head_dim):
    """qwen3_5.py:638: ``head_dim ** -0.5``."""
    return head_dim ** -0.5 if head_dim else math.nan


# ------------------------------------------------------------------------------ prologue
def rmsnorm_1pw(x, w, eps):
    """qwen3_5.py:48-55: fp32 ``x * rsqrt(mean(x^2) + eps) * (1 + w)``, back to x's dtype."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * (1.0 + w.float())).to(x.dtype)


def rope_cos_sin_cache(rotary_dim, max_position, base):
    """rotary_embedding.py:26-33: ``[max_position, 1, rotary_dim]`` fp32, cos then sin."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


def _rotate(x, cos, sin):
    """rotary_embedding.py:6-14 (halves of the rotated dims, fp32, back to x's dtype)."""
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


def partial_rope(positions, query, key, cos_sin_cache):
    """rotary_embedding.py:36-54: rotate the first ``rotary_dim`` dims of every head."""
    rot = cos_sin_cache.shape[-1]
    cos, sin = cos_sin_cache[positions.long()].chunk(2, dim=-1)
    out = []
    for x in (query, key):
        out.append(torch.cat([_rotate(x[..., :rot], cos, sin), x[..., rot:]], dim=-1))
    return out[0], out[1]


def attn_prologue(q_out, k_raw, v_raw, q_norm_w, k_norm_w, cos_sin_cache, positions, eps,
                  num_heads, head_dim):
    """qwen3_5.py:707-736 after the projections: ``q_out [N, Hq*2D]`` -> (query [N,Hq,D]
    normed + rotated, gate [N, Hq*D], key [N,Hkv,D] normed + rotated, value [N,Hkv,D])."""
    N = q_out.shape[0]
    q3 = q_out.view(N, num_heads, 2 * head_dim)
    query, gate = q3.chunk(2, dim=-1)
    gate = gate.reshape(N, num_heads * head_dim)
    k = k_raw.view(N, -1, head_dim)
    v = v_raw.view(N, -1, head_dim)
    query = rmsnorm_1pw(query, q_norm_w, eps)
    k = rmsnorm_1pw(k, k_norm_w, eps)
    query, k = partial_rope(positions, query, k, cos_sin_cache)
    return query, gate, k, v
