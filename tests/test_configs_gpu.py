"""GPU parity at the benchmark configurations' full sizes, on the launch shapes bench.py
times: C2 (a 2048-token chunk on a 2048-token prefix plus 128 decode sequences), C3 (the
E=512 top-10 MoE at T=256 and T=8192 under a Zipf(1.1) load) and the C4 hybrid step (the
whole gated attention layer over 512 decode sequences of up to 16384 tokens plus a
4096-token chunk, then the MoE at T=4608).  Inputs are drawn exactly as bench.py draws
them.

Every check compares the CUDA path with ``oracle/``:

* routing: router logits within one bf16 ulp of the exactly rounded product, top-k ids
  bit-exact against the oracle given the kernel's logits, and the expert permutation
  bit-exact against the oracle, over all T tokens;
* outputs: ``max|y - y32| / max|y32| <= 2e-2`` against the fp32 oracle, on EVERY row with
  the oracle's torch code evaluated in fp32 on the GPU (TF32 off), and on a seeded sample
  of rows with the oracle on the CPU: prefill rows spread over the whole chunk (first and
  last rows of every region included), 32 decode sequences (the longest and shortest
  included), and MoE tokens including those routed to the three hottest experts (whose
  long token-tile loops the Zipf load exercises);
* the attention prologue of the C4 layer within one bf16 ulp of the oracle, on the rows
  it stored into the paged cache and on the query rows it wrote.
"""
import numpy as np
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from oracle import attention as OA
from oracle import moe as OM

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda")


def _status_ok(dev, tag):
    assert ops.device_status(ops.workspace(0, dev, tag)) == 0, tag


def _bf16_within_ulp(a, b, min_exact=0.999):
    a, b = a.float().cpu(), b.float().cpu()
    exact = float((a == b).float().mean())
    ulp = torch.clamp(torch.maximum(a.abs(), b.abs()), min=1e-30) * 2.0 ** -7
    assert exact >= min_exact, exact
    assert bool(((a - b).abs() <= ulp + 1e-30).all()), float((a - b).abs().max())


# ------------------------------------------------------------------------------ MoE
def _moe_inputs(dev, T):
    """bench.py's MoE inputs: weights seed 0, tokens seed 1, Zipf(1.1) router bias."""
    p = W.make_moe_params(2048, 512, 512, 512, 10, seed=0, device=dev)
    x = W.make_moe_input(T, 2048, seed=1, device=dev)
    W.apply_zipf_bias(p, x)
    return p, x


def _check_moe_full(dev, T, p, x, out, logits, ids):
    k, E = 10, 512
    ids_c = ids.cpu().long()
    logits_c = logits.cpu()
    # router logits (F.linear in bf16 with fp32 accumulation, qwen3_5.py:769) against the
    # exact product (fp64 on the GPU): within one bf16 ulp plus the fp32 summation error
    # allowed for K = 2048 terms (2^-17 of sum |x w|; it only matters where the Zipf bias
    # column cancels the rest of the sum and the logit is near zero)
    exact = x.double() @ p.router.double().t()
    absum = x.double().abs() @ p.router.double().abs().t()
    ref = exact.to(torch.bfloat16).cpu()
    d = (logits_c.float() - ref.float()).abs()
    ulp = torch.maximum(ref.float().abs(), logits_c.float().abs()) * 2 ** -7
    slack = (absum * 2.0 ** -17).float().cpu()
    assert bool((d <= ulp + slack + 1e-6).all()), float((d / (ulp + slack)).max())
    assert float((d == 0).float().mean()) > 0.99
    del exact, absum
    # routing bit-exact given the kernel's logits, every token
    w32, ids_ref = OM.topk_route(logits_c, k)
    assert torch.equal(ids_c, ids_ref)
    # the permutation of all T*k pairs bit-exact
    row_start, perm_token, row_of = ops.moe_permute(ids, 0, E)
    torch.cuda.synchronize()
    counts, offsets, ptok, _, rof = OM.permutation(ids_c.numpy(), E)
    rs = row_start.cpu().numpy()
    assert rs[0] == 0 and rs[1] == T and np.array_equal(rs[1:] - T, offsets)
    pt = perm_token.cpu().numpy()
    assert np.array_equal(pt[:T], np.arange(T)) and np.array_equal(pt[T:T + T * k], ptok)
    assert np.array_equal(row_of.cpu().numpy(), np.where(rof >= 0, rof + T, -1))
    # every row against the fp32 oracle evaluated on the GPU
    y32 = OM.moe_block_fp32(x, p, ids.long(), w32.to(dev))
    err = OM.rel_err(out, y32)
    assert err <= TOL, err
    assert bool(torch.isfinite(out.float()).all())
    # a sample of rows against the CPU oracle: 256 seeded tokens plus up to 96 tokens of
    # each of the three hottest experts (its first and last routed token included)
    g = torch.Generator().manual_seed(T)
    hot = np.argsort(-counts, kind="stable")[:3]
    sub = set(torch.randperm(T, generator=g)[:256].tolist())
    for e in hot:
        tok = (ids_c == int(e)).any(dim=1).nonzero().flatten()
        pick = tok[torch.randperm(tok.numel(), generator=g)[:94]].tolist()
        sub.update(pick + [int(tok[0]), int(tok[-1])])
    sub = torch.tensor(sorted(sub))
    pc = p.to("cpu")
    ys = OM.moe_block_fp32(x.cpu()[sub], pc, ids_c[sub], w32[sub])
    oc = out.cpu()[sub]
    assert OM.rel_err(oc, ys) <= TOL
    for e in hot:
        m = (ids_c[sub] == int(e)).any(dim=1)
        assert OM.rel_err(oc[m], ys[m]) <= TOL, (int(e), int(counts[e]))
    return counts


@pytest.mark.parametrize("T", [256, 8192])
def test_c3_moe_full_size(cuda, T):
    p, x = _moe_inputs(cuda, T)
    out, logits, ids, _ = ops.moe_forward(x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up,
                                          p.sh_down, p.sh_gate_w, 10, return_routing=True,
                                          ws_tag="cfg_moe")
    torch.cuda.synchronize()
    _status_ok(cuda, "cfg_moe")
    counts = _check_moe_full(cuda, T, p, x, out, logits, ids)
    if T == 8192:
        # the Zipf load gives the hottest experts thousands of rows (tens of token tiles)
        assert counts.max() >= 2048 and (counts > 0).sum() == 512


# ------------------------------------------------------------------------------ attention
def _seq_rows(b, seq):
    cu = b.cu_seqlens_q.tolist()
    return cu[seq], cu[seq + 1]


def _pages_cpu(b, seq, k_cache, v_cache):
    """One sequence's K and V rows [ctx, Hkv, D], gathered on the device, moved to the CPU."""
    c = b.ctx_list[seq]
    nblk = (c + 255) // 256
    pages = b.block_tables[seq, :nblk].long()
    k = k_cache[pages].reshape(-1, k_cache.shape[2], k_cache.shape[3])[:c]
    v = v_cache[pages].reshape(-1, v_cache.shape[2], v_cache.shape[3])[:c]
    return k.cpu(), v.cpu()


def _sample_rows(b, seqs_pf, n_pf_rows, n_dec, seed):
    """(sequence, [token rows]) samples: n_pf_rows per prefill sequence spread over the
    chunk (first and last row of every 128-row query tile region included) and n_dec
    decode sequences including the longest and the shortest."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for s in seqs_pf:
        a, e = _seq_rows(b, s)
        L = e - a
        base = {0, L - 1, min(127, L - 1), min(128, L - 1), L // 2}
        rnd = torch.randperm(L, generator=g)[:n_pf_rows].tolist()
        out.append((s, sorted(base.union(rnd))))
    dec = [i for i, q in enumerate(b.qlen_list) if q == 1]
    if dec:
        ctx = [b.ctx_list[i] for i in dec]
        pick = {dec[int(np.argmax(ctx))], dec[int(np.argmin(ctx))]}
        for i in torch.randperm(len(dec), generator=g).tolist():
            if len(pick) >= n_dec:
                break
            pick.add(dec[i])
        out += [(s, [0]) for s in sorted(pick)]
    return out


def _check_attention_sample(b, q, gate, k_cache, v_cache, out, attn, w_o, samples):
    """CPU oracle on sampled rows: attention (attention_rows_fp32) and gate + o_proj."""
    w_o_c = w_o.cpu()
    got_o, got_y, ref_o, ref_y = [], [], [], []
    for s, rows in samples:
        a, e = _seq_rows(b, s)
        L, c = e - a, b.ctx_list[s]
        k, v = _pages_cpu(b, s, k_cache, v_cache)
        tok = torch.tensor([a + r for r in rows])
        pos = torch.tensor([c - L + r for r in rows])
        o = OA.attention_rows_fp32(q[tok.to(q.device)].cpu(), pos, k, v, b.scale)
        R = len(rows)
        gt = gate[tok.to(gate.device)].cpu().reshape(R, -1)
        ref_o.append(o.reshape(R, -1))
        ref_y.append(OA.gate_oproj_fp32(o.reshape(R, -1), gt, w_o_c))
        got_o.append(attn[tok.to(attn.device)].cpu())
        got_y.append(out[tok.to(out.device)].cpu())
    eo = OM.rel_err(torch.cat(got_o), torch.cat(ref_o))
    ey = OM.rel_err(torch.cat(got_y), torch.cat(ref_y))
    assert eo <= TOL and ey <= TOL, (eo, ey)


def _check_attention_every_row(b, q, gate, k_cache, v_cache, out, attn, w_o):
    """The fp32 oracle over every row of the batch, evaluated on the GPU."""
    o32 = OA.paged_attention(q, k_cache, v_cache, b.block_tables, b.context_lens,
                             b.cu_seqlens_q, b.scale)
    N = q.shape[0]
    y32 = OA.gate_oproj_fp32(o32.reshape(N, -1), gate.reshape(N, -1), w_o)
    eo = OM.rel_err(attn, o32.reshape(N, -1))
    ey = OM.rel_err(out, y32)
    assert eo <= TOL and ey <= TOL, (eo, ey)
    assert bool(torch.isfinite(out.float()).all())


def test_c2_pod_full_size(cuda):
    b = W.c2_batch(seed=1, device=cuda)
    N, Hq, D = b.q.shape
    attn = torch.empty(N, Hq * D, dtype=torch.bfloat16, device=cuda)
    out = ops.pod_attn_oproj(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                             b.cu_seqlens_q, b.w_o, b.scale, attn_out=attn,
                             max_q_len=max(b.qlen_list), ws_tag="cfg_pod",
                             work_hint=ops.pod_work_hint(b.ctx_list, b.qlen_list))
    torch.cuda.synchronize()
    _status_ok(cuda, "cfg_pod")
    _check_attention_every_row(b, b.q, b.gate, b.k_cache, b.v_cache, out, attn, b.w_o)
    samples = _sample_rows(b, [0], 256, 32, seed=2)
    _check_attention_sample(b, b.q, b.gate, b.k_cache, b.v_cache, out, attn, b.w_o, samples)


@pytest.mark.parametrize("mode", ["gemm", "kernel", "pod"])
def test_c4_step_full_size(cuda, mode):
    """The C4 step as bench.py runs it: the gated attention layer from hidden states
    (merged q/k/v GEMM, prologue with the K/V store, POD attention, gate, o_proj) over
    512 decode sequences and a 4096-token chunk, then the MoE at T = 4608; with the
    prologue in the projection GEMM's epilogue (bench.py's form), as its own launch and
    fused into the attention kernel."""
    b = W.c4_attn_batch(seed=1, device=cuda)
    N, Hq, D = b.q.shape
    Hkv = b.k_cache.shape[2]
    lp = W.make_attn_layer_params(seed=0, device=cuda)
    pos, slots = W.layer_positions_slots(b)
    x_attn = W.make_layer_input(N, 2048, seed=7, device=cuda)
    qkv = torch.empty(N, lp.w_qkv.shape[0], dtype=torch.bfloat16, device=cuda)
    qbuf = torch.empty(N, Hq, D, dtype=torch.bfloat16, device=cuda)
    attn = torch.empty(N, Hq * D, dtype=torch.bfloat16, device=cuda)
    # slots of the new tokens before the layer overwrites them (the store must touch
    # exactly these rows)
    kc_flat = b.k_cache.view(-1, Hkv, D)
    out = ops.gated_attention_layer(
        x_attn, lp.w_qkv, Hq, Hkv, lp.q_norm_w, lp.k_norm_w, lp.cos_sin_cache, lp.eps,
        pos.to(cuda), slots.to(cuda), b.k_cache, b.v_cache, b.block_tables, b.context_lens,
        b.cu_seqlens_q, b.w_o, b.scale, max_q_len=max(b.qlen_list),
        work_hint=ops.pod_work_hint(b.ctx_list, b.qlen_list), qkv=qkv, q=qbuf,
        attn_out=attn, ws_tag="cfg_c4", prologue=mode)
    torch.cuda.synchronize()
    _status_ok(cuda, "cfg_c4")
    _status_ok(cuda, "cfg_c4_prologue")
    # 1. merged projection GEMM, every row, against fp32 torch on the GPU (with the
    #    prologue in the GEMM's epilogue only the gate columns reach qkv; the projection
    #    the epilogue normalised is the plain GEMM's, same tiles and accumulation order)
    ref_qkv = x_attn.float() @ lp.w_qkv.float().t()
    if mode == "gemm":
        gate_of = lambda t: t[:, :Hq * 2 * D].reshape(N, Hq, 2, D)[:, :, 1]
        assert OM.rel_err(gate_of(qkv), gate_of(ref_qkv)) <= 1e-2
        proj = ops.gemm(x_attn, lp.w_qkv)
        assert OM.rel_err(proj, ref_qkv) <= 1e-2
        assert torch.equal(gate_of(proj), gate_of(qkv))
    else:
        assert OM.rel_err(qkv, ref_qkv) <= 1e-2
        proj = qkv
    # 2. prologue on a sample of tokens (chunk rows and decode tokens), from the kernel's
    #    own projection output: query rows and the K/V rows stored at the tokens' slots
    g = torch.Generator().manual_seed(11)
    sub = torch.cat([torch.tensor([0, 1, 4095, 4096, N - 1]),
                     torch.randperm(N, generator=g)[:384]]).unique()
    qkv_s = proj[sub.to(cuda)].cpu()
    q_in = qkv_s[:, :Hq * 2 * D]
    k_raw = qkv_s[:, Hq * 2 * D:Hq * 2 * D + Hkv * D]
    v_raw = qkv_s[:, Hq * 2 * D + Hkv * D:]
    rq, _, rk, rv = OA.attn_prologue(
        q_in, k_raw, v_raw, lp.q_norm_w.cpu(), lp.k_norm_w.cpu(),
        lp.cos_sin_cache.cpu().view(-1, 1, lp.cos_sin_cache.shape[1]), pos[sub], lp.eps, Hq, D)
    _bf16_within_ulp(qbuf[sub.to(cuda)], rq)
    st = slots[sub].long().to(cuda)
    _bf16_within_ulp(kc_flat[st], rk)
    assert torch.equal(b.v_cache.view(-1, Hkv, D)[st].cpu(), rv)
    # 3. attention + gate + o_proj from the kernel's query and cache, every row on the
    #    GPU, then sampled rows on the CPU
    gate = qkv[:, :Hq * 2 * D].view(N, Hq, 2 * D)[..., D:]
    _check_attention_every_row(b, qbuf, gate, b.k_cache, b.v_cache, out, attn, b.w_o)
    samples = _sample_rows(b, [0], 256, 32, seed=3)
    _check_attention_sample(b, qbuf, gate, b.k_cache, b.v_cache, out, attn, b.w_o, samples)
    del ref_qkv, x_attn, qkv, proj
    if mode != "gemm":
        return
    # 4. the MoE layer on the step's 4608 tokens
    p, x = _moe_inputs(cuda, N)
    mo, logits, ids, _ = ops.moe_forward(x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up,
                                         p.sh_down, p.sh_gate_w, 10, return_routing=True,
                                         ws_tag="cfg_moe")
    torch.cuda.synchronize()
    _status_ok(cuda, "cfg_moe")
    counts = _check_moe_full(cuda, N, p, x, mo, logits, ids)
    assert (counts > 0).sum() >= 500
