"""GPU parity of the MoE path (router top-k, permutation, grouped GEMMs, combine).

Bars: routing and permutation bit-exact against the oracle given the same bf16 logits;
block output within max|y - y32| / max|y32| <= 2e-2 of the fp32 oracle evaluated with the
same routing.  All calls go through the C ABI (``layerbatch_b200.ops``).
"""
import numpy as np
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from oracle import moe as OM
from tests.golden.make_golden import MOE_CASES

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (130, 512, 2048), (64, 2048, 4096),
                                   (300, 96, 128), (1000, 256, 512)])
def test_gemm_bf16(cuda, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    c = ops.gemm(a, b)
    torch.cuda.synchronize()
    assert OM.rel_err(c, ref) < 1e-2
    c32 = ops.gemm(a, b, accumulate_fp32=True, splits=2 if (K // 64) % 2 == 0 else 1)
    assert OM.rel_err(c32, ref) < 1e-4


@pytest.mark.parametrize("case", ["moe_c0", "moe_e512_t32", "router_ties"])
def test_router_topk_bit_exact(cuda, golden, case):
    g = golden[case]
    logits = g["logits"]
    k = g["k"] if case == "router_ties" else MOE_CASES[case][5]
    w_ref, ids_ref = OM.topk_route(logits, k)
    ids, wf, wb = ops.router_topk(logits.to(cuda), k)
    torch.cuda.synchronize()
    assert torch.equal(ids.cpu().long(), ids_ref), "top-k ids differ from the oracle"
    assert torch.allclose(wf.cpu(), w_ref, rtol=2e-6, atol=0)
    ulp = (wb.cpu().float() - w_ref.to(torch.bfloat16).float()).abs()
    assert float(ulp.max()) <= float(w_ref.abs().max()) * 2 ** -7
    # the reference's own torch.topk picks the same sets up to ties
    assert bool(OM.same_up_to_ties(ids.cpu(), g["topk_ids"], logits).all())


@pytest.mark.parametrize("T,k,E,base,nl", [(300, 10, 64, 0, 64), (37, 8, 512, 0, 512),
                                           (200, 4, 64, 16, 16), (1, 1, 32, 0, 32)])
def test_permute_bit_exact(cuda, T, k, E, base, nl):
    gen = torch.Generator().manual_seed(T * 31 + k)
    ids = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)]).to(torch.int32)
    row_start, perm_token, row_of = ops.moe_permute(ids.to(cuda), base, nl)
    torch.cuda.synchronize()
    loc = ids.numpy().astype(np.int64) - base
    loc[(loc < 0) | (loc >= nl)] = -1
    counts, offsets, ptok, pslot, rof = OM.permutation(loc, nl)
    rs = row_start.cpu().numpy()
    assert rs[0] == 0 and rs[1] == T
    assert np.array_equal(rs[1:] - T, offsets)
    P = int(offsets[-1])
    pt = perm_token.cpu().numpy()
    assert np.array_equal(pt[:T], np.arange(T))
    assert np.array_equal(pt[T:T + P], ptok)
    ro = row_of.cpu().numpy()
    exp = np.where(rof >= 0, rof + T, -1)
    assert np.array_equal(ro, exp)
    # determinism: a second run is bitwise identical
    r2 = ops.moe_permute(ids.to(cuda), base, nl)
    assert all(torch.equal(a, b) for a, b in zip((row_start, perm_token, row_of), r2))


def _run_block(cuda, T, H, E, I, k, zipf=False, seed=0):
    p = W.make_moe_params(H, E, I, I, k, seed=seed)
    x = W.make_moe_input(T, H, seed=seed + 1)
    if zipf:
        W.apply_zipf_bias(p, x)
    pd = p.to(cuda)
    out, logits, ids, wb = ops.moe_forward(x.to(cuda), pd.router, pd.gate_up, pd.down,
                                           pd.sh_gate, pd.sh_up, pd.sh_down, pd.sh_gate_w, k,
                                           return_routing=True)
    torch.cuda.synchronize()
    ws = ops.workspace(0, cuda, "moe")
    assert ops.device_status(ws) == 0
    return p, x, out.cpu(), logits.cpu(), ids.cpu().long(), wb.cpu()


@pytest.mark.parametrize("T,H,E,I,k,zipf", [(64, 2048, 64, 512, 8, False),
                                             (32, 2048, 512, 512, 10, True),
                                             (1, 256, 32, 128, 4, False),
                                             (300, 256, 32, 128, 4, False),
                                             (1000, 2048, 64, 512, 8, False)])
def test_moe_block(cuda, T, H, E, I, k, zipf):
    p, x, out, logits, ids, wb = _run_block(cuda, T, H, E, I, k, zipf)
    ref_logits = OM.router_logits(x, p.router)
    # fp32 accumulation order differs from the CPU's, so a logit may round to the
    # neighbouring bf16 value (one ulp <= |v| * 2^-7); most are identical.
    d = (logits.float() - ref_logits.float()).abs()
    ulp = torch.maximum(ref_logits.float().abs(), logits.float().abs()) * 2 ** -7
    assert bool((d <= ulp + 1e-6).all()), "router logits differ by more than one bf16 ulp"
    assert float((d == 0).float().mean()) > 0.9
    # routing is bit-exact given the kernel's own logits
    w32, ids_ref = OM.topk_route(logits, k)
    assert torch.equal(ids, ids_ref)
    y32 = OM.moe_block_fp32(x, p, ids, w32)
    err = OM.rel_err(out, y32)
    assert err <= TOL, err
    assert torch.isfinite(out.float()).all()


def test_grouped_gemm_token_tile_edges(cuda):
    """Experts whose row counts sit on both sides of the MMA widths and token tiles of the
    grouped GEMMs (N = rows rounded up to 16, 128-row token tiles, 32-row boxes), with the
    shared expert as a multi-tile group and two feature blocks in both GEMMs."""
    counts = [0, 1, 15, 16, 17, 31, 32, 33, 127, 128, 129, 255, 256, 257, 300, 5]
    E, H, I, k = len(counts), 512, 256, 1
    T = sum(counts)
    g = torch.Generator().manual_seed(7)
    ids = torch.cat([torch.full((c,), e, dtype=torch.int64) for e, c in enumerate(counts)])
    ids = ids[torch.randperm(T, generator=g)].view(T, k)
    w = torch.rand(T, k, generator=g) + 0.25
    p = W.make_moe_params(H, E, I, I, 4, seed=11)
    x = W.make_moe_input(T, H, seed=12)
    pd = p.to(cuda)
    out = ops.moe_forward(x.to(cuda), None, pd.gate_up, pd.down, pd.sh_gate, pd.sh_up,
                          pd.sh_down, pd.sh_gate_w, k, topk_ids=ids.to(cuda).int(),
                          topk_weights=w.to(cuda), num_experts=E, ws_tag="moe_edges")
    torch.cuda.synchronize()
    assert ops.device_status(ops.workspace(0, cuda, "moe_edges")) == 0
    y32 = OM.moe_block_fp32(x, p, ids, w)
    err = OM.rel_err(out.cpu(), y32)
    assert err <= TOL, err
    # every expert's rows, empty and one-row experts included, carry their own output
    for e, c in enumerate(counts):
        if c:
            tok = (ids[:, 0] == e).nonzero().flatten()
            assert OM.rel_err(out.cpu()[tok], y32[tok]) <= TOL, (e, c)


def test_moe_block_vs_reference_golden(cuda, golden):
    """Against the reference's own bf16 output where routing agrees."""
    g = golden["moe_c0"]
    T, H, E, I, Is, k, _ = g["shape"]
    p, x, out, logits, ids, wb = _run_block(cuda, T, H, E, I, k)
    same = OM.same_up_to_ties(ids, g["topk_ids"], g["logits"])
    assert float(same.float().mean()) >= 0.95
    assert OM.rel_err(out[same], g["y_sparse"][same]) <= TOL


def test_expert_parallel_building_blocks_emulated(cuda):
    """Routing given / no shared expert / rows added from elsewhere: splitting the experts
    over P virtual ranks in one process reproduces the single-call block bit for bit in
    routing and within tolerance in value."""
    T, H, E, I, k, P = 200, 2048, 64, 512, 8, 4
    p = W.make_moe_params(H, E, I, I, k, seed=3)
    x = W.make_moe_input(T, H, seed=4)
    pd, xd = p.to(cuda), x.to(cuda)
    ref, logits, ids, _ = ops.moe_forward(xd, pd.router, pd.gate_up, pd.down, pd.sh_gate,
                                          pd.sh_up, pd.sh_down, pd.sh_gate_w, k,
                                          return_routing=True)
    _, wf, _ = ops.router_topk(logits, k)
    nl = E // P
    dest = ids.long() // nl
    order = torch.argsort(dest.reshape(-1), stable=True)
    counts = torch.bincount(dest.reshape(-1), minlength=P).tolist()
    flat_ids, flat_w = ids.reshape(-1)[order], wf.reshape(-1)[order]
    rows_x = xd[(order // k)]
    y_parts, s0 = [], 0
    for r in range(P):
        n = counts[r]
        if n == 0:
            continue
        y_parts.append(ops.moe_forward(
            rows_x[s0:s0 + n].contiguous(), None, pd.gate_up[r * nl:(r + 1) * nl],
            pd.down[r * nl:(r + 1) * nl], None, None, None, None, 1, expert_base=r * nl,
            topk_ids=flat_ids[s0:s0 + n].view(n, 1), topk_weights=flat_w[s0:s0 + n].view(n, 1),
            num_experts=E, ws_tag=f"ep{r}"))
        s0 += n
    y_send = torch.cat(y_parts, 0)
    pair_pos = torch.empty(T * k, dtype=torch.int32, device=cuda)
    pair_pos[order] = torch.arange(T * k, dtype=torch.int32, device=cuda)
    out = ops.moe_forward(xd, None, None, None, pd.sh_gate, pd.sh_up, pd.sh_down, pd.sh_gate_w,
                          k, topk_ids=ids, topk_weights=wf, num_experts=E,
                          pair_rows=y_send, pair_index=pair_pos.view(T, k), ws_tag="ep_src")
    torch.cuda.synchronize()
    y32 = OM.moe_block_fp32(x, p, ids.cpu().long(), wf.cpu())
    assert OM.rel_err(out.cpu(), y32) <= TOL
    assert OM.rel_err(out.cpu(), ref.cpu()) <= TOL
