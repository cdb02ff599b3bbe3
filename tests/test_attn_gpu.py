"""GPU parity of the POD attention + gated o_proj path against the CPU oracle.

Bar: ``max|y - y32| / max|y32| <= 2e-2`` for the o_proj output and the attention output,
against the fp32 oracle (``oracle.attention``) on the same seeded paged inputs; decode
cases are also checked against the reference's own bf16 output (golden vectors).
"""
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from oracle import attention as OA
from oracle import moe as OM
from tests.golden.make_golden import DECODE_CASES, PREFILL_CASES

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def run_pod(b, cuda, split_pages=0, with_attn=True):
    g = b.to(cuda)
    N, Hq, D = g.q.shape
    attn = torch.empty(N, Hq * D, dtype=torch.bfloat16, device=cuda) if with_attn else None
    out = ops.pod_attn_oproj(g.q, g.gate, g.k_cache, g.v_cache, g.block_tables, g.context_lens,
                             g.cu_seqlens_q, g.w_o, g.scale, attn_out=attn,
                             max_q_len=max(b.qlen_list), kv_split_pages=split_pages)
    torch.cuda.synchronize()
    ws = ops.workspace(0, cuda, "pod")
    assert ops.device_status(ws) == 0
    return out.cpu(), (attn.cpu() if attn is not None else None)


def check(b, out, attn):
    y32, o32 = OA.attn_oproj_fp32(b)
    N = b.num_tokens
    if attn is not None:
        e = OM.rel_err(attn, o32.reshape(N, -1))
        assert e <= TOL, f"attention rel err {e}"
    e = OM.rel_err(out, y32)
    assert e <= TOL, f"o_proj rel err {e}"
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("name", list(DECODE_CASES))
def test_decode_vs_reference(cuda, golden, name):
    b = W.make_attn_batch(DECODE_CASES[name], (), seed=3)
    out, attn = run_pod(b, cuda)
    check(b, out, attn)
    g = golden[name]
    assert OM.rel_err(attn, g["attn"].reshape(b.num_tokens, -1)) <= TOL
    assert OM.rel_err(out, g["y"]) <= TOL


@pytest.mark.parametrize("name", list(PREFILL_CASES))
def test_prefill_noprefix_vs_reference(cuda, golden, name):
    b = W.make_attn_batch([], PREFILL_CASES[name], seed=4)
    out, attn = run_pod(b, cuda)
    check(b, out, attn)
    assert OM.rel_err(attn, golden[name]["attn"].reshape(b.num_tokens, -1)) <= TOL


@pytest.mark.parametrize("decode,prefill,split", [
    ([], [(300, 200)], 0),
    ([], [(2048, 130)], 0),
    ([1000, 3000, 17, 256], [(500, 300)], 0),
    ([4096, 1, 2, 129], [], 1),
    ([5000, 333], [], 2),
    ([700] * 20, [(0, 1)], 0),
])
def test_mixed_batches(cuda, decode, prefill, split):
    b = W.make_attn_batch(decode, prefill, seed=11)
    out, attn = run_pod(b, cuda, split_pages=split)
    check(b, out, attn)


@pytest.mark.parametrize("Hq,Hkv", [(8, 1), (16, 1), (4, 2)])
def test_gqa_shapes(cuda, Hq, Hkv):
    b = W.make_attn_batch([900, 260, 31], [(100, 150)], Hq=Hq, Hkv=Hkv, seed=12)
    out, attn = run_pod(b, cuda)
    check(b, out, attn)


def test_stale_nan_cache_rows_are_ignored(cuda):
    """Slots past a sequence's end hold NaN: the result must not see them."""
    b = W.make_attn_batch([300, 129], [(40, 90)], seed=13, extra_blocks=1)
    for i, c in enumerate(b.ctx_list):
        nblk = (c + 255) // 256
        last = int(b.block_tables[i, nblk - 1])
        off = c - (nblk - 1) * 256
        b.k_cache[last, off:] = float("nan")
        b.v_cache[last, off:] = float("nan")
    out, attn = run_pod(b, cuda)
    check(b, out, attn)


def test_c1_full(cuda):
    b = W.c1_batch()
    out, attn = run_pod(b, cuda)
    check(b, out, attn)


def test_without_attn_out_and_repeat_is_deterministic(cuda):
    b = W.make_attn_batch([1500, 64], [(256, 256)], seed=14)
    o1, _ = run_pod(b, cuda, with_attn=False)
    o2, _ = run_pod(b, cuda, with_attn=False)
    assert torch.equal(o1, o2)
    y32, _ = OA.attn_oproj_fp32(b)
    assert OM.rel_err(o1, y32) <= TOL


def test_store_kvcache(cuda):
    N, Hkv, D = 37, 2, 256
    kc = torch.zeros(4, 256, Hkv, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    k = torch.randn(N, Hkv, D).to(torch.bfloat16)
    v = torch.randn(N, Hkv, D).to(torch.bfloat16)
    slots = torch.randperm(4 * 256)[:N].to(torch.int32)
    slots[5] = -1
    kc_ref, vc_ref = kc.clone(), vc.clone()
    OA.store_kvcache(k, v, kc_ref, vc_ref, slots)
    kg, vg = kc.to(cuda), vc.to(cuda)
    ops.store_kvcache(k.to(cuda), v.to(cuda), kg, vg, slots.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(kg.cpu(), kc_ref) and torch.equal(vg.cpu(), vc_ref)
