"""GPU test of ``lb_moe_permute_noalloc``, the permutation entry point that allocates nothing.

Some callers of this library cannot allocate device memory when they call it: a plugin
host whose enqueue hook forbids allocation, or a language binding with no device
allocator.  For them the entry point keeps its scratch in a fixed array in the library's
own static device memory instead of a caller-provided workspace; the caller still passes
the inputs and the output buffers.  This test calls it through the C ABI and checks that
it returns exactly what ``lb_moe_permute`` (the workspace version) returns, on calls in a
row with different sizes, so scratch left over from one call cannot go unnoticed; that
its result is the oracle's permutation (``oracle.moe.permutation``) at a prefill-sized
T = 8192, E = 512; the edges of its scratch layout (no tokens, 1024 local experts, a local
range that ends at the last expert); and that sizes beyond its limits are refused.

The file name makes pytest collect it last, so a run that stops at the first failure has
already run every other test.
"""
import numpy as np
import pytest
import torch

from layerbatch_b200 import _lib
from oracle import moe as OM

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return _lib.lib()


def _ids(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)


def _outputs(T, k, nl, dev):
    return (torch.full((nl + 2,), -7, dtype=torch.int32, device=dev),
            torch.full((T + T * k,), -1, dtype=torch.int32, device=dev),
            torch.full((T, k), -3, dtype=torch.int32, device=dev))


def _with_workspace(L, ids, T, k, base, nl):
    row_start, perm_token, row_of = _outputs(T, k, nl, ids.device)
    nbytes = L.lb_moe_permute_workspace_size(T, k, nl)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=ids.device)
    rc = L.lb_moe_permute(ids.data_ptr(), T, k, base, nl, row_start.data_ptr(),
                          perm_token.data_ptr(), row_of.data_ptr(), ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.lb_get_last_error_string()
    return row_start, perm_token, row_of


def _no_alloc(L, ids, T, k, base, nl):
    row_start, perm_token, row_of = _outputs(T, k, nl, ids.device)
    rc = L.lb_moe_permute_noalloc(ids.data_ptr(), T, k, base, nl, row_start.data_ptr(),
                                  perm_token.data_ptr(), row_of.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.lb_get_last_error_string()
    return row_start, perm_token, row_of


def test_no_alloc_permute_matches_workspace_version(L):
    dev = torch.device("cuda")
    # calls in a row: a large one, then smaller ones that would expose stale counts;
    # the scratch layout's edges: no tokens with the most local experts, 1024 local
    # experts over 513 tokens, a local range ending at the last expert
    for T, k, E, base, nl, seed in [(300, 10, 512, 0, 512, 1), (77, 4, 64, 16, 16, 2),
                                    (0, 2, 1024, 0, 1024, 4), (513, 8, 1024, 0, 1024, 5),
                                    (129, 6, 96, 64, 32, 6)]:
        ids = (_ids(T, k, E, seed) if T else torch.zeros(0, k, dtype=torch.int32)).to(dev)
        got = _no_alloc(L, ids, T, k, base, nl)
        ref = _with_workspace(L, ids, T, k, base, nl)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a.cpu(), b.cpu())
        G = nl + 1
        assert int(got[0][G].item()) == T + int(((ids >= base) & (ids < base + nl)).sum())


def test_no_alloc_permute_is_the_oracle_permutation_at_prefill_size(L):
    """T = 8192 tokens, top-10 of 512 experts (a c3 prefill batch), against the oracle;
    one call timed with CUDA events (every local expert scans all pairs)."""
    dev = torch.device("cuda")
    T, k, E = 8192, 10, 512
    g = torch.Generator().manual_seed(8)
    # a skewed load: low expert ids are picked far more often (ranks of a random score)
    score = torch.rand(T, E, generator=g) * torch.arange(1, E + 1).float().pow(-1.1)
    ids = torch.topk(score, k, dim=1).indices.to(torch.int32)
    idd = ids.to(dev)
    _no_alloc(L, idd, T, k, 0, E)          # warm-up
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    row_start, perm_token, row_of = _no_alloc(L, idd, T, k, 0, E)
    en.record()
    torch.cuda.synchronize()
    print(f"lb_moe_permute_noalloc T={T} k={k} E={E}: {st.elapsed_time(en):.3f} ms")
    counts, offsets, ptok, _, rof = OM.permutation(ids.numpy(), E)
    rs = row_start.cpu().numpy()
    assert rs[0] == 0 and rs[1] == T and np.array_equal(rs[1:E + 2] - T, offsets)
    pt = perm_token.cpu().numpy()
    assert np.array_equal(pt[:T], np.arange(T)) and np.array_equal(pt[T:], ptok)
    assert np.array_equal(row_of.cpu().numpy(), np.where(rof >= 0, rof + T, -1))
    assert counts.max() > 4 * counts.mean()
    ref = _with_workspace(L, idd, T, k, 0, E)
    torch.cuda.synchronize()
    for a, b in zip((row_start, perm_token, row_of), ref):
        assert torch.equal(a.cpu(), b.cpu())


def test_no_alloc_permute_rejects_sizes_beyond_its_scratch(L):
    dev = torch.device("cuda")
    T, k, nl = 8, 2, 1025
    ids = _ids(T, k, 2048, 3).to(dev)
    row_start, perm_token, row_of = _outputs(T, k, nl, dev)
    rc = L.lb_moe_permute_noalloc(ids.data_ptr(), T, k, 0, nl, row_start.data_ptr(),
                                  perm_token.data_ptr(), row_of.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 2  # LB_ERR_UNSUPPORTED
    assert b"1024" in L.lb_get_last_error_string()
    # more (token, slot) pairs than the cap; the sizes are refused before any pointer is
    # dereferenced, so small buffers suffice
    rc = L.lb_moe_permute_noalloc(ids.data_ptr(), (1 << 20) // 4 + 1, 4, 0, 64,
                                  row_start.data_ptr(), perm_token.data_ptr(),
                                  row_of.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert b"pairs" in L.lb_get_last_error_string()
