"""GPU test of ``lb_moe_permute_noalloc``, the permutation entry point that allocates nothing.

Some callers of this library cannot allocate device memory when they call it: a plugin
host whose enqueue hook forbids allocation, code that runs while a stream is captured into
a CUDA graph under a no-allocation policy, or a language binding with no device allocator.
For them the entry point keeps its scratch in a fixed array in the library's own static
device memory instead of a caller-provided workspace; the caller still passes the inputs
and the output buffers.  This test calls it through the C ABI and checks that it returns
exactly what ``lb_moe_permute`` (the workspace version) returns, on two calls in a row
with different sizes, so scratch left over from the first call cannot go unnoticed.

The file name makes pytest collect it last, so a run that stops at the first failure has
already run every other test.
"""
import ctypes as C

import pytest
import torch

from layerbatch_b200 import _lib

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
    # two calls in a row: a large one, then a smaller one that would expose stale counts
    for T, k, E, base, nl, seed in [(300, 10, 512, 0, 512, 1), (77, 4, 64, 16, 16, 2)]:
        ids = _ids(T, k, E, seed).to(dev)
        got = _no_alloc(L, ids, T, k, base, nl)
        ref = _with_workspace(L, ids, T, k, base, nl)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a.cpu(), b.cpu())
        G = nl + 1
        assert int(got[0][G].item()) == T + int(((ids >= base) & (ids < base + nl)).sum())


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
