"""GPU parity of the CTA-pair dense GEMM (two CTAs of a cluster share one M = 256 MMA).

``lb_gemm_bf16`` and ``lb_qkv_prologue_gemm`` send a product to the pair kernel when its
256 x 256 tiles take fewer load-weighted waves than single-CTA tiles (the q/k/v projection
and o_proj shapes of a prefill-sized batch).  These cases take that path, including M not
a multiple of 256, where the second CTA of the last pair holds some or none of the valid
rows, and check the result against fp32 and that no row past M is written.
"""
import pytest
import torch

from layerbatch_b200 import ops
from oracle import moe as OM

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _takes_pair_path(M, N, sms):
    """The library's choice (pair_gemm_pays in lb_capi.cu) restated for the test."""
    if N % 256:
        return False
    mt = (M + 127) // 128

    def waves(tiles, slots):
        return (tiles + slots - 1) // slots

    def cost1(bn):
        return waves(mt * (N // bn), sms) * (128 + bn)

    bn = 256 if (M > 512 and cost1(256) <= cost1(128)) else 128
    pair = waves(((M + 255) // 256) * (N // 256), sms // 2) * 256
    return pair < cost1(bn)


@pytest.mark.parametrize("M,N,K", [(4608, 2048, 4096),   # o_proj of the c4 step
                                   (4608, 9216, 2048),   # q/k/v projection shape
                                   (4000, 2048, 1024),   # last pair: peer holds 32 rows
                                   (3900, 2048, 512)])   # last pair: peer holds none
def test_pair_gemm_matches_fp32(cuda, M, N, K):
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert _takes_pair_path(M, N, sms)
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    buf = torch.full((M + 64, N), 7.0, device=cuda, dtype=torch.bfloat16)
    c = ops.gemm(a, b, out=buf[:M])
    torch.cuda.synchronize()
    assert OM.rel_err(c, ref) < 1e-2
    assert bool((buf[M:] == 7.0).all()), "rows past M were written"
    # a second call into the same output is bitwise identical (deterministic tiles)
    c2 = ops.gemm(a, b)
    assert torch.equal(c2, buf[:M])
