"""Expert-parallel MoE over peer memory (``lb_ep_moe_forward``), emulated on one GPU.

P ranks live in one process: each has its own exchange buffer, expert shard, tokens and
workspace, and every rank maps every buffer.  The three phases of a call are issued for
all ranks in order on one stream (all dispatches, then all expert phases, then all
combines), so each bounded wait finds its flags already set.  Each rank's output must
match the single-GPU block on its own tokens and the fp32 oracle; two consecutive calls
exercise the per-call epochs and buffer reuse.  The real multi-GPU run is in
``test_multigpu.py``.
"""
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W
from layerbatch_b200._lib import LB_EP_PHASE_COMBINE, LB_EP_PHASE_DISPATCH, LB_EP_PHASE_EXPERTS
from layerbatch_b200.engine.ep import EPExchange, ep_moe_forward_nvlink
from layerbatch_b200.layers.fused_moe import Qwen3_5SparseMoeBlock
from oracle import moe as OM

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def ep_blocks(pd, P, H, E, k, I, dev, placement=None):
    blks = []
    for r in range(P):
        b = Qwen3_5SparseMoeBlock(H, E, k, I, I, ep_rank=r, ep_size=P).to(torch.bfloat16).to(dev)
        with torch.no_grad():
            b.gate.weight.copy_(pd.router)
            b.load_expert_shard(pd.gate_up, pd.down, placement=placement)
            b.shared_expert.gate_proj.weight.copy_(pd.sh_gate)
            b.shared_expert.up_proj.weight.copy_(pd.sh_up)
            b.shared_expert.down_proj.weight.copy_(pd.sh_down)
            b.shared_expert_gate.weight.copy_(pd.sh_gate_w)
        blks.append(b)
    return blks


@pytest.mark.parametrize("P,E,k,Ts,C,placed", [(4, 64, 8, [200, 64, 0, 150], 256, False),
                                               (2, 512, 10, [96, 33], 128, False),
                                               (4, 64, 8, [120, 7, 250, 64], 256, True)])
def test_ep_nvlink_emulated_ranks(cuda, P, E, k, Ts, C, placed):
    H, I = 2048, 512
    p = W.make_moe_params(H, E, I, I, k, seed=7)
    pd = p.to(cuda)
    placement = None
    if placed:   # experts spread over the ranks by a seeded permutation
        placement = torch.randperm(E, generator=torch.Generator().manual_seed(3))
    blks = ep_blocks(pd, P, H, E, k, I, cuda, placement)
    exs = EPExchange.emulated(P, C, H, k, device=cuda)
    try:
        for call in range(2):
            xs = [W.make_moe_input(T, H, seed=100 * call + r).to(cuda) if T else
                  torch.empty(0, H, dtype=torch.bfloat16, device=cuda) for r, T in enumerate(Ts)]
            outs = [torch.empty_like(x) for x in xs]
            for ph in (LB_EP_PHASE_DISPATCH, LB_EP_PHASE_EXPERTS, LB_EP_PHASE_COMBINE):
                for r in range(P):
                    ep_moe_forward_nvlink(blks[r], xs[r], exs[r], out=outs[r], phases=ph,
                                          ws_tag=f"ep_emu{r}")
            torch.cuda.synchronize()
            for r in range(P):
                assert ops.device_status(ops._WS[(torch.cuda.current_device(), f"ep_emu{r}")]) == 0
                if Ts[r] == 0:
                    continue
                ref, logits, ids, _ = ops.moe_forward(
                    xs[r], pd.router, pd.gate_up, pd.down, pd.sh_gate, pd.sh_up, pd.sh_down,
                    pd.sh_gate_w, k, return_routing=True, ws_tag="ep_ref")
                _, wf, _ = ops.router_topk(logits, k)
                torch.cuda.synchronize()
                y32 = OM.moe_block_fp32(xs[r].cpu(), p, ids.cpu().long(), wf.cpu())
                assert OM.rel_err(outs[r].cpu(), y32) <= TOL, (call, r)
                assert OM.rel_err(outs[r].cpu(), ref.cpu()) <= TOL, (call, r)
    finally:
        exs[0].close()


def test_peer_wait_times_out_and_reports(cuda):
    """Failure detection without a fault: rank 0 of an emulated pair runs its phases but
    rank 1 never makes the call, so the flags rank 0 waits for are never set.  Each wait
    gives up after its time limit (~1 s), the kernels finish, the workspace status word
    reads LB_DEV_TIMEOUT on the host, and the context keeps working."""
    H, E, I, k, C = 2048, 64, 512, 8, 64
    p = W.make_moe_params(H, E, I, I, k, seed=8)
    pd = p.to(cuda)
    blks = ep_blocks(pd, 2, H, E, k, I, cuda)
    exs = EPExchange.emulated(2, C, H, k, device=cuda)
    try:
        x = W.make_moe_input(32, H, seed=9).to(cuda)
        ep_moe_forward_nvlink(blks[0], x, exs[0], ws_tag="ep_dead_peer")   # rank 1 absent
        torch.cuda.synchronize()
        ws = ops._WS[(torch.cuda.current_device(), "ep_dead_peer")]
        assert ops.device_status(ws) == 1          # LB_DEV_TIMEOUT
        # the device is still usable: a normal call runs and is correct
        y, logits, ids, _ = ops.moe_forward(x, pd.router, pd.gate_up, pd.down, pd.sh_gate,
                                            pd.sh_up, pd.sh_down, pd.sh_gate_w, k,
                                            return_routing=True, ws_tag="ep_after_timeout")
        _, wf, _ = ops.router_topk(logits, k)
        torch.cuda.synchronize()
        y32 = OM.moe_block_fp32(x.cpu(), p, ids.cpu().long(), wf.cpu())
        assert OM.rel_err(y.cpu(), y32) <= TOL
    finally:
        exs[0].close()
