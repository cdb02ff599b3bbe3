"""The library inside CUDA graphs on an external stream (the reference replays its layers
as CUDA graphs on Green-Context external streams, nanovllm/engine/layer_batch.py:103-226
and model_runner.py:1045-1130).

Every entry point is stream-ordered with no host synchronisation, so a whole step (the
fused attention layer and the MoE block) is captured once on a stream that torch only
wraps (``torch.cuda.ExternalStream``) and replayed with new inputs copied into the
captured buffers; the replays must match eager calls on the same inputs.
"""
import pytest
import torch

from layerbatch_b200 import ops
from layerbatch_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def test_step_captured_in_cuda_graph_on_external_stream(cuda):
    b = W.make_attn_batch([700, 33, 1900, 256], [(128, 300)], seed=31).to(cuda)
    mq = max(b.qlen_list)
    p = W.make_moe_params(2048, 64, 512, 512, 8, seed=2).to(cuda)
    x = W.make_moe_input(b.num_tokens, 2048, seed=3).to(cuda)

    def step(out_a, out_m):
        ops.pod_attn_oproj(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                           b.cu_seqlens_q, b.w_o, b.scale, out=out_a, max_q_len=mq,
                           ws_tag="graph_pod")
        ops.moe_forward(x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up, p.sh_down,
                        p.sh_gate_w, 8, out=out_m, ws_tag="graph_moe")

    raw = torch.cuda.Stream()
    ext = torch.cuda.ExternalStream(raw.cuda_stream)
    out_a = torch.empty(b.num_tokens, 2048, dtype=torch.bfloat16, device=cuda)
    out_m = torch.empty_like(x)
    with torch.cuda.stream(ext):
        step(out_a, out_m)                     # sizes the workspaces before capture
    torch.cuda.synchronize()
    ref_a, ref_m = out_a.clone(), out_m.clone()

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ext):
        step(out_a, out_m)
    for it in range(3):
        if it:
            # new inputs in the captured buffers: the replay must follow them
            b.q.copy_(torch.randn_like(b.q.float()).to(torch.bfloat16))
            x.copy_(torch.randn_like(x.float()).to(torch.bfloat16))
            with torch.cuda.stream(ext):
                ea = torch.empty_like(out_a)
                em = torch.empty_like(out_m)
                step(ea, em)
            torch.cuda.synchronize()
            ref_a, ref_m = ea.clone(), em.clone()
        out_a.zero_()
        out_m.zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(ext):
            g.replay()
        torch.cuda.synchronize()
        # both layers are deterministic (fixed reduction orders, no atomics on values),
        # so a replay reproduces the eager call bit for bit
        assert torch.equal(out_a, ref_a), it
        assert torch.equal(out_m, ref_m), it
    del g
