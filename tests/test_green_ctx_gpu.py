"""The library on Green-Context streams in the Layer-Batch two-stream schedule.

The reference splits a decode batch into two nano-batches A and B and runs them through
the model's units (runs of layers of one kind) in a lag-by-one pipeline: at step t, unit
t of A and unit t-1 of B, each on the stream of its unit's kind, the two streams living in
SM-disjoint Green Contexts (nanovllm/utils/green_ctx.py:69-107 creates them;
nanovllm/engine/layer_batch.py:103-226 runs the schedule, also inside a CUDA graph whose
capture starts on one of the green streams, nanovllm/engine/model_runner.py:1045-1130).

Here two decoder layers' hot path form the units: the gated attention layer (q/k/v GEMM,
prologue with the K/V store, POD attention, gate, o_proj; on the first green stream) and
the MoE block (on the second), each followed by its residual add.  The two nano-batches use
separate workspaces, as they run at the same time.  The pipelined schedule, run eagerly on
the green streams and as a captured CUDA graph replayed twice, must reproduce bit for bit
the plain sequential run of both nano-batches on the default stream.
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


def _check(ret, name):
    err = ret[0]
    if int(err) != 0:
        raise RuntimeError(f"{name} failed: {err}")
    rest = ret[1:]
    return rest if len(rest) != 1 else rest[0]


class GreenStreams:
    """Two SM-disjoint Green Contexts of the current device with one stream each, wrapped
    as torch ExternalStreams (the construction of green_ctx.py:69-107: split the SM
    resource by count, a descriptor and a green context per part, a stream per context)."""

    def __init__(self, device_index: int, first_sms: int):
        from cuda.bindings import driver as drv
        self.drv = drv
        _check(drv.cuInit(0), "cuInit")
        dev = _check(drv.cuDeviceGet(device_index), "cuDeviceGet")
        total = _check(drv.cuDeviceGetDevResource(
            dev, drv.CUdevResourceType.CU_DEV_RESOURCE_TYPE_SM), "cuDeviceGetDevResource")
        self.total_sms = total.sm.smCount
        out = drv.cuDevSmResourceSplitByCount(1, total, 0, first_sms)
        if int(out[0]) != 0:
            raise RuntimeError(f"cuDevSmResourceSplitByCount: {out[0]}")
        groups, _, rest = out[1], out[2], out[3]
        parts = [groups[0], rest]
        self.sms = [p.sm.smCount for p in parts]
        flag = drv.CUgreenCtxCreate_flags.CU_GREEN_CTX_DEFAULT_STREAM.value
        sflag = drv.CUstream_flags.CU_STREAM_NON_BLOCKING.value
        self.ctxs, self.raw, self.streams = [], [], []
        for p in parts:
            desc = _check(drv.cuDevResourceGenerateDesc([p], 1), "cuDevResourceGenerateDesc")
            g = _check(drv.cuGreenCtxCreate(desc, dev, flag), "cuGreenCtxCreate")
            s = _check(drv.cuGreenCtxStreamCreate(g, sflag, 0), "cuGreenCtxStreamCreate")
            self.ctxs.append(g)
            self.raw.append(s)
            self.streams.append(torch.cuda.ExternalStream(int(s), device=device_index))

    def synchronize(self):
        """Wait for both green streams.  A green context is a context of its own, so
        ``torch.cuda.synchronize()`` (the primary context) does not wait for them."""
        for s in self.raw:
            _check(self.drv.cuStreamSynchronize(s), "cuStreamSynchronize")

    def close(self):
        self.synchronize()
        torch.cuda.synchronize()
        for s in self.raw:
            _check(self.drv.cuStreamDestroy(s), "cuStreamDestroy")
        for g in self.ctxs:
            _check(self.drv.cuGreenCtxDestroy(g), "cuGreenCtxDestroy")


def _same(got, ref, what):
    if torch.equal(got, ref):
        return
    d = (got.float() - ref.float()).abs()
    rows = (d > 0).any(dim=1).nonzero().flatten().tolist()
    raise AssertionError(f"{what}: {int((d > 0).sum())} elements differ (max {float(d.max()):.3g}) "
                         f"in rows {rows[:16]}")


def test_layer_batch_schedule_on_green_context_streams(cuda):
    try:
        from cuda.bindings import driver  # noqa: F401
    except Exception:
        pytest.skip("cuda-python driver bindings unavailable")
    H, E, I, k = 2048, 64, 512, 8
    ctx = W.uniform_ctx(64, 300, 3000, seed=21)
    b = W.make_attn_batch(ctx, (), seed=21, device=cuda)      # decode step, 64 sequences
    n_layers = 2
    caches = [(b.k_cache, b.v_cache)] + [
        (torch.randn_like(b.k_cache, dtype=torch.float32).to(torch.bfloat16),
         torch.randn_like(b.v_cache, dtype=torch.float32).to(torch.bfloat16))
        for _ in range(n_layers - 1)]
    lps = [W.make_attn_layer_params(seed=30 + l, device=cuda) for l in range(n_layers)]
    w_os = [b.w_o] + [W.make_attn_batch([1], (), seed=40 + l, device=cuda).w_o
                      for l in range(n_layers - 1)]
    moes = [W.make_moe_params(H, E, I, I, k, seed=50 + l, device=cuda) for l in range(n_layers)]
    pos, slots = W.layer_positions_slots(b)
    pos, slots = pos.to(cuda), slots.to(cuda)
    x = W.make_layer_input(b.num_seqs, H, seed=22, device=cuda)

    # nano-batches A = sequences [0, 24), B = [24, 64) with their own metadata and buffers
    B1 = 24
    groups = []
    for name, lo, hi in (("A", 0, B1), ("B", B1, b.num_seqs)):
        n = hi - lo
        groups.append(dict(
            name=name, lo=lo, hi=hi, n=n,
            bt=b.block_tables[lo:hi].contiguous(), cl=b.context_lens[lo:hi].contiguous(),
            cu=torch.arange(n + 1, dtype=torch.int32, device=cuda),
            pos=pos[lo:hi].contiguous(), slots=slots[lo:hi].contiguous(),
            h=torch.empty(n, H, dtype=torch.bfloat16, device=cuda),
            o=torch.empty(n, H, dtype=torch.bfloat16, device=cuda),
            qkv=torch.empty(n, lps[0].w_qkv.shape[0], dtype=torch.bfloat16, device=cuda),
            q=torch.empty(n, 16, 256, dtype=torch.bfloat16, device=cuda)))
    units = []
    for l in range(n_layers):
        units += [("FA", l), ("MOE", l)]

    def run_unit(g, unit):
        kind, l = unit
        if kind == "FA":
            lp = lps[l]
            kc, vc = caches[l]
            ops.gated_attention_layer(
                g["h"], lp.w_qkv, 16, 2, lp.q_norm_w, lp.k_norm_w, lp.cos_sin_cache, lp.eps,
                g["pos"], g["slots"], kc, vc, g["bt"], g["cl"], g["cu"], w_os[l], b.scale,
                out=g["o"], max_q_len=1, qkv=g["qkv"], q=g["q"], ws_tag="lb" + g["name"])
        else:
            p = moes[l]
            ops.moe_forward(g["h"], p.router, p.gate_up, p.down, p.sh_gate, p.sh_up,
                            p.sh_down, p.sh_gate_w, k, out=g["o"],
                            ws_tag="lb" + g["name"] + "_moe")
        g["h"].add_(g["o"])                      # residual

    def start(anchor):
        for g in groups:
            g["h"].copy_(x[g["lo"]:g["hi"]])

    # ---- reference: both nano-batches through every unit, one after the other
    start(None)
    for g in groups:
        for u in units:
            run_unit(g, u)
    torch.cuda.synchronize()
    ref = [g["h"].clone() for g in groups]
    for (tag,) in (("lbA",), ("lbB",), ("lbA_moe",), ("lbB_moe",), ("lbA_prologue",),
                   ("lbB_prologue",)):
        assert ops.device_status(ops.workspace(0, cuda, tag)) == 0, tag

    gs = GreenStreams(cuda.index if cuda.index is not None else 0,
                      first_sms=torch.cuda.get_device_properties(cuda).multi_processor_count // 2)
    fa_stream, la_stream = gs.streams
    assert sum(gs.sms) <= gs.total_sms and min(gs.sms) >= 8

    def layer_batch(anchor):
        """layer_batch.py:103-226: unit t of A and unit t-1 of B, each on its kind's
        stream; every cross-stream step waits for the nano-batch's previous stream."""
        start(anchor)
        last = {"A": anchor, "B": anchor}
        for s in (fa_stream, la_stream):
            if s is not anchor:
                s.wait_stream(anchor)
        for t in range(len(units) + 1):
            for g, u_idx in ((groups[0], t), (groups[1], t - 1)):
                if not 0 <= u_idx < len(units):
                    continue
                unit = units[u_idx]
                stream = fa_stream if unit[0] == "FA" else la_stream
                if stream is not last[g["name"]]:
                    stream.wait_stream(last[g["name"]])
                with torch.cuda.stream(stream):
                    run_unit(g, unit)
                last[g["name"]] = stream
        for s in set(last.values()):
            if s is not anchor:
                anchor.wait_stream(s)

    try:
        # eager, anchored on the default stream
        for g in groups:
            g["h"].zero_()
        layer_batch(torch.cuda.current_stream())
        gs.synchronize()
        torch.cuda.synchronize()
        for g, r in zip(groups, ref):
            _same(g["h"], r, "eager " + g["name"])
        # captured as one CUDA graph whose capture starts on the second green stream
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=la_stream):
            layer_batch(la_stream)
        for it in range(2):
            for g in groups:
                g["h"].zero_()
            torch.cuda.synchronize()
            with torch.cuda.stream(la_stream):
                graph.replay()
            gs.synchronize()
            torch.cuda.synchronize()
            for g, r in zip(groups, ref):
                _same(g["h"], r, f"replay {it} " + g["name"])
        del graph
        for tag in ("lbA", "lbB", "lbA_moe", "lbB_moe", "lbA_prologue", "lbB_prologue"):
            assert ops.device_status(ops.workspace(0, cuda, tag)) == 0, tag
    finally:
        gs.close()
