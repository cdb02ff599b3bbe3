#!/usr/bin/env python
"""Benchmark of the LayerBatch hot path on B200: the gated full-attention layer (merged
q/k/v projection, (1+w) RMSNorm + partial RoPE prologue with the K/V store, POD paged
attention over prefill + decode, sigmoid gate, o_proj) followed by the Qwen3.5 MoE layer.

Default workload (``--config c4``): 512 decode sequences with contexts ~U[1024,16384] plus
one 4096-token prefill chunk through the attention layer (Hq=16, Hkv=2, D=256, H=2048,
256-token pages, shuffled block tables, RoPE theta 1e7 on 64 dims), then the MoE layer
(E=512 top-10, I=512, one shared expert, Zipf(1.1) routing skew) on the step's 4608 tokens.
One step = both layers on one batch, from hidden states to layer outputs.  Inputs exceed
L2 (the KV cache and expert weights are gigabytes), so no L2 flush is needed between steps.
The other configs are the attention + o_proj call alone (c1, c2) and the MoE layer alone
(c3s, c3l).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c2|c3s|c3l|c4]
    python bench.py --impl reference ...   # the reference's CPU path (restated) only

Under torchrun (``--gpus N``, N even) the c4 step is sharded: ranks form tensor-parallel
pairs that split the attention by KV head (each rank projects, normalises and attends its
own heads; the o_proj GEMM stores its fp32 partial tiles into the owning rank's memory
over NVLink and the owners reduce and send back the bf16 rows), the pairs run different
batches (data parallel), and the 512 experts are split over all N ranks with the NVLink
peer-memory dispatch and return of lb_ep_moe_forward.  No NCCL collective is on the data
path.  Each GPU keeps one c4 batch of work, so scaling is weak.  Rank 0 prints one JSON
line; the time is the max over ranks of CUDA-event time.

``value`` is device throughput with inputs resident in HBM, timed over K steps with no
events inside them (on one GPU the step is captured once as a CUDA graph and replayed, so
short steps are not bounded by the host's launch rate); a second pass over K eager steps
records CUDA events between the stages for the per-phase times and the roofline kernel's
duration.  ``e2e`` is the same step through
the same public calls in a serving loop: each step uploads its inputs (hidden states and
batch metadata) from pinned host memory and downloads its outputs, on copy streams that
overlap the previous and next steps' kernels (double-buffered device inputs and outputs).
After the timed loops every workspace's device status word must be 0 and every output
finite, else the run fails.

The reference arm (``--impl reference``) and ``cpu_baseline`` time the reference's CPU code
for the same step (restated in ``oracle/``: torch linears, the prologue, paged SDPA for
decode and prefill, gate + o_proj, the sparse MoE path) on FULL steps of the workload, all
host threads; the reference arm bounds its run by ``--ref-budget-s`` seconds and reports
the steps it timed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return dict(PEAKS_FALLBACK, source="fallback")


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the dominant
# kernel on the single-GPU workload, from one ncu capture of the current kernel
# (summaries under profiles/); re-captured whenever the kernel changes.  k_pod_attn for
# the attention workloads, the grouped gate/up GEMM (k_gemm_tok, SwiGLU) for c3.
NCU_GATE_UP_TRAFFIC = {"c3s": 1556182016 + 6260480, "c3l": 2548653056 + 86476800}
NCU_POD_TRAFFIC = {"c1": 293298688 + 4990976, "c2": 1225966080 + 24515328,
                   "c4": 9144729344 + 47202048}

# ---------------------------------------------------------------------------- workloads
CONFIGS = {
    "c1": "c1: 64 decode seqs ctx~U[512,4096] -> gated paged attention + o_proj 4096->2048",
    "c2": "c2: 2048-token prefill chunk on a 2048 prefix + 128 decode seqs ctx~U[256,8192] "
          "-> POD attention + gate + o_proj",
    "c3s": "c3: MoE E=512 top-10 I=512 +shared, H=2048, T=256 (decode batch), Zipf(1.1)",
    "c3l": "c3: MoE E=512 top-10 I=512 +shared, H=2048, T=8192 (prefill batch), Zipf(1.1)",
    "c4": "c4: 512 decode seqs ctx~U[1024,16384] + 4096-token prefill chunk -> gated "
          "full-attention layer from hidden states (q/k/v proj, q/k (1+w) RMSNorm, RoPE "
          "theta 1e7 on 64 dims, K/V store, POD attention, sigmoid gate, o_proj; "
          "Hq16/Hkv2/D256/H2048), then MoE E=512 top-10 I=512 +shared at T=4608, Zipf(1.1)",
}
LAYER_CONFIGS = ("c4",)      # configs that run the whole attention layer from hidden states
MOE_TOKENS = {"c3s": 256, "c3l": 8192}


def config_dict(cfg, tokens_per_gpu):
    """The ``config`` object of the JSON line; identical on both arms."""
    return {"workload": CONFIGS[cfg], "tokens_per_step_per_gpu": tokens_per_gpu,
            "l2": "inputs larger than L2 (KV cache and expert weights are GBs)"}


def tokens_per_step(cfg):
    return {"c1": 64, "c2": 2048 + 128, "c3s": 256, "c3l": 8192, "c4": 4096 + 512}[cfg]


def attn_batch_for(cfg, seed, device, **kw):
    from layerbatch_b200 import workloads as W
    if cfg == "c1":
        return W.c1_batch(seed=seed, device=device, **kw)
    if cfg == "c2":
        return W.c2_batch(seed=seed, device=device, **kw)
    if cfg == "c4":
        return W.c4_attn_batch(seed=seed, device=device, **kw)
    return None


def attn_work(b, fused_prologue=False):
    """Algorithmic FLOPs and bytes of the attention kernel for one batch: every KV byte of
    every context read once, the query and gate rows read once, the gated row written.
    With the prologue fused into the kernel it also reads the new tokens' raw key and
    value rows once and stores them into the cache once (the normalised query it writes
    and reads back is scratch)."""
    Hq, D = b.q.shape[1], b.q.shape[2]
    Hkv = b.k_cache.shape[2]
    kv_tokens = sum(b.ctx_list)
    pairs = 0
    for c, L in zip(b.ctx_list, b.qlen_list):
        # query i of the chunk sees c - L + i + 1 keys
        pairs += L * (c - L) + L * (L + 1) // 2
    flops = 4.0 * pairs * Hq * D
    bytes_ = kv_tokens * Hkv * D * 2 * 2 + 3 * b.num_tokens * Hq * D * 2
    if fused_prologue:
        bytes_ += 4 * b.num_tokens * Hkv * D * 2
    return flops, bytes_


def moe_work(T, hit, H=2048, I=512, k=10, E=512):
    """Algorithmic bytes and FLOPs of the MoE layer and of its two grouped expert GEMMs.

    Bytes: every weight the routing needs read once (the hit experts', the shared
    expert's; for the layer also the router's and the shared gate's), the T input rows
    read once and the T output rows written once.  The rows passed between the layer's
    kernels (gathered inputs, SwiGLU activations, weighted expert rows) are scratch and
    not counted.  FLOPs: 2 per multiply-add of every routed pair and shared row."""
    rows = T * k + T
    x_b = out_b = T * H * 2
    gate_up = {"bytes": (hit + 1) * 2 * I * H * 2 + x_b, "flops": 2.0 * rows * H * 2 * I}
    down = {"bytes": (hit + 1) * H * I * 2 + out_b, "flops": 2.0 * rows * I * H}
    layer = {"bytes": E * H * 2 + gate_up["bytes"] + down["bytes"] + H * 2,
             "flops": 2.0 * T * H * E + gate_up["flops"] + down["flops"] + 2.0 * T * H}
    return gate_up, down, layer


def layer_proj_work(N, H=2048, Hq=16, Hkv=2, D=256):
    """Algorithmic bytes / FLOPs of the projection GEMM and the prologue for N tokens."""
    cols = Hq * 2 * D + 2 * Hkv * D
    gemm = {"bytes": cols * H * 2 + N * H * 2 + N * cols * 2, "flops": 2.0 * N * H * cols}
    # prologue: query + key + value rows read once; query written, K/V stored once
    pro = {"bytes": 2 * N * (Hq + 2 * Hkv) * D * 2, "flops": 0.0}
    return gemm, pro


def step_floor(attn, T_moe, moe_hit, Hq, Hkv, peaks, H=2048):
    """The c4 layer step's floor per stage (seconds): the slower of its algorithmic bytes
    over the measured HBM bandwidth and its FLOPs over the measured bf16 peak (attention
    and the MoE layer are byte-bound, the projections FLOP-bound)."""
    bw, pf = peaks["hbm_gbs"] * 1e9, peaks["bf16_tflops"] * 1e12
    fa, ba = attn_work(attn)
    g, _ = layer_proj_work(attn.num_tokens, H=H, Hq=Hq, Hkv=Hkv)
    n_t, kd = attn.num_tokens, Hq * attn.q.shape[2]
    o_fl = 2.0 * n_t * kd * H
    o_by = kd * H * 2 + n_t * kd * 2 + n_t * H * 2
    _, _, ly = moe_work(T_moe, moe_hit, H=H)
    return {"attention": max(ba / bw, fa / pf),
            "qkv_projection": max(g["bytes"] / bw, g["flops"] / pf),
            "o_proj": max(o_by / bw, o_fl / pf),
            "moe_layer": max(ly["bytes"] / bw, ly["flops"] / pf)}


# ---------------------------------------------------------------------------- clocks
def nvml_handle(device_index: int):
    """NVML handle of a CUDA device, matched by PCI bus id (CUDA and NVML may order
    devices differently)."""
    import pynvml
    pynvml.nvmlInit()
    pr = torch.cuda.get_device_properties(device_index)
    bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
    try:
        return pynvml.nvmlDeviceGetHandleByPciBusId_v2(bus)
    except Exception:
        return pynvml.nvmlDeviceGetHandleByIndex(device_index)


def bind_to_gpu_cpus(device_index: int) -> list:
    """Pin this process to the host cores NVML reports as close to the GPU (its NUMA
    node), so pinned host buffers and the copy threads live next to the GPU's PCIe link.
    Process-local; changes no GPU setting.  Returns the cores (empty if unknown)."""
    try:
        import pynvml
        h = nvml_handle(device_index)
        n = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
        cpus = [64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1]
        cpus = [c for c in cpus if c < n]
        if cpus:
            os.sched_setaffinity(0, cpus)
        return cpus
    except Exception:
        return []


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running (read-only)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index, period=0.005):
        self.index, self.period = index, period
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = nvml_handle(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self.ok = False
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        rs = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": rs, "samples": len(self.samples)}


# ---------------------------------------------------------------------------- CPU side
_CPU_INPUTS: dict = {}


def cpu_inputs(cfg):
    """The workload's full inputs on the host, built once per process.  Same shapes and
    distributions as the GPU arm (K/V pages tiled from a seeded N(0,1) block of 512 pages:
    the values do not change the CPU's work)."""
    if cfg in _CPU_INPUTS:
        return _CPU_INPUTS[cfg]
    from layerbatch_b200 import workloads as W
    d = {}
    if cfg in ("c1", "c2", "c4"):
        b = attn_batch_for(cfg, 1, "cpu", tile_pages=512)
        d["attn"] = b
        if cfg in LAYER_CONFIGS:
            d["lp"] = W.make_attn_layer_params(seed=0)
            d["pos"], d["slots"] = W.layer_positions_slots(b)
            d["x_attn"] = W.make_layer_input(b.num_tokens, 2048, seed=7)
    if cfg in ("c3s", "c3l", "c4"):
        T = MOE_TOKENS.get(cfg) or d["attn"].num_tokens
        p = W.make_moe_params(2048, 512, 512, 512, 10, seed=0)
        x = W.make_moe_input(T, 2048, seed=1)
        W.apply_zipf_bias(p, x)
        d["moe"] = (p, x)
    _CPU_INPUTS[cfg] = d
    return d


def cpu_reference_step(cfg):
    """One full step of ``cfg`` through the reference's CPU code (restated in oracle/):
    the attention layer's linears, prologue and K/V store (qwen3_5.py:705-736,
    attention.py:50-80), paged SDPA for the decode sequences and the prefill chunk
    (sdpa_fallback.py:61-159), ``o * sigmoid(gate)`` and o_proj (qwen3_5.py:742-746), and
    the MoE block's sparse path (qwen3_5.py:815-905).  Returns seconds."""
    import torch.nn.functional as F
    from oracle import attention as OA
    from oracle import moe as OM
    d = cpu_inputs(cfg)
    t0 = time.perf_counter()
    with torch.no_grad():
        b = d.get("attn")
        if b is not None:
            N, Hq, D = b.q.shape
            if "lp" in d:
                lp = d["lp"]
                x = d["x_attn"]
                qd = Hq * 2 * D
                kd = b.k_cache.shape[2] * D
                q_out = F.linear(x, lp.w_qkv[:qd])
                k_raw = F.linear(x, lp.w_qkv[qd:qd + kd])
                v_raw = F.linear(x, lp.w_qkv[qd + kd:])
                q, gate, k, v = OA.attn_prologue(
                    q_out, k_raw, v_raw, lp.q_norm_w, lp.k_norm_w,
                    lp.cos_sin_cache.view(-1, 1, lp.cos_sin_cache.shape[1]), d["pos"], lp.eps,
                    Hq, D)
                OA.store_kvcache(k, v, b.k_cache, b.v_cache, d["slots"])
            else:
                q, gate = b.q, b.gate.reshape(N, -1)
            npf = b.num_prefill
            parts = []
            if npf:
                e = int(b.cu_seqlens_q[npf])
                o = OA.paged_prefill_bf16(q[:e], b.k_cache, b.v_cache, b.block_tables[:npf],
                                          b.context_lens[:npf], b.cu_seqlens_q[:npf + 1],
                                          b.scale)
                parts.append(o.reshape(e, -1))
            if b.num_seqs > npf:
                e = int(b.cu_seqlens_q[npf])
                o = OA.paged_decode_bf16(q[e:], b.k_cache, b.v_cache, b.block_tables[npf:],
                                         b.context_lens[npf:], b.scale)
                parts.append(o.reshape(N - e, -1))
            OA.gate_oproj_bf16(torch.cat(parts, 0), gate.reshape(N, -1), b.w_o)
        if "moe" in d:
            p, x = d["moe"]
            OM.moe_block_bf16(x, p, "sparse")
    return time.perf_counter() - t0


def cpu_reference_run(cfg, warmup, steps, budget_s):
    """Warm-up then timed FULL steps until ``steps`` or the time budget; returns
    (tokens/s of the median step, steps timed, warm-ups run, cores, description)."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    t_start = time.perf_counter()
    cpu_inputs(cfg)
    t_setup = time.perf_counter() - t_start
    n_w = 0
    for _ in range(max(1, min(warmup, 1))):
        cpu_reference_step(cfg)
        n_w += 1
    times = []
    while len(times) < max(1, steps):
        times.append(cpu_reference_step(cfg))
        if time.perf_counter() - t_start + times[-1] > budget_s:
            break
    med = statistics.median(times)
    desc = (f"full {cfg} step (every token and sequence of the workload), median of "
            f"{len(times)} timed step(s) after {n_w} warm-up; {cores} threads; "
            f"input setup {t_setup:.0f} s untimed")
    return tokens_per_step(cfg) / med, len(times), n_w, cores, desc


# ---------------------------------------------------------------------------- GPU side
def _time_cuda(fn, warmup=3, iters=10):
    """Median of ``iters`` CUDA-event timings (ms) of ``fn`` on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return statistics.median(ts)


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def gpu_library_baselines(device):
    """GPU implementations of the c4 step's two halves other than this library's, timed
    on the same inputs: flashinfer's paged prefill/decode attention (then the gate and
    o_proj as torch ops), vLLM's fused-MoE Triton kernels for the routed experts (router,
    top-k and shared expert as torch ops), and the reference's own algorithm as plain
    torch on the GPU (the expert loop of its sparse path).  Each is checked against this
    library's output.  Libraries that are missing or fail to build report why."""
    import torch.nn.functional as F
    from layerbatch_b200 import ops
    from layerbatch_b200 import workloads as W
    out = {}
    b = W.c4_attn_batch(seed=1, device=device)
    N, Hq, D = b.q.shape
    Hkv = b.k_cache.shape[2]
    hint = ops.pod_work_hint(b.ctx_list, b.qlen_list)
    o_ours = torch.empty(N, 2048, dtype=torch.bfloat16, device=device)
    att = {"workload": "c4 attention + gate + o_proj (given q, gate; 512 decode + 4096 chunk)"}
    att["ours_ms"] = _time_cuda(lambda: ops.pod_attn_oproj(
        b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.context_lens, b.cu_seqlens_q,
        b.w_o, b.scale, out=o_ours, max_q_len=max(b.qlen_list), work_hint=hint, ws_tag="gb"))
    try:
        import flashinfer
        ps = b.k_cache.shape[1]
        lens = b.context_lens.long().cpu()
        npg = (lens + ps - 1) // ps
        kv_indptr = torch.zeros(len(lens) + 1, dtype=torch.int32)
        kv_indptr[1:] = torch.cumsum(npg, 0).to(torch.int32)
        bt = b.block_tables.cpu()
        kv_idx = torch.cat([bt[i, :int(npg[i])] for i in range(len(lens))]).to(torch.int32)
        last = (lens - (npg - 1) * ps).to(torch.int32)
        wsb = torch.empty(512 << 20, dtype=torch.uint8, device=device)
        o_fi = torch.empty(N, Hq, D, dtype=torch.bfloat16, device=device)
        att["flashinfer"] = flashinfer.__version__
        for backend in ("auto", "fa2", "trtllm-gen", "cudnn"):
            try:
                w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(wsb, kv_layout="NHD",
                                                                   backend=backend)
                extra = {}
                qo = b.cu_seqlens_q.to(device)
                if backend == "cudnn":   # element offsets, lengths and tables
                    qo = (b.cu_seqlens_q.long() * Hq * D).to(device)
                    qlens = (b.cu_seqlens_q[1:] - b.cu_seqlens_q[:-1]).to(device)
                    extra = dict(seq_lens=b.context_lens.to(device), seq_lens_q=qlens,
                                 block_tables=b.block_tables.to(device),
                                 max_token_per_sequence=max(b.qlen_list),
                                 max_sequence_kv=max(b.ctx_list))
                w.plan(qo, kv_indptr.to(device), kv_idx.to(device),
                       last.to(device), Hq, Hkv, D, ps, causal=True,
                       q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
                       sm_scale=b.scale, **extra)

                def fi_attn():
                    w.run(b.q, (b.k_cache, b.v_cache), out=o_fi)

                def fi_layer():
                    fi_attn()
                    og = (o_fi.float() * torch.sigmoid(b.gate.float())).to(torch.bfloat16)
                    return F.linear(og.reshape(N, Hq * D), b.w_o)

                att[f"flashinfer_{backend}"] = {
                    "attention_ms": _time_cuda(fi_attn),
                    "plus_torch_gate_oproj_ms": _time_cuda(fi_layer),
                    "rel_err_vs_ours": _rel_err(fi_layer(), o_ours)}
            except Exception as e:
                att[f"flashinfer_{backend}"] = f"unavailable: {type(e).__name__}: {str(e)[:160]}"
    except Exception as e:  # a missing or failing library is reported, not fatal
        att["flashinfer"] = f"unavailable: {type(e).__name__}: {str(e)[:200]}"
    out["attention"] = att
    del b
    torch.cuda.empty_cache()

    T, k = 4608, 10
    p = W.make_moe_params(2048, 512, 512, 512, k, seed=0, device=device)
    x = W.make_moe_input(T, 2048, seed=1, device=device)
    W.apply_zipf_bias(p, x)
    moe = {"workload": "c4 MoE layer, T=4608, E=512 top-10, I=512, shared expert, Zipf(1.1)"}
    m_ours = torch.empty_like(x)
    moe["ours_ms"] = _time_cuda(lambda: ops.moe_forward(
        x, p.router, p.gate_up, p.down, p.sh_gate, p.sh_up, p.sh_down, p.sh_gate_w, k,
        out=m_ours, ws_tag="gb_moe"))

    def routing():
        logits = F.linear(x, p.router)
        probs = torch.softmax(logits.float(), dim=-1)
        wts, ids = torch.topk(probs, k, dim=-1)
        return wts / wts.sum(-1, keepdim=True), ids

    def shared():
        h = F.silu(F.linear(x, p.sh_gate)) * F.linear(x, p.sh_up)
        return F.linear(h, p.sh_down) * torch.sigmoid(F.linear(x, p.sh_gate_w))

    try:
        from vllm.model_executor.layers.fused_moe.fused_moe import fused_experts

        def vllm_moe():
            wts, ids = routing()
            return fused_experts(x, p.gate_up, p.down, wts, ids.to(torch.int32)) + shared()

        moe["vllm_fused_experts_plus_torch_ms"] = _time_cuda(vllm_moe)
        moe["rel_err_vllm_vs_ours"] = _rel_err(vllm_moe(), m_ours)
    except Exception as e:
        moe["vllm"] = f"unavailable: {type(e).__name__}: {str(e)[:200]}"

    def torch_loop():
        wts, ids = routing()
        y = torch.zeros_like(x)
        for e in torch.unique(ids).tolist():
            tok, slot = torch.nonzero(ids == e, as_tuple=True)
            g, u = F.linear(x[tok], p.gate_up[e]).chunk(2, dim=-1)
            r = F.linear(F.silu(g) * u, p.down[e]) * wts[tok, slot, None].to(x.dtype)
            y.index_add_(0, tok, r)
        return y + shared()

    moe["torch_expert_loop_ms"] = _time_cuda(torch_loop, warmup=1, iters=3)
    moe["rel_err_torch_vs_ours"] = _rel_err(torch_loop(), m_ours)
    out["moe"] = moe
    return out


def run_ours(args, rank, world, device):
    from layerbatch_b200 import ops
    from layerbatch_b200 import workloads as W
    cfg = args.config
    seed = 1 + rank
    sharded = world > 1 and cfg == "c4"
    layer = cfg in LAYER_CONFIGS
    tp = 2 if (sharded and world % 2 == 0) else 1
    tp_group, ep_block = None, None
    lp = None
    if sharded:
        # TP pairs by KV head, data parallel across pairs, experts split over all ranks.
        # Per-GPU work stays that of one c4 batch: a TP pair runs tp batches.
        from layerbatch_b200.layers.fused_moe import Qwen3_5SparseMoeBlock
        groups = [torch.distributed.new_group(list(range(g * tp, (g + 1) * tp)))
                  for g in range(world // tp)] if tp > 1 else []
        gid = rank // tp
        tp_group = groups[gid] if tp > 1 else None
        dec = W.uniform_ctx(512 * tp, 1024, 16384, seed=100 + gid)
        attn = W.make_attn_batch(dec, [(0, 4096)] * tp, Hq=16 // tp, Hkv=2 // tp, H=2048,
                                 seed=1000 + rank, device=device)
        attn.scale = 256 ** -0.5
        lp = W.make_attn_layer_params(Hq=16 // tp, Hkv=2 // tp, seed=2000 + rank,
                                      device=device)
        x_attn = W.make_layer_input(attn.num_tokens, 2048, seed=3000 + gid, device=device)
    else:
        attn = attn_batch_for(cfg, seed, device)
        if layer:
            lp = W.make_attn_layer_params(seed=0, device=device)
            x_attn = W.make_layer_input(attn.num_tokens, 2048, seed=7, device=device)
    if layer:
        pos, slots = W.layer_positions_slots(attn)
        pos, slots = pos.to(device), slots.to(device)
        Hq_l, Hkv_l = attn.q.shape[1], attn.k_cache.shape[2]
        qkv_buf = torch.empty(attn.num_tokens, lp.w_qkv.shape[0], dtype=torch.bfloat16,
                              device=device)
        q_buf = torch.empty_like(attn.q)
    T_moe = 4608 if sharded else (MOE_TOKENS.get(cfg) or (attn.num_tokens if cfg == "c4" else 0))
    moe = None
    moe_hit = None
    if T_moe:
        p = W.make_moe_params(2048, 512, 512, 512, 10, seed=0, device=device)
        x = W.make_moe_input(T_moe, 2048, seed=seed, device=device)
        W.apply_zipf_bias(p, x)
        moe = (p, x)
        if not sharded:
            # experts the step's routing hits (the weights the grouped GEMMs must read)
            with torch.no_grad():
                ids_w, _, _ = ops.router_topk(ops.gemm(x, p.router), 10)
                moe_hit = int(torch.unique(ids_w).numel())
                del ids_w
        else:
            # Experts are placed by popularity (heaviest first to the least-loaded rank),
            # from the routing counts of a separate calibration batch of the same
            # distribution summed over the ranks, so every rank computes the same placement.
            from layerbatch_b200.engine.ep import placement_by_load
            with torch.no_grad():
                xc = W.make_moe_input(T_moe, 2048, seed=5000 + rank, device=device)
                xc[:, 0] = x[:, 0]          # the Zipf bias column of the benchmark inputs
                ids_c, _, _ = ops.router_topk(ops.gemm(xc, p.router), 10)
                loads = torch.bincount(ids_c.reshape(-1).long(), minlength=512).float()
                torch.distributed.all_reduce(loads)
                del xc
            placement = placement_by_load(loads, world)
            ep_block = Qwen3_5SparseMoeBlock(2048, 512, 10, 512, 512, ep_rank=rank,
                                             ep_size=world).to(torch.bfloat16).to(device)
            with torch.no_grad():
                ep_block.gate.weight.copy_(p.router)
                ep_block.load_expert_shard(p.gate_up, p.down, placement=placement)
                ep_block.shared_expert.gate_proj.weight.copy_(p.sh_gate)
                ep_block.shared_expert.up_proj.weight.copy_(p.sh_up)
                ep_block.shared_expert.down_proj.weight.copy_(p.sh_down)
                ep_block.shared_expert_gate.weight.copy_(p.sh_gate_w)
            del p
            moe = (None, x)
            torch.cuda.empty_cache()
            from layerbatch_b200.engine.ep import EPExchange
            ep_block.attach_exchange(EPExchange(T_moe, 2048, 10, device=device))
    tp_ex = None
    if sharded and tp > 1:
        from layerbatch_b200.engine.peer import TPExchange
        tp_ex = TPExchange(attn.num_tokens, 2048, group=tp_group, device=device)
    tokens = (attn.num_tokens // tp) if attn is not None else T_moe
    max_q = max(attn.qlen_list) if attn is not None else 0
    hint = ops.pod_work_hint(attn.ctx_list, attn.qlen_list) if attn is not None else None
    pod_tag = "pod" if not sharded else f"tp_attn{rank}"

    a_out = torch.empty(attn.num_tokens, attn.w_o.shape[0], dtype=torch.bfloat16,
                        device=device) if attn is not None else None
    m_out = torch.empty_like(moe[1]) if moe else None

    def step(ev=None, inp=None, out_a=None, out_m=None):
        """One step.  ``ev``: dict of event lists for the phase pass; ``inp``: device input
        buffers of the e2e loop (else the resident inputs)."""
        ev = ev or {}
        inp = inp or {}
        if attn is not None:
            bt, cl, cu = inp.get("meta") or (attn.block_tables, attn.context_lens,
                                              attn.cu_seqlens_q)
            oa = out_a if out_a is not None else a_out
            if layer:
                if "attn0" in ev:
                    ev["attn0"].record()
                ops.gated_attention_layer(
                    inp.get("x_attn", x_attn), lp.w_qkv, Hq_l, Hkv_l, lp.q_norm_w,
                    lp.k_norm_w, lp.cos_sin_cache, lp.eps, inp.get("pos", pos),
                    inp.get("slots", slots), attn.k_cache, attn.v_cache, bt, cl, cu, attn.w_o,
                    attn.scale, out=oa, max_q_len=max_q, work_hint=hint, events=ev.get("pod"),
                    qkv=qkv_buf, q=q_buf, ws_tag=pod_tag, tp=tp_ex,
                    stage_events=ev.get("stages"), prologue=args.prologue)
            else:
                if "attn0" in ev:
                    ev["attn0"].record()
                ops.pod_attn_oproj(inp.get("q", attn.q), inp.get("gate", attn.gate),
                                   attn.k_cache, attn.v_cache, bt, cl, cu, attn.w_o,
                                   attn.scale, out=oa, max_q_len=max_q, events=ev.get("pod"),
                                   work_hint=hint)
            if "attn1" in ev:
                ev["attn1"].record()
        if moe:
            pm, xm = moe
            xx = inp.get("x_moe", xm)
            om = out_m if out_m is not None else m_out
            if "moe0" in ev:
                ev["moe0"].record()
            if sharded:
                from layerbatch_b200.engine.ep import ep_moe_forward_nvlink
                ep_moe_forward_nvlink(ep_block, xx, ep_block.ep_exchange, out=om,
                                      events=ev.get("moe"))
            else:
                ops.moe_forward(xx, pm.router, pm.gate_up, pm.down, pm.sh_gate, pm.sh_up,
                                pm.sh_down, pm.sh_gate_w, 10, out=om, events=ev.get("moe"))
            if "moe1" in ev:
                ev["moe1"].record()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def mk():
        return torch.cuda.Event(enable_timing=True)

    K, Wu = args.steps, args.warmup
    for _ in range(Wu):
        step()
    torch.cuda.synchronize()
    # On one GPU the step is captured once as a CUDA graph and the timed loop replays it,
    # as the reference replays its decode steps (nanovllm/engine/model_runner.py:862-891):
    # the device time is then not bounded by the host's launch rate (which matters for the
    # 0.1 ms steps of c1).  The library's launch counter sees the launches at capture.
    graph, per_step = None, None
    if world == 1 and not args.no_graph:
        n0 = ops.launch_count()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        per_step = ops.launch_count() - n0
        graph.replay()
        torch.cuda.synchronize()
    # ---------------- the timed region: K steps, no events inside them
    st, en = mk(), mk()
    n0 = ops.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        st.record()
        for _ in range(K):
            if graph is not None:
                graph.replay()
            else:
                step()
        en.record()
        torch.cuda.synchronize()
    barrier()
    launches = per_step * K if graph is not None else ops.launch_count() - n0
    ms = st.elapsed_time(en) / K
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms = float(ms_t)

    # ---------------- phase pass: K more steps with events between the stages
    evs = []
    for _ in range(K):
        e = {"attn0": mk(), "attn1": mk(), "moe0": mk(), "moe1": mk(),
             "pod": [mk() for _ in range(4)], "moe": [mk() for _ in range(4)],
             "stages": [mk(), mk()]}
        evs.append(e)
    for i in range(K):
        step(ev=evs[i] if attn is not None or moe else None)
    torch.cuda.synchronize()

    def mean_ms(a, b):
        return statistics.mean(a(e).elapsed_time(b(e)) for e in evs)

    res = {"ms": ms, "tokens": tokens, "launches": launches, "launches_per_step": launches / K,
           "clocks": clk.summary(),
           "timed_loop": "CUDA graph replay of the captured step" if graph is not None
           else "eager launches"}
    del graph
    peaks = load_peaks()
    phases = {}
    if attn is not None:
        t_attn = mean_ms(lambda e: e["pod"][0], lambda e: e["pod"][1]) * 1e-3
        flops, byts = attn_work(attn)
        res["attn"] = {"ms": t_attn * 1e3, "flops": flops, "bytes": byts,
                       "gbs": byts / t_attn / 1e9, "tflops": flops / t_attn / 1e12}
        if layer and args.prologue == "gemm":
            phases["qkv_gemm_prologue"] = mean_ms(lambda e: e["attn0"], lambda e: e["stages"][1])
            phases["plan"] = mean_ms(lambda e: e["stages"][1], lambda e: e["pod"][0])
        elif layer:
            phases["qkv_gemm"] = mean_ms(lambda e: e["attn0"], lambda e: e["stages"][0])
            phases["prologue"] = mean_ms(lambda e: e["stages"][0], lambda e: e["stages"][1])
            phases["plan"] = mean_ms(lambda e: e["stages"][1], lambda e: e["pod"][0])
        else:
            phases["plan"] = mean_ms(lambda e: e["attn0"], lambda e: e["pod"][0])
        phases["pod_attn"] = t_attn * 1e3
        # split merge + gate (k_pod_merge), then the o_proj GEMM (with tensor parallelism:
        # the GEMM storing fp32 tiles into the owners' memory, the owners' reduction and
        # the gather of the other ranks' rows)
        phases["merge"] = mean_ms(lambda e: e["pod"][1], lambda e: e["pod"][2])
        phases["oproj"] = mean_ms(lambda e: e["pod"][2], lambda e: e["pod"][3])
        phases["attention_layer"] = mean_ms(lambda e: e["attn0"], lambda e: e["attn1"])
        if layer and args.prologue == "gemm":
            g, pr = layer_proj_work(attn.num_tokens, Hq=Hq_l, Hkv=Hkv_l)
            res["proj"] = {"gemm_tflops": g["flops"] / phases["qkv_gemm_prologue"] / 1e9,
                           "prologue": "in the q/k/v GEMM's epilogue (lb_qkv_prologue_gemm)"}
        elif layer:
            g, pr = layer_proj_work(attn.num_tokens, Hq=Hq_l, Hkv=Hkv_l)
            res["proj"] = {"gemm_gbs": g["bytes"] / phases["qkv_gemm"] / 1e6,
                           "gemm_tflops": g["flops"] / phases["qkv_gemm"] / 1e9,
                           "prologue_gbs": pr["bytes"] / phases["prologue"] / 1e6}
    if moe:
        phases["moe_layer"] = mean_ms(lambda e: e["moe0"], lambda e: e["moe1"])
        if sharded:
            # expert parallel: router + top-k + routing table + row dispatch over NVLink;
            # the wait for every source's rows + permutation + gather; the grouped GEMMs;
            # the per-row sums sent back + the wait for them + the combine
            phases["moe_dispatch"] = mean_ms(lambda e: e["moe0"], lambda e: e["moe"][1])
            phases["moe_wait_permute"] = mean_ms(lambda e: e["moe"][1], lambda e: e["moe"][2])
            phases["moe_experts"] = mean_ms(lambda e: e["moe"][2], lambda e: e["moe"][3])
            phases["moe_return_combine"] = mean_ms(lambda e: e["moe"][3], lambda e: e["moe1"])
        else:
            t_g1 = mean_ms(lambda e: e["moe"][0], lambda e: e["moe"][1]) * 1e-3
            t_g2 = mean_ms(lambda e: e["moe"][2], lambda e: e["moe"][3]) * 1e-3
            phases["moe_gate_up"] = t_g1 * 1e3
            phases["moe_down"] = t_g2 * 1e3
            gu, dn, ly = moe_work(T_moe, moe_hit)
            t_l = phases["moe_layer"] * 1e-3
            res["moe_gate_up"] = dict(gu, ms=t_g1 * 1e3, gbs=gu["bytes"] / t_g1 / 1e9,
                                      tflops=gu["flops"] / t_g1 / 1e12)
            res["moe_layer"] = {"ms": t_l * 1e3, "experts_hit": moe_hit,
                                "algorithmic_bytes": ly["bytes"],
                                "algorithmic_flops": ly["flops"],
                                "gbs": ly["bytes"] / t_l / 1e9,
                                "frac": ly["bytes"] / t_l / 1e9 / peaks["hbm_gbs"],
                                "gate_up_frac": gu["bytes"] / t_g1 / 1e9 / peaks["hbm_gbs"],
                                "down_frac": dn["bytes"] / t_g2 / 1e9 / peaks["hbm_gbs"],
                                "bytes_counted": "weights hit + shared + router, x, out "
                                                 "(no scratch rows)"}
    res["phases_ms"] = {k: round(v, 4) for k, v in phases.items()}
    if layer and moe and not sharded:
        stages = step_floor(attn, T_moe, moe_hit, Hq_l, Hkv_l, peaks)
        floor = sum(stages.values())
        res["step_roofline"] = {"floor_ms": floor * 1e3, "frac": floor * 1e3 / res["ms"],
                                "stage_floor_ms": {k: round(v * 1e3, 4) for k, v in stages.items()},
                                "basis": "per stage max(algorithmic bytes / measured HBM GB/s, "
                                         "FLOPs / measured bf16 TFLOP/s), summed"}
    res["parallelism"] = (f"tp{tp} x dp{world // tp} attention (KV-head shards, o_proj GEMM "
                          f"reducing over NVLink peer memory), ep{world} MoE (NVLink "
                          f"peer-memory dispatch/return, experts placed by popularity)"
                          if sharded else
                          ("single GPU" if world == 1 else
                           f"dp{world}: per-rank batches, experts replicated"))
    res["peaks"] = peaks

    # ---------------- end-to-end through the public API with host buffers
    # A serving loop: every step copies its inputs from pinned host memory and reads its
    # outputs back.  The copies run on their own streams into double-buffered device
    # inputs/outputs, so step i+1's upload and step i-1's download overlap step i's
    # kernels; events order each buffer's reuse.  All copies are inside the timed region.
    if not args.no_e2e:
        pin = {}
        if attn is not None:
            if layer:
                pin["x_attn"] = x_attn.cpu().pin_memory()
                pin["pos"] = pos.cpu().pin_memory()
                pin["slots"] = slots.cpu().pin_memory()
            else:
                pin["q"] = attn.q.cpu().pin_memory()
                pin["gate"] = attn.gate.cpu().pin_memory()
            pin["meta"] = [t.cpu().pin_memory() for t in
                           (attn.block_tables, attn.context_lens, attn.cu_seqlens_q)]
        if moe:
            pin["x_moe"] = moe[1].cpu().pin_memory()
        bufs, host_out = [], []
        for _ in range(2):
            bd = {}
            for name, v in pin.items():
                bd[name] = ([torch.empty(t.shape, dtype=t.dtype, device=device) for t in v]
                            if isinstance(v, list) else
                            torch.empty(v.shape, dtype=v.dtype, device=device))
            if attn is not None:
                bd["out_a"] = torch.empty_like(a_out)
            if moe:
                bd["out_m"] = torch.empty_like(m_out)
            bufs.append(bd)
            host_out.append({k: torch.empty(bd[k].shape, dtype=bd[k].dtype).pin_memory()
                             for k in ("out_a", "out_m") if k in bd})
        h2d = d2h = 0
        for v in pin.values():
            h2d += sum(t.numel() * t.element_size() for t in (v if isinstance(v, list) else [v]))
        for v in host_out[0].values():
            d2h += v.numel() * v.element_size()
        comp = torch.cuda.current_stream()
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_used = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        # On one GPU the step on each buffer set is captured as a CUDA graph (as for the
        # device-time loop); the copies stay outside the graphs, on their own streams.
        e2e_graphs = None
        if world == 1 and not args.no_graph:
            e2e_graphs = []
            for bd in bufs:
                for name, v in pin.items():   # real inputs in the buffers before the capture
                    if isinstance(v, list):
                        for dst, src in zip(bd[name], v):
                            dst.copy_(src)
                    else:
                        bd[name].copy_(v)
                kw = dict(inp={n: bd[n] for n in pin}, out_a=bd.get("out_a"), out_m=bd.get("out_m"))
                step(**kw)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    step(**kw)
                e2e_graphs.append(g)
            torch.cuda.synchronize()

        def e2e_step(i):
            k = i % 2
            bd, ho = bufs[k], host_out[k]
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_used[k])          # step i-2 is done reading buffer k
                for name, v in pin.items():
                    if isinstance(v, list):
                        for dst, src in zip(bd[name], v):
                            dst.copy_(src, non_blocking=True)
                    else:
                        bd[name].copy_(v, non_blocking=True)
                ev_in[k].record(s_in)
            comp.wait_event(ev_in[k])
            comp.wait_event(ev_out[k])                # step i-2's outputs have been read
            if e2e_graphs is not None:
                e2e_graphs[k].replay()
            else:
                step(inp={n: bd[n] for n in pin}, out_a=bd.get("out_a"), out_m=bd.get("out_m"))
            ev_used[k].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[k])
                for name, h in ho.items():
                    h.copy_(bd[name], non_blocking=True)
                ev_out[k].record(s_out)

        for i in range(max(2, Wu)):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        Ke = max(4, K)
        s2, e2 = mk(), mk()
        s2.record(comp)
        s_in.wait_event(s2)
        for i in range(Ke):
            e2e_step(i)
        comp.wait_event(ev_out[0])
        comp.wait_event(ev_out[1])
        e2.record(comp)
        torch.cuda.synchronize()
        ms_e = s2.elapsed_time(e2) / Ke
        mt = torch.tensor([ms_e], dtype=torch.float64, device=device)
        if world > 1:
            torch.distributed.all_reduce(mt, op=torch.distributed.ReduceOp.MAX)
        res["e2e"] = {"ms": float(mt), "h2d": h2d, "d2h": d2h}
        del e2e_graphs
        for ho in host_out:
            for name, h in ho.items():
                if not bool(torch.isfinite(h.float()).all()):
                    res.setdefault("errors", []).append(f"e2e output {name} not finite")

    # ---------------- outside the timed regions: device status words and outputs
    status = 0
    for (dev_i, tag), ws in list(ops._WS.items()):
        if dev_i == torch.cuda.current_device():
            status |= ops.device_status(ws)
    for name, t in (("attention output", a_out), ("moe output", m_out)):
        if t is not None and not bool(torch.isfinite(t.float()).all()):
            res.setdefault("errors", []).append(f"{name} not finite")
    if status:
        res.setdefault("errors", []).append(f"device status word {status} (1 = a bounded "
                                            f"wait timed out, 2 = an index was out of range)")
    res["device_status"] = status
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=list(CONFIGS), default="c4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--prologue", choices=["gemm", "kernel", "pod"], default="gemm",
                    help="where the c4 layer's attention prologue runs: in the q/k/v GEMM's "
                         "epilogue (default), its own kernel, or inside the attention kernel")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager launches instead of replaying a captured step")
    ap.add_argument("--ref-budget-s", type=float, default=240.0,
                    help="wall-clock bound of the reference arm's CPU run")
    ap.add_argument("--gpu-baselines", action="store_true",
                    help="also time flashinfer / vLLM / plain-torch GPU versions of the c4 "
                         "attention and MoE on the same inputs (1 GPU, after the timed run)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg_desc = config_dict(args.config, tokens_per_step(args.config))

    if args.impl == "reference":
        # The reference path is CPU code: rank 0 alone times it on the host cores.
        if rank != 0:
            return
        v, n, n_w, cores, sample = cpu_reference_run(args.config, args.warmup, args.steps,
                                                     args.ref_budget_s)
        line = {"metric": "hot-path tokens/s", "value": v, "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": n, "warmup": n_w,
                "ms_per_step": tokens_per_step(args.config) / v * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded)", "config": cfg_desc,
                "impl": "reference", "parallelism": "host CPU",
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores,
                                 "kind": "port", "sample": sample},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        # the reference-arm CPU sample (rank 0, N=1 only) keeps every host core
        bind_to_gpu_cpus(local)
    res = run_ours(args, rank, world, device)
    errors = list(res.get("errors", []))
    if world > 1:
        bad = torch.tensor([len(errors)], dtype=torch.int32, device=device)
        torch.distributed.all_reduce(bad)
        if int(bad) and not errors:
            errors.append("another rank reported an error")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not errors:
        v, n, n_w, cores, sample = cpu_reference_run(args.config, 1, 1, 60.0)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        peaks = res["peaks"]
        value = res["tokens"] * world / (res["ms"] * 1e-3)
        roof = None
        if "attn" in res:
            a = res["attn"]
            t_hbm = a["bytes"] / (peaks["hbm_gbs"] * 1e9)
            t_tc = a["flops"] / (peaks["bf16_tflops"] * 1e12)
            if t_hbm >= t_tc:
                roof = {"bound": "hbm", "achieved": a["gbs"], "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": a["gbs"] / peaks["hbm_gbs"]}
            else:
                roof = {"bound": "tensor", "achieved": a["tflops"], "peak": peaks["bf16_tflops"],
                        "unit": "TFLOP/s", "frac": a["tflops"] / peaks["bf16_tflops"]}
            traffic = NCU_POD_TRAFFIC.get(args.config) if world == 1 else None
            roof.update({"kernel": "k_pod_attn", "traffic": traffic,
                         "peak_source": peaks["source"], "kernel_ms": a["ms"],
                         "algorithmic_bytes": a["bytes"], "algorithmic_flops": a["flops"]})
        elif "moe_gate_up" in res:
            # MoE-only workloads: the dominant kernel is the grouped gate/up GEMM
            g = res["moe_gate_up"]
            t_hbm = g["bytes"] / (peaks["hbm_gbs"] * 1e9)
            t_tc = g["flops"] / (peaks["bf16_tflops"] * 1e12)
            if t_hbm >= t_tc:
                roof = {"bound": "hbm", "achieved": g["gbs"], "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": g["gbs"] / peaks["hbm_gbs"]}
            else:
                roof = {"bound": "tensor", "achieved": g["tflops"], "peak": peaks["bf16_tflops"],
                        "unit": "TFLOP/s", "frac": g["tflops"] / peaks["bf16_tflops"]}
            roof.update({"kernel": "k_gemm_tok (gate/up, SwiGLU)",
                         "traffic": NCU_GATE_UP_TRAFFIC.get(args.config) if world == 1 else None,
                         "peak_source": peaks["source"], "kernel_ms": g["ms"],
                         "algorithmic_bytes": g["bytes"], "algorithmic_flops": g["flops"],
                         "tensor_frac": g["tflops"] / peaks["bf16_tflops"]})
        line = {
            "metric": "hot-path tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": cfg_desc, "parallelism": res["parallelism"],
            "roofline": roof, "cpu_baseline": cpu, "clocks": res["clocks"],
            "gpu_launches": res["launches"], "phases_ms": res["phases_ms"],
            "timed_loop": res["timed_loop"],
        }
        for key in ("moe_layer", "proj", "step_roofline"):
            if key in res:
                line[key] = res[key]
        if "e2e" in res:
            e = res["e2e"]
            line["e2e"] = {"value": res["tokens"] * world / (e["ms"] * 1e-3), "unit": "tokens/s",
                           "h2d_bytes_per_step": e["h2d"], "d2h_bytes_per_step": e["d2h"]}
        if args.gpu_baselines and world == 1:
            line["gpu_baselines"] = gpu_library_baselines(device)
        if errors:
            line["errors"] = errors
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    if errors:
        sys.exit(1)


if __name__ == "__main__":
    main()
