#!/usr/bin/env python
"""Benchmark of the LayerBatch hot path on B200: gated full-attention layer (POD paged
attention over prefill + decode, sigmoid gate, o_proj) followed by the Qwen3.5 MoE layer.

Default workload (``--config c4``): 512 decode sequences with contexts ~U[1024,16384] plus
one 4096-token prefill chunk through the attention layer (Hq=16, Hkv=2, D=256, H=2048,
256-token pages, shuffled block tables), then the MoE layer (E=512 top-10, I=512, one
shared expert, Zipf(1.1) routing skew) on the step's 4608 tokens.  One step = both layers
on one batch.  Inputs exceed L2 (the KV cache and expert weights are gigabytes), so no L2
flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c2|c3s|c3l|c4]
    python bench.py --impl reference ...   # the reference's CPU path (restated) only

Under torchrun (``--gpus N``, N even) the c4 step is sharded: ranks form tensor-parallel
pairs that split the attention by KV head (the o_proj GEMM stores its fp32 partial tiles
into the owning rank's memory over NVLink and the owners reduce and send back the bf16
rows), the pairs run different batches (data parallel), and the 512 experts are split
over all N ranks with the NVLink peer-memory dispatch and return of lb_ep_moe_forward.
No NCCL collective is on the data path.  Each GPU keeps one c4 batch of work, so
scaling is weak.  Rank 0 prints one JSON line; the time is the max over ranks of
CUDA-event time.

``value`` is device throughput with inputs resident in HBM.  ``e2e`` is the same step
through the same public calls in a serving loop: each step uploads its inputs from
pinned host memory and downloads its outputs, on copy streams that overlap the previous
and next steps' kernels (double-buffered device inputs and outputs).
"""
from __future__ import annotations

import argparse
import json
import math
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
NCU_POD_TRAFFIC = {"c1": 293260800 + 5938432, "c2": 1220505088 + 22828800,
                   "c4": 9129531904 + 59853824}

# ---------------------------------------------------------------------------- workloads
CONFIGS = {
    "c1": "c1: 64 decode seqs ctx~U[512,4096] -> gated paged attention + o_proj 4096->2048",
    "c2": "c2: 2048-token prefill chunk on a 2048 prefix + 128 decode seqs ctx~U[256,8192] "
          "-> POD attention + gate + o_proj",
    "c3s": "c3: MoE E=512 top-10 I=512 +shared, H=2048, T=256 (decode batch), Zipf(1.1)",
    "c3l": "c3: MoE E=512 top-10 I=512 +shared, H=2048, T=8192 (prefill batch), Zipf(1.1)",
    "c4": "c4: 512 decode seqs ctx~U[1024,16384] + 4096-token prefill chunk -> gated attention"
          " + o_proj (Hq16/Hkv2/D256/H2048), then MoE E=512 top-10 I=512 +shared at T=4608, "
          "Zipf(1.1)",
}


def attn_batch_for(cfg, seed, device):
    from layerbatch_b200 import workloads as W
    if cfg == "c1":
        return W.c1_batch(seed=seed, device=device)
    if cfg == "c2":
        return W.c2_batch(seed=seed, device=device)
    if cfg == "c4":
        return W.c4_attn_batch(seed=seed, device=device)
    return None


def moe_tokens_for(cfg, attn):
    if cfg == "c3s":
        return 256
    if cfg == "c3l":
        return 8192
    if cfg == "c4":
        return attn.num_tokens
    return 0


def attn_work(b):
    """Algorithmic FLOPs and bytes of the attention kernel for one batch."""
    Hq, D = b.q.shape[1], b.q.shape[2]
    Hkv = b.k_cache.shape[2]
    kv_tokens = sum(b.ctx_list)
    pairs = 0
    for c, L in zip(b.ctx_list, b.qlen_list):
        # query i of the chunk sees c - L + i + 1 keys
        pairs += L * (c - L) + L * (L + 1) // 2
    flops = 4.0 * pairs * Hq * D
    bytes_ = kv_tokens * Hkv * D * 2 * 2 + 3 * b.num_tokens * Hq * D * 2
    return flops, bytes_


def moe_work(T, hit, H=2048, I=512, k=10):
    """Algorithmic bytes and FLOPs of the two grouped expert GEMMs for T tokens whose
    routing hits `hit` experts: each hit expert's weights once, the shared expert's once,
    every routed pair's and shared row's input read once and output written once."""
    rows = T * k + T
    gate_up = {"bytes": (hit + 1) * 2 * I * H * 2 + rows * H * 2 + rows * I * 2,
               "flops": 2.0 * rows * H * 2 * I}
    down = {"bytes": (hit + 1) * H * I * 2 + rows * I * 2 + rows * H * 2,
            "flops": 2.0 * rows * I * H}
    return gate_up, down


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

    def __init__(self, index, period=0.01):
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


def _cached(key, fn):
    if key not in _CPU_INPUTS:
        _CPU_INPUTS[key] = fn()
    return _CPU_INPUTS[key]


def cpu_reference_sample(cfg, seed=1):
    """Time the reference's CPU path (restated in ``oracle/``) on a bounded sample and
    extrapolate it to one full step of ``cfg``.  Returns (tokens/s, cores, description)."""
    from layerbatch_b200 import workloads as W
    from oracle import attention as OA
    from oracle import moe as OM
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    t_total = 0.0
    parts = []
    full_tokens = 0
    with torch.no_grad():
        if cfg in ("c1", "c2", "c4"):
            full = {"c1": (64, (512, 4096), None), "c2": (128, (256, 8192), (2048, 2048)),
                    "c4": (512, (1024, 16384), (0, 4096))}[cfg]
            n_dec, (lo, hi), pf = full
            ns = min(16, n_dec)
            dec = W.uniform_ctx(ns, lo, hi, seed)
            b = _cached(("dec", cfg), lambda: W.make_attn_batch(dec, (), seed=seed))
            t0 = time.perf_counter()
            o = OA.paged_decode_bf16(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                                     b.scale)
            OA.gate_oproj_bf16(o.flatten(1, -1), b.gate.reshape(ns, -1), b.w_o)
            t_dec = (time.perf_counter() - t0) * n_dec / ns
            parts.append(f"{ns}/{n_dec} decode seqs (x{n_dec / ns:.0f})")
            t_total += t_dec
            full_tokens += n_dec
            if pf is not None:
                prefix, chunk = pf
                sc = 512
                bp = _cached(("pf", cfg), lambda: W.make_attn_batch(
                    [], [(min(prefix, sc), sc)], seed=seed))
                t0 = time.perf_counter()
                o = OA.paged_prefill_bf16(bp.q, bp.k_cache, bp.v_cache, bp.block_tables,
                                          bp.context_lens, bp.cu_seqlens_q, bp.scale)
                OA.gate_oproj_bf16(o.reshape(sc, -1), bp.gate.reshape(sc, -1), bp.w_o)
                dt = time.perf_counter() - t0
                pairs_s = sc * min(prefix, sc) + sc * (sc + 1) / 2
                pairs_f = chunk * prefix + chunk * (chunk + 1) / 2
                t_total += dt * pairs_f / pairs_s
                parts.append(f"{sc}-token prefill chunk (x{pairs_f / pairs_s:.0f} by causal pairs)")
                full_tokens += chunk
        if cfg in ("c3s", "c3l", "c4"):
            T_full = {"c3s": 256, "c3l": 8192, "c4": 4608}[cfg]
            Ts = min(256, T_full)
            def mk():
                p = W.make_moe_params(2048, 512, 512, 512, 10, seed=0)
                x = W.make_moe_input(Ts, 2048, seed=seed)
                W.apply_zipf_bias(p, x)
                return p, x
            p, x = _cached(("moe", Ts), mk)
            t0 = time.perf_counter()
            OM.moe_block_bf16(x, p, "sparse")
            dt = time.perf_counter() - t0
            t_total += dt * T_full / Ts
            parts.append(f"MoE sparse path at T={Ts} (x{T_full / Ts:.0f})")
            if cfg != "c4":
                full_tokens = T_full
    return full_tokens / t_total, cores, "; ".join(parts) + f"; {cores} threads"


# ---------------------------------------------------------------------------- GPU side
def run_ours(args, rank, world, device):
    from layerbatch_b200 import ops
    from layerbatch_b200 import workloads as W
    cfg = args.config
    seed = 1 + rank
    sharded = world > 1 and cfg == "c4"
    tp = 2 if (sharded and world % 2 == 0) else 1
    tp_group, shard, ep_block = None, None, None
    if sharded:
        # TP pairs by KV head, data parallel across pairs, experts split over all ranks.
        # Per-GPU work stays that of one c4 batch: a TP pair runs tp batches.
        from layerbatch_b200.engine import sharding as S
        from layerbatch_b200.layers.fused_moe import Qwen3_5SparseMoeBlock
        groups = [torch.distributed.new_group(list(range(g * tp, (g + 1) * tp)))
                  for g in range(world // tp)] if tp > 1 else []
        gid, tp_rank = rank // tp, rank % tp
        tp_group = groups[gid] if tp > 1 else None
        shard = S.attention_shard(16, 2, tp_rank, tp)
        dec = W.uniform_ctx(512 * tp, 1024, 16384, seed=100 + gid)
        attn = W.make_attn_batch(dec, [(0, 4096)] * tp, Hq=16 // tp, Hkv=2 // tp, H=2048,
                                 seed=1000 + rank, device=device)
        attn.scale = 256 ** -0.5
    else:
        attn = attn_batch_for(cfg, seed, device)
    T_moe = moe_tokens_for(cfg, attn) if not sharded else 4608
    moe = None
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
        if sharded:
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

    a_out = torch.empty(attn.num_tokens, attn.w_o.shape[0], dtype=torch.bfloat16,
                        device=device) if attn is not None else None
    m_out = torch.empty_like(moe[1]) if moe else None

    def step(ev_a=None, ev_m=None, q=None, gate=None, x=None, meta=None, out_a=None,
             out_m=None):
        if attn is not None:
            qq = q if q is not None else attn.q
            gg = gate if gate is not None else attn.gate
            bt, cl, cu = meta if meta is not None else (attn.block_tables, attn.context_lens,
                                                        attn.cu_seqlens_q)
            oa = out_a if out_a is not None else a_out
            if sharded:
                S.tp_attention_oproj(shard, qq, gg, attn.k_cache, attn.v_cache, bt, cl, cu,
                                     attn.w_o, attn.scale, group=tp_group, max_q_len=max_q,
                                     events=ev_a, out=oa, work_hint=hint, exchange=tp_ex)
            else:
                ops.pod_attn_oproj(qq, gg, attn.k_cache, attn.v_cache, bt, cl, cu, attn.w_o,
                                   attn.scale, out=oa, max_q_len=max_q, events=ev_a,
                                   work_hint=hint)
        if moe:
            pm, xm = moe
            xx = x if x is not None else xm
            om = out_m if out_m is not None else m_out
            if sharded:
                from layerbatch_b200.engine.ep import ep_moe_forward_nvlink
                ep_moe_forward_nvlink(ep_block, xx, ep_block.ep_exchange, out=om)
            else:
                ops.moe_forward(xx, pm.router, pm.gate_up, pm.down, pm.sh_gate, pm.sh_up,
                                pm.sh_down, pm.sh_gate_w, 10, out=om, events=ev_m)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    K, Wu = args.steps, args.warmup
    for _ in range(Wu):
        step()
    torch.cuda.synchronize()
    ev_attn = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(K)]
    ev_moe = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = ops.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        st.record()
        for i in range(K):
            step(ev_attn[i] if attn is not None else None,
                 ev_moe[i] if (moe and not sharded) else None)
        en.record()
        torch.cuda.synchronize()
    barrier()
    launches = ops.launch_count() - n0
    ms = st.elapsed_time(en) / K
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms = float(ms_t)
    ws_status = 0
    for tag in ("pod", "moe", "tp_attn", "ep_owner", "ep_source"):
        if (torch.cuda.current_device(), tag) in ops._WS:
            ws_status |= ops.device_status(ops._WS[(torch.cuda.current_device(), tag)])

    res = {"ms": ms, "tokens": tokens, "launches": launches, "clocks": clk.summary(),
           "device_status": ws_status}
    peaks = load_peaks()
    if attn is not None:
        t_attn = statistics.mean(e[0].elapsed_time(e[1]) for e in ev_attn) * 1e-3
        flops, byts = attn_work(attn)
        res["attn"] = {"ms": t_attn * 1e3, "flops": flops, "bytes": byts,
                       "gbs": byts / t_attn / 1e9, "tflops": flops / t_attn / 1e12}
    if moe and not sharded:
        t_g1 = statistics.mean(e[0].elapsed_time(e[1]) for e in ev_moe) * 1e-3
        t_g2 = statistics.mean(e[2].elapsed_time(e[3]) for e in ev_moe) * 1e-3
        res["moe_gemm"] = {"gate_up_ms": t_g1 * 1e3, "down_ms": t_g2 * 1e3,
                           "experts_hit": moe_hit}
        gu, dn = moe_work(T_moe, moe_hit)
        res["moe_gate_up"] = dict(gu, ms=t_g1 * 1e3, gbs=gu["bytes"] / t_g1 / 1e9,
                                  tflops=gu["flops"] / t_g1 / 1e12)
        res["moe_gemm"].update(gate_up_gbs=gu["bytes"] / t_g1 / 1e9,
                               down_gbs=dn["bytes"] / t_g2 / 1e9)
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
            pin["q"] = attn.q.cpu().pin_memory()
            pin["gate"] = attn.gate.cpu().pin_memory()
            pin["meta"] = [t.cpu().pin_memory() for t in
                           (attn.block_tables, attn.context_lens, attn.cu_seqlens_q)]
        if moe:
            pin["x"] = moe[1].cpu().pin_memory()
        bufs, host_out = [], []
        for _ in range(2):
            bd = {}
            if attn is not None:
                bd["q"] = torch.empty_like(attn.q)
                bd["gate"] = torch.empty_like(attn.gate)
                bd["meta"] = [torch.empty_like(t) for t in
                              (attn.block_tables, attn.context_lens, attn.cu_seqlens_q)]
                bd["out_a"] = torch.empty_like(a_out)
            if moe:
                bd["x"] = torch.empty_like(moe[1])
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

        def e2e_step(i):
            k = i % 2
            bd, ho = bufs[k], host_out[k]
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_used[k])          # step i-2 is done reading buffer k
                if attn is not None:
                    bd["q"].copy_(pin["q"], non_blocking=True)
                    bd["gate"].copy_(pin["gate"], non_blocking=True)
                    for dst, src in zip(bd["meta"], pin["meta"]):
                        dst.copy_(src, non_blocking=True)
                if moe:
                    bd["x"].copy_(pin["x"], non_blocking=True)
                ev_in[k].record(s_in)
            comp.wait_event(ev_in[k])
            comp.wait_event(ev_out[k])                # step i-2's outputs have been read
            step(q=bd.get("q"), gate=bd.get("gate"), x=bd.get("x"), meta=bd.get("meta"),
                 out_a=bd.get("out_a"), out_m=bd.get("out_m"))
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
        Ke = max(4, K // 2)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg_desc = {"workload": CONFIGS[args.config]}

    if args.impl == "reference":
        # The reference path is CPU code: rank 0 alone times it on the host cores.
        if rank != 0:
            return
        vals = []
        for i in range(args.warmup + args.steps):
            v, cores, sample = cpu_reference_sample(args.config)
            if i >= args.warmup:
                vals.append(v)
        v = statistics.median(vals)
        line = {"metric": "hot-path tokens/s", "value": v, "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
                "config": dict(cfg_desc, parallelism="host CPU"), "impl": "reference",
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

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_reference_sample(args.config)
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
            "config": dict(cfg_desc, tokens_per_step_per_gpu=res["tokens"],
                           l2="inputs larger than L2 (KV cache and expert weights are GBs)",
                           parallelism=res["parallelism"]),
            "roofline": roof, "cpu_baseline": cpu, "clocks": res["clocks"],
            "gpu_launches": res["launches"],
        }
        if "moe_gemm" in res:
            line["moe_gemm_ms"] = res["moe_gemm"]
        if "e2e" in res:
            e = res["e2e"]
            line["e2e"] = {"value": res["tokens"] * world / (e["ms"] * 1e-3), "unit": "tokens/s",
                           "h2d_bytes_per_step": e["h2d"], "d2h_bytes_per_step": e["d2h"]}
        if res["device_status"]:
            line["device_status"] = res["device_status"]
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
