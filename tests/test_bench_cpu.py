"""bench.py on the CPU: the algorithmic work behind its roofline numbers, and the
reference arm's JSON line (the reference's CPU path, restated in oracle/, timed on full
steps of the workload)."""
import json
import os
import subprocess
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402
from layerbatch_b200 import workloads as W  # noqa: E402


def test_attention_work_counts_kv_bytes_and_causal_pairs():
    b = W.make_attn_batch([300, 1000], [(512, 256)], seed=1)
    flops, byts = bench.attn_work(b)
    Hq, D, Hkv = 16, 256, 2
    kv_tokens = 300 + 1000 + 768
    # decode rows see their whole context; the chunk's query i sees 512 + i + 1 keys
    pairs = 300 + 1000 + sum(512 + i + 1 for i in range(256))
    assert flops == 4.0 * pairs * Hq * D
    assert byts == kv_tokens * Hkv * D * 2 * 2 + 3 * b.num_tokens * Hq * D * 2


def test_moe_work_counts_weights_inputs_and_outputs_not_scratch_rows():
    gu, dn, layer = bench.moe_work(256, 367)
    rows = 256 * 10 + 256
    x = out = 256 * 2048 * 2
    # the hit experts' and the shared expert's weights, the token rows once; the gathered
    # rows, activations and weighted expert rows between the kernels are scratch
    assert gu["bytes"] == 368 * 2 * 512 * 2048 * 2 + x
    assert dn["bytes"] == 368 * 2048 * 512 * 2 + out
    assert layer["bytes"] == 512 * 2048 * 2 + gu["bytes"] + dn["bytes"] + 2048 * 2
    assert gu["flops"] == 2.0 * rows * 2048 * 1024 and dn["flops"] == 2.0 * rows * 512 * 2048
    assert layer["flops"] == 2.0 * 256 * 2048 * 512 + gu["flops"] + dn["flops"] + 2.0 * 256 * 2048


def test_both_arms_describe_the_same_config():
    for cfg in bench.CONFIGS:
        d = bench.config_dict(cfg, bench.tokens_per_step(cfg))
        assert set(d) == {"workload", "tokens_per_step_per_gpu", "l2"}
    assert bench.tokens_per_step("c4") == 4096 + 512


def test_layer_positions_and_slots_follow_the_block_tables():
    b = W.make_attn_batch([300, 1000], [(512, 256)], seed=1)
    pos, slots = W.layer_positions_slots(b)
    assert pos.tolist()[:2] == [512, 513] and pos.tolist()[-2:] == [299, 999]
    bt = b.block_tables
    for i, (n, p) in enumerate([(0, 512), (255, 767), (256, 299), (257, 999)]):
        seq = 0 if n < 256 else n - 255
        assert int(slots[n]) == int(bt[seq, p // 256]) * 256 + p % 256


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--config", "c1", "--steps", "2", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "hot-path tokens/s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # full steps of the workload, the same config object as the GPU arm's line
    assert "full c1 step" in cb["sample"] and 1 <= line["steps"] <= 2
    assert line["config"] == bench.config_dict("c1", 64)


def test_step_floor_is_the_slower_of_bytes_and_flops_per_stage():
    """The whole-step roofline of the c4 line: attention and the MoE layer bound by their
    bytes, the projections by their FLOPs, at the measured peaks."""
    b = W.make_attn_batch([4000] * 8, [(0, 512)], seed=3)
    peaks = {"hbm_gbs": 6546.6, "bf16_tflops": 1619.4}
    st = bench.step_floor(b, b.num_tokens, 500, 16, 2, peaks)
    fa, ba = bench.attn_work(b)
    assert st["attention"] == max(ba / 6546.6e9, fa / 1619.4e12) == ba / 6546.6e9
    g, _ = bench.layer_proj_work(b.num_tokens)
    assert st["qkv_projection"] == g["flops"] / 1619.4e12 > g["bytes"] / 6546.6e9
    assert st["o_proj"] == 2.0 * b.num_tokens * 4096 * 2048 / 1619.4e12
    _, _, ly = bench.moe_work(b.num_tokens, 500)
    assert st["moe_layer"] == ly["bytes"] / 6546.6e9
