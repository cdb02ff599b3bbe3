"""bench.py on the CPU: the algorithmic work behind its roofline numbers, and the
reference arm's JSON line (the reference's CPU path, restated in oracle/, timed on a
bounded sample)."""
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


def test_moe_work_is_the_hit_experts_weights_plus_rows():
    gu, dn = bench.moe_work(256, 367)
    rows = 256 * 10 + 256
    assert gu["bytes"] == 368 * 2 * 512 * 2048 * 2 + rows * 2048 * 2 + rows * 512 * 2
    assert dn["bytes"] == 368 * 2048 * 512 * 2 + rows * 512 * 2 + rows * 2048 * 2
    assert gu["flops"] == 2.0 * rows * 2048 * 1024 and dn["flops"] == 2.0 * rows * 512 * 2048


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "hot-path tokens/s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
