"""Mixed prefill + decode scheduling and metadata (host side, CPU)."""
import random

import torch

from layerbatch_b200 import ops
from layerbatch_b200.engine.batch_builder import (MixedScheduler, Sequence, SequenceStatus,
                                                  prepare_mixed, work_hint)


def _run_step(sched, rng):
    batch = sched.schedule()
    toks = {it.seq.seq_id: rng.randrange(1000) for it in batch.items}
    return batch, sched.postprocess(batch, toks)


def test_mixed_step_packs_decode_tokens_and_prompt_chunks():
    sched = MixedScheduler(num_blocks=64, max_num_batched_tokens=1000, chunk_size=512)
    seqs = [Sequence(list(range(n)), max_tokens=8) for n in (700, 300, 50)]
    for s in seqs:
        sched.add(s)
    rng = random.Random(0)
    b1, _ = _run_step(sched, rng)
    assert [(it.seq.seq_id, it.start, it.length) for it in b1.prefill] == [
        (seqs[0].seq_id, 0, 512), (seqs[1].seq_id, 0, 300), (seqs[2].seq_id, 0, 50)]
    assert not b1.decode
    # step 2: seqs 1 and 2 decode, seq 0 finishes its prompt in a chunk on its prefix
    b2 = sched.schedule()
    assert [it.seq.seq_id for it in b2.decode] == [seqs[1].seq_id, seqs[2].seq_id]
    assert [(it.seq.seq_id, it.start, it.length) for it in b2.prefill] == [(seqs[0].seq_id, 512, 188)]
    meta = prepare_mixed(b2)
    assert meta["cu_seqlens_q"].tolist() == [0, 188, 189, 190]
    assert meta["context_lens"].tolist() == [700, 301, 51]
    assert meta["positions"].tolist() == list(range(512, 700)) + [300, 50]
    bt = meta["block_tables"]
    pos, slots = meta["positions"].tolist(), meta["slot_mapping"].tolist()
    rows = [0] * 188 + [1, 2]
    for p, s_, r in zip(pos, slots, rows):
        assert s_ == int(bt[r, p // 256]) * 256 + p % 256
    # host work hint = the kernel wrapper's definition over (context, query length)
    assert work_hint(b2) == ops.pod_work_hint(meta["context_lens"].tolist(),
                                              [188, 1, 1])
    assert meta["max_seqlen_q"] == 188 and meta["num_prefill"] == 1


def test_random_workload_invariants():
    rng = random.Random(7)
    sched = MixedScheduler(num_blocks=40, max_num_seqs=16, max_num_batched_tokens=900,
                           chunk_size=400)
    for _ in range(30):
        sched.add(Sequence([1] * rng.randrange(1, 1200), max_tokens=rng.randrange(1, 40)))
    steps = 0
    while not sched.is_finished():
        steps += 1
        assert steps < 5000
        batch = sched.schedule()
        assert batch.items, "scheduler stalled"
        assert batch.num_tokens <= 900 and len(batch.items) <= 16
        # blocks of running sequences are disjoint and cover the step's tokens
        seen = set()
        for s in sched.running:
            assert not (set(s.block_table) & seen)
            seen |= set(s.block_table)
        meta = prepare_mixed(batch)
        slots = meta["slot_mapping"].tolist()
        assert len(set(slots)) == len(slots)
        for it in batch.items:
            assert len(it.seq.block_table) * 256 >= it.start + it.length
        toks = {it.seq.seq_id: rng.randrange(1000) for it in batch.items}
        sched.postprocess(batch, toks)
    assert len(sched.pool.free) == 40


def test_preemption_frees_blocks_and_recomputes():
    sched = MixedScheduler(num_blocks=3, max_num_batched_tokens=2048, chunk_size=2048)
    a, b = Sequence([1] * 256, max_tokens=300), Sequence([2] * 255, max_tokens=300)
    sched.add(a)
    sched.add(b)
    rng = random.Random(1)
    for _ in range(40):
        batch, _ = _run_step(sched, rng)
    # 3 blocks cannot hold both once they grow: the newer one was preempted and waits
    assert b.status == SequenceStatus.WAITING or a.status == SequenceStatus.WAITING
    assert sum(len(s.block_table) for s in sched.running) <= 3


def test_expert_placement_by_load_balances_ranks():
    from layerbatch_b200.engine.ep import placement_by_load
    g = torch.Generator().manual_seed(0)
    loads = (1.0 / torch.arange(1, 513).double() ** 1.1)[torch.randperm(512, generator=g)] * 1e5
    for P in (2, 4, 8):
        pl = placement_by_load(loads, P)
        assert sorted(pl.tolist()) == list(range(512))
        epr = 512 // P
        per = [float(loads[pl[r * epr:(r + 1) * epr]].sum()) for r in range(P)]
        contig = [float(loads[r * epr:(r + 1) * epr].sum()) for r in range(P)]
        mean = sum(per) / P
        # never worse than contiguous ranges, and within 5 % of the lower bound of any
        # placement with E/P experts per rank: the mean, or the heaviest expert plus the
        # E/P - 1 lightest ones
        srt = loads.sort().values
        bound = max(mean, float(srt[-1]) + float(srt[:epr - 1].sum()))
        assert max(per) <= max(contig) + 1e-6
        assert max(per) <= bound * 1.05 + 1e-6
