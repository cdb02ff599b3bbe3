"""Mixed prefill + decode batch builder for the POD attention kernel.

The reference scheduler (nanovllm/engine/scheduler.py:25-59) returns either a prefill
batch or a decode batch, never both, and the runner prepares them separately
(nanovllm/engine/model_runner.py:499-650).  ``lb_pod_attn_oproj`` runs prefill chunks
and decode steps in one launch, so this scheduler packs both into every step:

* every running sequence whose prompt is fully processed contributes its one decode
  token (a new KV block is taken when its last block is full; when the pool is empty the
  newest running sequence is preempted, as the reference does, ``scheduler.py:44-52``);
* the remaining token budget (``max_num_batched_tokens``) goes to prompt chunks, first to
  the sequence whose prompt is partly processed, then to waiting sequences in arrival
  order, at most ``chunk_size`` tokens per sequence and step (chunked prefill; a chunk
  attends to the sequence's cached prefix with bottom-right causal alignment).

``prepare_mixed`` turns a step into the kernel's metadata (``cu_seqlens_q``,
``context_lens``, ``block_tables`` padded with -1, ``slot_mapping``, ``positions``,
``input_ids``) plus the host work hint (prefill query-key pairs, decode context
tokens), with the prefill chunks first.  It reads no device memory: everything comes
from host-side sequence state, and the tensors are copied to the device from pinned
memory without a synchronisation.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from enum import Enum, auto
from itertools import count

import torch


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    """Token state of one request (the fields of nanovllm/engine/sequence.py:14-31 this
    builder uses); ``num_computed`` counts tokens whose K/V are in the cache."""

    block_size = 256
    _ids = count()

    def __init__(self, token_ids: list[int], max_tokens: int = 64, ignore_eos: bool = False):
        self.seq_id = next(Sequence._ids)
        self.status = SequenceStatus.WAITING
        self.token_ids = list(token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.num_computed = 0
        self.block_table: list[int] = []
        self.max_tokens = max_tokens
        self.ignore_eos = ignore_eos

    def __len__(self):
        return len(self.token_ids)

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def in_prefill(self) -> bool:
        """Prompt tokens remain to be processed (more than the one token a decode runs)."""
        return self.num_computed < self.num_tokens - 1 or self.num_computed < self.num_prompt_tokens

    def blocks_for(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size


class BlockPool:
    """Free list of KV-cache blocks (no prefix caching)."""

    def __init__(self, num_blocks: int):
        self.free = deque(range(num_blocks))

    def can_grow(self, seq: Sequence, n_tokens: int) -> bool:
        return seq.blocks_for(n_tokens) - len(seq.block_table) <= len(self.free)

    def grow(self, seq: Sequence, n_tokens: int):
        need = seq.blocks_for(n_tokens) - len(seq.block_table)
        for _ in range(max(0, need)):
            seq.block_table.append(self.free.popleft())

    def release(self, seq: Sequence):
        self.free.extend(seq.block_table)
        seq.block_table = []


@dataclass
class StepItem:
    seq: Sequence
    start: int     # first token position computed this step
    length: int    # tokens computed this step (1 for a decode step)


@dataclass
class MixedBatch:
    prefill: list = field(default_factory=list)   # StepItem, chunks of prompts
    decode: list = field(default_factory=list)    # StepItem, one token each

    @property
    def items(self):
        return self.prefill + self.decode

    @property
    def num_tokens(self) -> int:
        return sum(i.length for i in self.items)


class MixedScheduler:
    """Packs decode tokens and prompt chunks into one step (API after
    nanovllm/engine/scheduler.py: ``add``, ``schedule``, ``postprocess``,
    ``is_finished``)."""

    def __init__(self, num_blocks: int, max_num_seqs: int = 512,
                 max_num_batched_tokens: int = 8192, chunk_size: int | None = None,
                 eos: int = -1, max_model_len: int = 1 << 20):
        self.pool = BlockPool(num_blocks)
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.chunk_size = chunk_size or max_num_batched_tokens
        self.eos = eos
        self.max_model_len = max_model_len
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()

    def add(self, seq: Sequence):
        self.waiting.append(seq)

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def _preempt(self, seq: Sequence):
        seq.status = SequenceStatus.WAITING
        seq.num_computed = 0
        self.pool.release(seq)
        self.waiting.appendleft(seq)

    def schedule(self) -> MixedBatch:
        batch = MixedBatch()
        budget = self.max_num_batched_tokens
        # decode tokens of the running sequences, oldest first
        decoding = [s for s in self.running if not s.in_prefill]
        scheduled = set()
        for seq in decoding:
            if len(batch.decode) >= self.max_num_seqs or budget == 0:
                break
            if seq.status != SequenceStatus.RUNNING:    # preempted to make room
                continue
            while not self.pool.can_grow(seq, seq.num_tokens):
                # the newest running sequence not yet in this step makes room
                others = [s for s in self.running if s is not seq and s.seq_id not in scheduled]
                victim = others[-1] if others else seq
                self.running.remove(victim)
                self._preempt(victim)
                if victim is seq:
                    break
            if seq.status != SequenceStatus.RUNNING:
                continue
            self.pool.grow(seq, seq.num_tokens)
            batch.decode.append(StepItem(seq, seq.num_tokens - 1, 1))
            scheduled.add(seq.seq_id)
            budget -= 1
        # prompt chunks: partly prefilled running sequences first, then waiting ones
        nseq = len(batch.decode)
        candidates = [s for s in self.running if s.in_prefill] + list(self.waiting)
        for seq in candidates:
            if budget == 0 or nseq >= self.max_num_seqs:
                break
            # a sequence resumed after preemption recomputes all its tokens the same way
            todo = seq.num_tokens - seq.num_computed
            n = min(todo, budget, self.chunk_size)
            if n <= 0 or not self.pool.can_grow(seq, seq.num_computed + n):
                break
            self.pool.grow(seq, seq.num_computed + n)
            if seq.status == SequenceStatus.WAITING:
                self.waiting.remove(seq)
                seq.status = SequenceStatus.RUNNING
                self.running.append(seq)
            batch.prefill.append(StepItem(seq, seq.num_computed, n))
            budget -= n
            nseq += 1
        return batch

    def postprocess(self, batch: MixedBatch, token_ids: dict[int, int]) -> list[Sequence]:
        """Advance the computed counts; append the sampled token of every sequence whose
        step reached the end of its tokens (``token_ids[seq_id]``); retire finished ones
        (EOS, max_tokens, max_model_len), as scheduler.py:68-78."""
        finished = []
        for it in batch.items:
            seq = it.seq
            seq.num_computed = it.start + it.length
            if seq.num_computed < seq.num_tokens:
                continue                          # prompt chunk in the middle of the prompt
            tok = token_ids[seq.seq_id]
            seq.token_ids.append(tok)
            if ((not seq.ignore_eos and tok == self.eos)
                    or seq.num_completion_tokens >= seq.max_tokens
                    or seq.num_tokens >= self.max_model_len):
                seq.status = SequenceStatus.FINISHED
                self.pool.release(seq)
                self.running.remove(seq)
                finished.append(seq)
        return finished


def work_hint(batch: MixedBatch) -> tuple[int, int]:
    """(prefill query-key pairs, decode context tokens) of a step, as lb_pod_attn_oproj's
    host hint: a chunk of L tokens ending at context C sees L*(C-L) + L*(L+1)/2 pairs."""
    pairs = 0
    for it in batch.prefill:
        C, L = it.start + it.length, it.length
        pairs += L * (C - L) + L * (L + 1) // 2
    dec = sum(it.start + 1 for it in batch.decode)
    return pairs, dec


def prepare_mixed(batch: MixedBatch, device=None, block_size: int = 256) -> dict:
    """Kernel metadata of one mixed step, prefill chunks first (host-side, pinned copies)."""
    items = batch.items
    input_ids, positions, slots, ctx, cu = [], [], [], [], [0]
    max_blocks = 1
    for it in items:
        seq = it.seq
        end = it.start + it.length
        input_ids.extend(seq.token_ids[it.start:end])
        positions.extend(range(it.start, end))
        for p in range(it.start, end):
            slots.append(seq.block_table[p // block_size] * block_size + p % block_size)
        ctx.append(end)
        cu.append(cu[-1] + it.length)
        max_blocks = max(max_blocks, (end + block_size - 1) // block_size)
    tables = [it.seq.block_table[:(it.start + it.length + block_size - 1) // block_size] for it in items]
    tables = [t + [-1] * (max_blocks - len(t)) for t in tables]
    cu_k = [0]
    for c in ctx:
        cu_k.append(cu_k[-1] + c)

    def dev(x, dtype):
        t = torch.tensor(x, dtype=dtype)
        if device is None or torch.device(device).type == "cpu":
            return t
        return t.pin_memory().to(device, non_blocking=True)

    return dict(
        input_ids=dev(input_ids, torch.int64), positions=dev(positions, torch.int64),
        slot_mapping=dev(slots, torch.int32), context_lens=dev(ctx, torch.int32),
        cu_seqlens_q=dev(cu, torch.int32), cu_seqlens_k=dev(cu_k, torch.int32),
        block_tables=dev(tables if items else [[-1]], torch.int32),
        max_seqlen_q=max((it.length for it in items), default=0),
        max_seqlen_k=max(ctx, default=0), num_prefill=len(batch.prefill),
        work_hint=work_hint(batch))


def set_mixed_context(meta: dict):
    """Publish a mixed step to the layers: the prefill-with-block-tables context, which
    carries every sequence's query rows, context length (via cu_seqlens_k) and pages."""
    from ..utils.context import set_context
    set_context(True, cu_seqlens_q=meta["cu_seqlens_q"], cu_seqlens_k=meta["cu_seqlens_k"],
                max_seqlen_q=meta["max_seqlen_q"], max_seqlen_k=meta["max_seqlen_k"],
                slot_mapping=meta["slot_mapping"], context_lens=meta["context_lens"],
                block_tables=meta["block_tables"])
