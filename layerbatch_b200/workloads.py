"""Seeded synthetic workloads for the hot path (no checkpoints or datasets exist offline).

Shapes follow the five benchmark configurations of the hot path:

* ``c0``: one MoE block, T=64, H=2048, E=64, top-8, I=512, shared I=512.
* ``c1``: decode-only paged attention + gated o_proj, B=64, ctx ~ U[512,4096],
  Hq=16, Hkv=2, D=256, 256-token pages, shuffled block tables.
* ``c2``: mixed batch: one 2048-token prefill chunk on a 2048-token cached prefix
  plus 128 decode sequences with ctx ~ U[256,8192].
* ``c3``: full-width MoE, H=2048, E=512, top-10, I=512, shared I=512, T=256 or 8192,
  router biased towards a Zipf(1.1) expert load.
* ``c4``: hybrid pair: c1-shaped attention over 512 decode sequences with
  ctx ~ U[1024,16384] plus one 4096-token prefill chunk, then the c3 MoE at T=4608.

The whole gated attention layer (``make_attn_layer_params`` / ``layer_positions_slots``)
starts from hidden states: one merged q/k/v projection, the (1+w) RMSNorm + partial RoPE
prologue with the K/V store of the new tokens, then POD attention, gate and o_proj.

Weights are N(0, 0.02) bf16, activations N(0, 1) bf16.  Small cases are drawn from a
CPU ``torch.Generator`` so that the CPU oracle and the GPU path see identical bytes;
large bench cases may be drawn directly on the device (``device='cuda'``), which gives
different (but equally seeded) values.

The KV cache layout is the reference engine's: ``[num_blocks, 256, Hkv, D]`` per layer
(nanovllm/engine/model_runner.py:387-416), block tables ``[B, max_blocks]`` int32 padded
with -1 (model_runner.py:493-657), ``context_lens`` = cached + current tokens
(model_runner.py:634).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK_SIZE = 256


def _gen(seed: int, device) -> torch.Generator:
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g


def _randn(g, shape, std, device, dtype=torch.bfloat16):
    t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


# ----------------------------------------------------------------------------------------
# MoE
# ----------------------------------------------------------------------------------------
@dataclass
class MoEParams:
    """Parameter tensors with the reference's names and shapes (qwen3_5.py:762-917).

    router        = mlp.gate.weight                     [E, H]
    gate_up       = mlp.experts.gate_up_proj            [E, 2I, H] (gate rows [0,I), up [I,2I))
    down          = mlp.experts.down_proj               [E, H, I]
    sh_gate       = mlp.shared_expert.gate_proj.weight  [Is, H]
    sh_up         = mlp.shared_expert.up_proj.weight    [Is, H]
    sh_down       = mlp.shared_expert.down_proj.weight  [H, Is]
    sh_gate_w     = mlp.shared_expert_gate.weight       [1, H]
    """
    router: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    sh_gate: torch.Tensor
    sh_up: torch.Tensor
    sh_down: torch.Tensor
    sh_gate_w: torch.Tensor
    top_k: int

    @property
    def num_experts(self):
        return self.router.shape[0]

    @property
    def hidden(self):
        return self.router.shape[1]

    @property
    def inter(self):
        return self.down.shape[2]

    @property
    def shared_inter(self):
        return self.sh_down.shape[1]

    def to(self, device):
        return MoEParams(*(getattr(self, f).to(device) for f in
                           ("router", "gate_up", "down", "sh_gate", "sh_up", "sh_down",
                            "sh_gate_w")), top_k=self.top_k)


def make_moe_params(H, E, I, Is, top_k, seed=0, device="cpu", std=0.02) -> MoEParams:
    """Draw MoE weights in a fixed order from one seeded generator."""
    g = _gen(seed, device)
    router = _randn(g, (E, H), std, device)
    gate_up = _randn(g, (E, 2 * I, H), std, device)
    down = _randn(g, (E, H, I), std, device)
    sh_gate = _randn(g, (Is, H), std, device)
    sh_up = _randn(g, (Is, H), std, device)
    sh_down = _randn(g, (H, Is), std, device)
    sh_gate_w = _randn(g, (1, H), std, device)
    return MoEParams(router, gate_up, down, sh_gate, sh_up, sh_down, sh_gate_w, top_k)


def make_moe_input(T, H, seed=1, device="cpu") -> torch.Tensor:
    g = _gen(seed, device)
    return _randn(g, (T, H), 1.0, device)


def zipf_targets(E: int, total: int, cap: int, s: float = 1.1) -> torch.Tensor:
    """Expert loads proportional to rank^-s summing to ``total``, none above ``cap``
    (one expert can take each token at most once)."""
    w = torch.arange(1, E + 1, dtype=torch.float64) ** (-s)
    lo, hi = 0.0, float(total) / float(w.min())
    for _ in range(100):
        c = 0.5 * (lo + hi)
        if torch.clamp(c * w, max=cap).sum() > total:
            hi = c
        else:
            lo = c
    return torch.clamp(lo * w, max=cap)


def apply_zipf_bias(params: MoEParams, x: torch.Tensor, s: float = 1.1, seed: int = 2,
                    calib_tokens: int = 2048, iters: int = 60):
    """Bias the router so that the expert LOAD (selections per expert) follows Zipf(s).

    Hidden dimension 0 of every token is set to 1 and router column 0 of expert e is set
    to a bias b_e, so the router operator itself is unchanged.  Experts get Zipf ranks
    from a seeded permutation; the biases are calibrated by a fixed-point iteration on a
    seeded calibration batch (``calib_tokens`` N(0,1) tokens) so that the top-k selection
    counts match ``zipf_targets`` (rank^-s, capped at one selection per token).
    Returns the rank of every expert (1 = most loaded).
    """
    E, H = params.router.shape
    k = params.top_k
    g = torch.Generator().manual_seed(seed)
    rank = torch.randperm(E, generator=g) + 1
    xc = torch.randn(calib_tokens, H, generator=g).to(torch.bfloat16).float()
    w = params.router.detach().float().cpu()
    noise = xc[:, 1:] @ w[:, 1:].t()                     # [Tc, E] logit part without bias
    target = zipf_targets(E, calib_tokens * k, calib_tokens, s)[rank - 1]
    b = -s * torch.log(rank.double()).float()
    for _ in range(iters):
        top = torch.topk(noise + b, k, dim=-1).indices
        cnt = torch.bincount(top.reshape(-1), minlength=E).float()
        b = b + 0.5 * (torch.log(target.float() + 1.0) - torch.log(cnt + 1.0))
        b = b - b.max()
    params.router[:, 0] = b.to(torch.bfloat16).to(params.router.device)
    x[:, 0] = 1.0
    return rank


C0 = dict(T=64, H=2048, E=64, I=512, Is=512, top_k=8)
C3 = dict(H=2048, E=512, I=512, Is=512, top_k=10)


# ----------------------------------------------------------------------------------------
# Attention
# ----------------------------------------------------------------------------------------
@dataclass
class AttnBatch:
    """One forward batch for the full-attention layer's hot path.

    Tokens are packed as ``[prefill chunk tokens..., decode tokens...]``:
    ``q``/``gate`` are ``[N, Hq, D]`` with N = sum(prefill q lens) + num_decode.
    ``seq_q_start``/``seq_q_len`` describe each sequence's query rows; prefill sequences
    come first.  ``context_lens[b]`` counts cached + new tokens of sequence b.
    """
    q: torch.Tensor                  # [N, Hq, D] bf16 (post norm/RoPE query)
    gate: torch.Tensor               # [N, Hq, D] bf16 (output gate pre-sigmoid)
    k_cache: torch.Tensor            # [num_blocks, 256, Hkv, D]
    v_cache: torch.Tensor
    block_tables: torch.Tensor       # [B, max_blocks] int32, -1 padded
    context_lens: torch.Tensor       # [B] int32
    cu_seqlens_q: torch.Tensor       # [B+1] int32
    num_prefill: int                 # sequences [0, num_prefill) are prefill chunks
    w_o: torch.Tensor                # [H, Hq*D] bf16
    scale: float
    ctx_list: list = field(default_factory=list)
    qlen_list: list = field(default_factory=list)

    @property
    def num_seqs(self):
        return self.context_lens.numel()

    @property
    def num_tokens(self):
        return self.q.shape[0]

    def to(self, device):
        kw = {}
        for f in ("q", "gate", "k_cache", "v_cache", "block_tables", "context_lens",
                  "cu_seqlens_q", "w_o"):
            kw[f] = getattr(self, f).to(device)
        return AttnBatch(num_prefill=self.num_prefill, scale=self.scale,
                         ctx_list=list(self.ctx_list), qlen_list=list(self.qlen_list), **kw)


def make_attn_batch(decode_ctx, prefill=(), Hq=16, Hkv=2, D=256, H=2048, seed=1,
                    device="cpu", extra_blocks=0, w_std=0.02, tile_pages=0) -> AttnBatch:
    """Build a paged batch.

    decode_ctx: list of context lengths (cached + 1) of the decode sequences.
    prefill: list of (prefix_len, chunk_len) for prefill sequences (put first).
    Pages are drawn as a seeded random permutation of the block pool (shuffled tables).
    The K/V cache holds N(0,1) values for every slot (new tokens' K/V are assumed
    already stored, as the reference stores them before attending, attention.py:103).
    ``tile_pages > 0`` draws only that many pages of N(0,1) K/V and repeats them over the
    pool: a gigabyte-sized host cache in seconds, for CPU timing where values do not
    change the work.
    """
    g = _gen(seed, device)
    gcpu = torch.Generator().manual_seed(seed + 1000)
    ctx_list = [p + c for p, c in prefill] + list(decode_ctx)
    qlen_list = [c for _, c in prefill] + [1] * len(decode_ctx)
    B = len(ctx_list)
    nblk = [math.ceil(c / BLOCK_SIZE) for c in ctx_list]
    max_blocks = max(nblk) if nblk else 1
    num_blocks = sum(nblk) + extra_blocks
    perm = torch.randperm(num_blocks, generator=gcpu).to(torch.int32)
    bt = torch.full((B, max_blocks), -1, dtype=torch.int32)
    pos = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[pos:pos + n]
        pos += n
    N = sum(qlen_list)
    q = _randn(g, (N, Hq, D), 1.0, device)
    gate = _randn(g, (N, Hq, D), 1.0, device)
    if tile_pages > 0 and num_blocks > tile_pages:
        caches = []
        for _ in range(2):
            blk = _randn(g, (tile_pages, BLOCK_SIZE, Hkv, D), 1.0, device)
            c = torch.empty((num_blocks, BLOCK_SIZE, Hkv, D), dtype=torch.bfloat16,
                            device=device)
            for i in range(0, num_blocks, tile_pages):
                n = min(tile_pages, num_blocks - i)
                c[i:i + n] = blk[:n]
            caches.append(c)
        k_cache, v_cache = caches
    else:
        k_cache = _randn(g, (num_blocks, BLOCK_SIZE, Hkv, D), 1.0, device)
        v_cache = _randn(g, (num_blocks, BLOCK_SIZE, Hkv, D), 1.0, device)
    w_o = _randn(g, (H, Hq * D), w_std, device)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(qlen_list, dtype=torch.int64), 0).to(torch.int32)
    return AttnBatch(q=q, gate=gate, k_cache=k_cache, v_cache=v_cache,
                     block_tables=bt.to(device),
                     context_lens=torch.tensor(ctx_list, dtype=torch.int32, device=device),
                     cu_seqlens_q=cu.to(device), num_prefill=len(prefill), w_o=w_o,
                     scale=D ** -0.5, ctx_list=ctx_list, qlen_list=qlen_list)


def uniform_ctx(n, lo, hi, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def c1_batch(seed=1, device="cpu", **kw):
    return make_attn_batch(uniform_ctx(64, 512, 4096, seed), (), seed=seed, device=device, **kw)


def c2_batch(seed=1, device="cpu", **kw):
    return make_attn_batch(uniform_ctx(128, 256, 8192, seed), [(2048, 2048)], seed=seed,
                           device=device, **kw)


def c4_attn_batch(seed=1, device="cpu", **kw):
    return make_attn_batch(uniform_ctx(512, 1024, 16384, seed), [(0, 4096)], seed=seed,
                           device=device, **kw)


# ----------------------------------------------------------------------------------------
# The whole gated attention layer (projections and prologue in front of the POD call)
# ----------------------------------------------------------------------------------------
@dataclass
class AttnLayerParams:
    """Weights of one gated full-attention layer (nanovllm/models/qwen3_5.py:587-746)
    besides ``w_o`` (which lives in the ``AttnBatch``).

    ``w_qkv`` stacks ``q_proj.weight [Hq*2D, H]`` (query and gate interleaved per head,
    qwen3_5.py:710-713), ``k_proj.weight [Hkv*D, H]`` and ``v_proj.weight [Hkv*D, H]`` so
    that one GEMM computes all three projections.  ``cos_sin_cache`` is the rotary module's
    fp32 ``[max_position, rotary_dim]`` table (rotary_embedding.py:26-33).
    """
    w_qkv: torch.Tensor
    q_norm_w: torch.Tensor
    k_norm_w: torch.Tensor
    cos_sin_cache: torch.Tensor
    num_heads: int
    num_kv_heads: int
    head_dim: int
    eps: float = 1e-6

    def split(self, qkv: torch.Tensor):
        """Views of one ``[N, Hq*2D + 2*Hkv*D]`` projection output: query ``[N, Hq, D]``,
        gate ``[N, Hq, D]`` (both strided inside q_proj's per-head ``[query | gate]``),
        key and value ``[N, Hkv, D]``."""
        N = qkv.shape[0]
        Hq, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        q3 = qkv[:, :Hq * 2 * D].view(N, Hq, 2 * D)
        k = qkv[:, Hq * 2 * D:Hq * 2 * D + Hkv * D].view(N, Hkv, D)
        v = qkv[:, Hq * 2 * D + Hkv * D:].view(N, Hkv, D)
        return q3[..., :D], q3[..., D:], k, v


def rotary_cache(rotary_dim: int, max_position: int, base: float) -> torch.Tensor:
    """fp32 ``[max_position, rotary_dim]`` cos|sin table built with the reference's own
    torch operations (rotary_embedding.py:26-33), so every device reads identical bits."""
    from .layers.full_attention import RotaryEmbedding
    rope = RotaryEmbedding(rotary_dim, rotary_dim, max_position, base)
    return rope.cos_sin_cache.reshape(max_position, rotary_dim).contiguous()


def make_attn_layer_params(H=2048, Hq=16, Hkv=2, D=256, rotary_dim=64, theta=1.0e7,
                           max_position=16384 + 4096, seed=0, device="cpu",
                           std=0.02) -> AttnLayerParams:
    g = _gen(seed, device)
    w_qkv = _randn(g, (Hq * 2 * D + 2 * Hkv * D, H), std, device)
    q_norm_w = _randn(g, (D,), std, device)
    k_norm_w = _randn(g, (D,), std, device)
    cs = rotary_cache(rotary_dim, max_position, theta).to(device)
    return AttnLayerParams(w_qkv, q_norm_w, k_norm_w, cs, Hq, Hkv, D)


def layer_positions_slots(batch: AttnBatch):
    """Positions and KV slots of the batch's new tokens: sequence b's query rows are its
    last ``qlen_b`` positions of ``ctx_b`` (model_runner.py:493-657); the slot of position
    p is ``block_tables[b, p // 256] * 256 + p % 256``.  Returns CPU (int64, int32)."""
    bt = batch.block_tables.cpu()
    pos, slot = [], []
    for b, (c, L) in enumerate(zip(batch.ctx_list, batch.qlen_list)):
        p = torch.arange(c - L, c, dtype=torch.int64)
        pos.append(p)
        slot.append(bt[b, p // BLOCK_SIZE].to(torch.int64) * BLOCK_SIZE + p % BLOCK_SIZE)
    if not pos:
        return torch.zeros(0, dtype=torch.int64), torch.zeros(0, dtype=torch.int32)
    return torch.cat(pos), torch.cat(slot).to(torch.int32)


def make_layer_input(N, H, seed=7, device="cpu") -> torch.Tensor:
    """Hidden states entering the attention layer, N(0, 1) bf16."""
    g = _gen(seed, device)
    return _randn(g, (N, H), 1.0, device)
