"""CPU oracle of the MoE block (router top-k, permutation, experts, shared expert).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Each function cites the reference
lines it restates (paths are inside the reference project).

Two numerical flavours are provided:

* ``*_bf16``: the reference as written -- bf16 weights/activations with a bf16 rounding
  after every torch op (nanovllm/models/qwen3_5.py:767-917).
* ``moe_block_fp32``: the same math with every tensor upcast to fp32 ("fp32-accumulate
  result"), given a fixed routing.  The CUDA path is held to
  ``max|y - y_fp32| / max|y_fp32| <= 2e-2`` against it.

Routing contract: the reference's ``torch.topk`` has no defined order among equal
probabilities.  The oracle (and the CUDA kernel) break ties by lowest expert index;
``topk_route_reference`` keeps ``torch.topk`` for comparing with the reference's own output
up to tie-equivalent swaps.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


# ---------------------------------------------------------------- router (qwen3_5.py:767-774)
def router_logits(x: torch.Tensor, w_router: torch.Tensor) -> torch.Tensor:
    """``F.linear(hidden, W)`` in the input dtype (qwen3_5.py:769)."""
    return F.linear(x, w_router)


def topk_route(logits: torch.Tensor, k: int):
    """Softmax(fp32) -> top-k (ties: lowest index) -> renormalise (qwen3_5.py:770-772).

    Returns (weights_fp32 [T,k], ids int64 [T,k]); weights are NOT cast to bf16 here
    (``.to(bf16)`` at qwen3_5.py:773 is applied by the caller when wanted).
    """
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    vals, ids = torch.sort(probs, dim=-1, descending=True, stable=True)
    vals, ids = vals[:, :k], ids[:, :k]
    vals = vals / vals.sum(dim=-1, keepdim=True)
    return vals, ids


def topk_route_reference(logits: torch.Tensor, k: int, dtype=torch.bfloat16):
    """The reference router tail verbatim: ``torch.topk`` order (qwen3_5.py:770-774)."""
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    vals, ids = torch.topk(probs, k, dim=-1)
    vals = vals / vals.sum(dim=-1, keepdim=True)
    return vals.to(dtype), ids


def same_up_to_ties(ids_a, ids_b, logits) -> torch.Tensor:
    """Per-row check that two top-k selections are equivalent under ties.

    Rows match when the selected expert sets are equal, or when they differ only in
    experts whose logit equals the k-th largest logit (a tie across the boundary).
    """
    ids_a = ids_a.long()
    ids_b = ids_b.long()
    k = ids_a.shape[1]
    kth = torch.sort(logits.float(), dim=-1, descending=True).values[:, k - 1]
    ok = torch.ones(ids_a.shape[0], dtype=torch.bool)
    for r in range(ids_a.shape[0]):
        sa, sb = set(ids_a[r].tolist()), set(ids_b[r].tolist())
        if sa == sb:
            continue
        diff = sa ^ sb
        ok[r] = all(float(logits[r, e]) == float(kth[r]) for e in diff)
    return ok


# ---------------------------------------------------------------- permutation
def permutation(ids: np.ndarray, num_groups: int):
    """Expert-major permutation of the (token, slot) pairs.

    Order inside an expert follows the reference's ``torch.where(expert_mask[e])`` on the
    ``[top_k, N]`` mask (qwen3_5.py:823-831): slot j major, token t minor.  Entries with an
    id outside ``[0, num_groups)`` (e.g. experts owned by another rank) are dropped.

    Returns ``(counts[G], offsets[G+1], perm_token[P], perm_slot[P], row_of[T,k])`` where
    ``row_of[t, j]`` is the permuted row of pair (t, j) or -1 if dropped.
    """
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    flat = ids.T.reshape(-1)                 # j-major: f = j*T + t
    valid = (flat >= 0) & (flat < num_groups)
    counts = np.bincount(flat[valid], minlength=num_groups).astype(np.int64)
    offsets = np.zeros(num_groups + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    f_idx = np.nonzero(valid)[0]
    order = f_idx[np.argsort(flat[valid], kind="stable")]
    perm_token = (order % T).astype(np.int64)
    perm_slot = (order // T).astype(np.int64)
    row_of = np.full((T, k), -1, dtype=np.int64)
    row_of[perm_token, perm_slot] = np.arange(order.size)
    return counts, offsets, perm_token, perm_slot, row_of


# ---------------------------------------------------------------- experts, bf16 (reference)
def experts_sparse_bf16(x, gate_up, down, ids, w):
    """``Qwen3_5Experts._forward_sparse`` restated (qwen3_5.py:815-841)."""
    E = gate_up.shape[0]
    out = torch.zeros_like(x)
    mask = F.one_hot(ids.long(), num_classes=E).permute(2, 1, 0)   # [E, k, N]
    hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero()
    for e in hit:
        e = e[0]
        pos, tok = torch.where(mask[e])
        cur = x[tok]
        g, u = F.linear(cur, gate_up[e]).chunk(2, dim=-1)
        h = F.silu(g) * u
        h = F.linear(h, down[e])
        h = h * w[tok, pos, None]
        out.index_add_(0, tok, h.to(out.dtype))
    return out


def experts_dense_bf16(x, gate_up, down, ids, w):
    """``Qwen3_5Experts._forward_dense`` restated (qwen3_5.py:843-874)."""
    N, k = ids.shape
    flat = ids.reshape(-1).long()
    gu = gate_up[flat]
    dn = down[flat]
    h = x.repeat_interleave(k, dim=0)
    y = torch.bmm(gu, h.unsqueeze(-1)).squeeze(-1)
    g, u = y.chunk(2, dim=-1)
    y = F.silu(g) * u
    y = torch.bmm(dn, y.unsqueeze(-1)).squeeze(-1)
    y = y.view(N, k, -1)
    return (y * w.unsqueeze(-1)).sum(dim=1)


def shared_expert_bf16(x, p):
    """Shared expert and its sigmoid gate (qwen3_5.py:903, 916-917)."""
    s = F.linear(F.silu(F.linear(x, p.sh_gate)) * F.linear(x, p.sh_up), p.sh_down)
    return torch.sigmoid(F.linear(x, p.sh_gate_w)) * s


def moe_block_bf16(x, p, path="sparse", ids=None, w=None):
    """``Qwen3_5SparseMoeBlock.forward`` restated (qwen3_5.py:899-905).

    ``path`` selects the prefill (sparse) or decode (dense) expert dispatch, which the
    reference picks from ``get_context().is_prefill`` (qwen3_5.py:808-813).  When ``ids``
    and ``w`` are given they replace the router's output.
    """
    shared = shared_expert_bf16(x, p)
    if ids is None:
        w, ids = topk_route_reference(router_logits(x, p.router), p.top_k, x.dtype)
    fn = experts_sparse_bf16 if path == "sparse" else experts_dense_bf16
    return fn(x, p.gate_up, p.down, ids, w) + shared


# ---------------------------------------------------------------- fp32 oracle
def experts_fp32(x, gate_up, down, ids, w, expert_base=0):
    """The routed experts alone in fp32 (``Qwen3_5Experts.forward``, qwen3_5.py:815-841):
    ``sum_j w[t,j] * down_e(silu(gate_e x) * up_e x)`` over the slots whose expert id lies
    in ``[expert_base, expert_base + len(gate_up))``."""
    xf = x.float()
    T = ids.shape[0]
    out = torch.zeros(T, down.shape[1], dtype=torch.float32, device=xf.device)
    ids = ids.long()
    for e in torch.unique(ids).tolist():
        le = e - expert_base
        if le < 0 or le >= gate_up.shape[0]:
            continue
        tok, pos = torch.where(ids == e)
        g, u = (xf[tok] @ gate_up[le].float().t()).chunk(2, dim=-1)
        y = (F.silu(g) * u) @ down[le].float().t()
        out.index_add_(0, tok, y * w[tok, pos, None].float())
    return out


def shared_expert_fp32(x, sh_gate, sh_up, sh_down):
    """``Qwen3_5SharedExpertMLP.forward`` (qwen3_5.py:916-917) in fp32, ungated."""
    xf = x.float()
    return (F.silu(xf @ sh_gate.float().t()) * (xf @ sh_up.float().t())) @ sh_down.float().t()


def moe_block_fp32(x, p, ids, w):
    """The block in fp32 for a fixed routing (ids [T,k], w [T,k] fp32).  Returns fp32.

    Plain torch, so it runs wherever its inputs live: the tests also evaluate it on the
    GPU (fp32 matmuls, TF32 off) to check full-size launches row by row."""
    xf = x.float()
    T, k = ids.shape
    out = torch.zeros(T, p.hidden, dtype=torch.float32, device=xf.device)
    ids = ids.long()
    for e in torch.unique(ids).tolist():
        tok, pos = torch.where(ids == e)
        gu = p.gate_up[e].float()
        y = xf[tok] @ gu.t()
        g, u = y.chunk(2, dim=-1)
        h = F.silu(g) * u
        y = h @ p.down[e].float().t()
        out.index_add_(0, tok, y * w[tok, pos, None].float())
    s = F.silu(xf @ p.sh_gate.float().t()) * (xf @ p.sh_up.float().t())
    s = s @ p.sh_down.float().t()
    sg = torch.sigmoid(xf @ p.sh_gate_w.float().t())
    return out + sg * s


def rel_err(y, ref) -> float:
    """``max|y - ref| / max|ref|`` in fp32."""
    y = y.float()
    ref = ref.float()
    return float((y - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
