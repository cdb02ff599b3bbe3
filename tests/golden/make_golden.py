"""Generate golden vectors by running the REFERENCE's own torch modules on the CPU.

Run in a container where the reference project is importable (its path is given by
``--ref`` or ``LB_REFERENCE_PATH``).  Inputs are not stored: they are regenerated from
seeds by ``layerbatch_b200.workloads`` and a SHA-256 of their bytes is stored beside the
outputs so that a test can tell a regeneration mismatch from a numerical one.

Reference entry points exercised:
* ``Qwen3_5SparseMoeBlock.forward`` (nanovllm/models/qwen3_5.py:899-905) on its prefill
  (sparse, :815-841) and decode (dense, :843-874) paths, selected through
  ``set_context(is_prefill)`` (nanovllm/utils/context.py:37-45);
* ``Qwen3_5TopKRouter.forward`` (qwen3_5.py:767-774);
* ``sdpa_decode_paged`` and ``sdpa_prefill_varlen`` (nanovllm/layers/sdpa_fallback.py);
* the output gate and o_proj of ``Qwen3_5FullAttention.forward`` (qwen3_5.py:742-746)
  through the reference's ``RowParallelLinear`` (nanovllm/layers/linear.py:138-159);
* the attention prologue of ``Qwen3_5FullAttention.forward`` (qwen3_5.py:707-736): the
  (query, gate) split, ``Qwen3_5RMSNorm`` on query and key (qwen3_5.py:39-55) and
  ``RotaryEmbedding`` (partial, theta 1e7, nanovllm/layers/rotary_embedding.py:17-54),
  called uncompiled through ``RotaryEmbedding.forward.__wrapped__``.

Usage: ``python tests/golden/make_golden.py --ref <reference checkout>``
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from layerbatch_b200 import workloads as W  # noqa: E402

MOE_CASES = {
    # name: (T, H, E, I, Is, k, zipf)
    "moe_small": (16, 256, 8, 64, 64, 2, False),
    "moe_c0": (64, 2048, 64, 512, 512, 8, False),
    "moe_e512_t32": (32, 2048, 512, 512, 512, 10, True),
}

DECODE_CASES = {
    # name: decode ctx list
    "decode_edges": [1, 255, 256, 257, 700, 1024],
    "decode_c1_like": [512, 4096, 1777, 2900],
}

PREFILL_CASES = {
    # name: list of (prefix, chunk) -- no prefix so Sq == Sk (alignment-independent)
    "prefill_noprefix": [(0, 33), (0, 70)],
}


def sha(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def moe_inputs(T, H, E, I, Is, k, zipf):
    p = W.make_moe_params(H, E, I, Is, k, seed=0)
    x = W.make_moe_input(T, H, seed=1)
    if zipf:
        W.apply_zipf_bias(p, x)
    return p, x


def tie_inputs():
    """Router logits with many exact ties: integer-valued x and weights in {-1,0,1}/8."""
    T, H, E, k = 32, 64, 16, 4
    g = torch.Generator().manual_seed(5)
    x = torch.randint(-2, 3, (T, H), generator=g).to(torch.bfloat16)
    w = (torch.randint(-1, 2, (E, H), generator=g).float() / 8).to(torch.bfloat16)
    return x, w, k


PROLOGUE_CASES = {
    # name: (N, Hq, Hkv, D, rotary_dim, max_position, theta, positions seed)
    "prologue_small": (7, 16, 2, 256, 64, 40000, 1.0e7, 11),
}


def prologue_inputs(N, Hq, Hkv, D, max_pos, seed):
    g = torch.Generator().manual_seed(seed)
    q_out = torch.randn(N, Hq * 2 * D, generator=g).to(torch.bfloat16)
    k_raw = (3.0 * torch.randn(N, Hkv * D, generator=g)).to(torch.bfloat16)
    v_raw = torch.randn(N, Hkv * D, generator=g).to(torch.bfloat16)
    q_w = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    k_w = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (N,), generator=g, dtype=torch.long)
    pos[0], pos[1] = 0, max_pos - 1
    return q_out, k_raw, v_raw, q_w, k_w, pos


def prologue_goldens(out):
    from nanovllm.models.qwen3_5 import Qwen3_5RMSNorm
    from nanovllm.layers.rotary_embedding import RotaryEmbedding
    for name, (N, Hq, Hkv, D, rot, max_pos, theta, seed) in PROLOGUE_CASES.items():
        q_out, k_raw, v_raw, q_w, k_w, pos = prologue_inputs(N, Hq, Hkv, D, max_pos, seed)
        qn = Qwen3_5RMSNorm(D, eps=1e-6).to(torch.bfloat16)
        kn = Qwen3_5RMSNorm(D, eps=1e-6).to(torch.bfloat16)
        rope = RotaryEmbedding(D, rot, max_pos, theta)
        with torch.no_grad():
            qn.weight.copy_(q_w)
            kn.weight.copy_(k_w)
            query, gate = q_out.view(N, Hq, 2 * D).chunk(2, dim=-1)
            gate = gate.reshape(N, Hq * D)
            k = k_raw.view(N, Hkv, D)
            query = qn(query)
            k = kn(k)
            query, k = RotaryEmbedding.forward.__wrapped__(rope, pos, query, k)
        out[name] = dict(shape=(N, Hq, Hkv, D, rot, max_pos, theta, seed), query=query,
                         gate=gate, key=k, cos_sin_rows=rope.cos_sin_cache[pos].clone(),
                         in_sha=sha(q_out, k_raw, v_raw, q_w, k_w, pos))
        print(name, "done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LB_REFERENCE_PATH", ""))
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default="", help="regenerate only these cases "
                    "(comma list of prefixes; others are kept from the existing file)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        sys.exit("pass --ref <path to the reference project>")
    sys.path.insert(0, args.ref)
    if args.only:
        path = os.path.join(args.out, "golden.pt")
        out = torch.load(path, weights_only=False)
        if "prologue" in args.only:
            prologue_goldens(out)
        for rec in out.values():
            if isinstance(rec, dict):
                for key, val in rec.items():
                    if torch.is_tensor(val):
                        rec[key] = val.detach().clone().contiguous()
        torch.save(out, path)
        print("updated", path, os.path.getsize(path), "bytes")
        return
    import torch.distributed as dist
    from nanovllm.models.qwen3_5 import Qwen3_5SparseMoeBlock, Qwen3_5TopKRouter
    from nanovllm.layers.sdpa_fallback import sdpa_decode_paged, sdpa_prefill_varlen
    from nanovllm.layers.linear import RowParallelLinear
    from nanovllm.utils.context import set_context, reset_context

    torch.manual_seed(0)
    out = {"torch_version": str(torch.__version__)}

    # ---------------- MoE blocks
    for name, (T, H, E, I, Is, k, zipf) in MOE_CASES.items():
        p, x = moe_inputs(T, H, E, I, Is, k, zipf)
        blk = Qwen3_5SparseMoeBlock(H, E, k, I, Is).to(torch.bfloat16)
        with torch.no_grad():
            blk.gate.weight.copy_(p.router)
            blk.experts.gate_up_proj.copy_(p.gate_up)
            blk.experts.down_proj.copy_(p.down)
            blk.shared_expert.gate_proj.weight.copy_(p.sh_gate)
            blk.shared_expert.up_proj.weight.copy_(p.sh_up)
            blk.shared_expert.down_proj.weight.copy_(p.sh_down)
            blk.shared_expert_gate.weight.copy_(p.sh_gate_w)
            logits = torch.nn.functional.linear(x, blk.gate.weight)
            tw, ti = blk.gate(x)
            set_context(True)
            y_sparse = blk(x)
            set_context(False)
            y_dense = blk(x) if T * k <= 1024 else None
            reset_context()
        rec = dict(shape=(T, H, E, I, Is, k, zipf), x_sha=sha(x),
                   w_sha=sha(p.router, p.gate_up, p.down, p.sh_gate, p.sh_up, p.sh_down,
                             p.sh_gate_w),
                   logits=logits, topk_w=tw, topk_ids=ti, y_sparse=y_sparse)
        if y_dense is not None:
            rec["y_dense"] = y_dense
        out[name] = rec
        print(name, "done")

    # ---------------- router ties
    x, w, k = tie_inputs()
    r = Qwen3_5TopKRouter(w.shape[0], w.shape[1], k).to(torch.bfloat16)
    with torch.no_grad():
        r.weight.copy_(w)
        tw, ti = r(x)
    out["router_ties"] = dict(logits=torch.nn.functional.linear(x, w), topk_w=tw, topk_ids=ti,
                              x_sha=sha(x), w_sha=sha(w), k=k)

    # ---------------- paged decode attention + gate + o_proj (tp=1)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("gloo", rank=0, world_size=1)
    for name, ctx in DECODE_CASES.items():
        b = W.make_attn_batch(ctx, (), seed=3)
        o = sdpa_decode_paged(b.q, b.k_cache, b.v_cache, b.block_tables, b.context_lens,
                              b.scale, block_size=W.BLOCK_SIZE)
        o_flat = o.flatten(1, -1)
        g_flat = b.gate.reshape(b.num_tokens, -1)
        lin = RowParallelLinear(b.w_o.shape[1], b.w_o.shape[0]).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(b.w_o)
            y = lin(o_flat * torch.sigmoid(g_flat))
        out[name] = dict(ctx=ctx, attn=o, y=y,
                         in_sha=sha(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.w_o))
        print(name, "done")

    for name, pf in PREFILL_CASES.items():
        b = W.make_attn_batch([], pf, seed=4)
        cu_k = b.cu_seqlens_q.clone()
        o = sdpa_prefill_varlen(b.q, None, None, b.cu_seqlens_q, cu_k, b.scale,
                                block_tables=b.block_tables, k_cache=b.k_cache,
                                v_cache=b.v_cache, block_size=W.BLOCK_SIZE)
        out[name] = dict(prefill=pf, attn=o,
                         in_sha=sha(b.q, b.gate, b.k_cache, b.v_cache, b.block_tables, b.w_o))
        print(name, "done")

    prologue_goldens(out)

    dist.destroy_process_group()
    for rec in out.values():
        if isinstance(rec, dict):
            for key, val in rec.items():
                if torch.is_tensor(val):
                    rec[key] = val.detach().clone().contiguous()
    path = os.path.join(args.out, "golden.pt")
    torch.save(out, path)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
