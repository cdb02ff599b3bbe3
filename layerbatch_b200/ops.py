"""Thin torch-facing wrappers over the C ABI (``include/layerbatch_b200.h``).

Tensors are passed by pointer; every call is stream-ordered on the current torch stream,
allocates nothing inside the library and is CUDA-graph capturable once its workspace has
been sized (workspaces are cached per device and grown on demand outside capture).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import LbMoeArgs, LbPodArgs, LbPrologueArgs, check, lib, ptr, stream_ptr

_WS: dict = {}


def workspace(nbytes: int, device, tag: str = "default") -> torch.Tensor:
    """A cached uint8 workspace of at least ``nbytes`` bytes (256-byte header zeroed)."""
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), tag)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("workspace must be sized before CUDA-graph capture")
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _WS[key] = buf
    return buf


def launch_count() -> int:
    """Kernels launched by the CUDA library so far in this process."""
    return int(lib().lb_kernel_launch_count())


def _events(a, events):
    """Attach up to four recorded torch.cuda.Event handles to an args struct."""
    if events:
        for i, e in enumerate(events[:4]):
            if e is not None:
                if not e.cuda_event:
                    e.record()  # creates the underlying CUDA event
                a.timing_events[i] = e.cuda_event


def device_status(ws: torch.Tensor, clear: bool = True) -> int:
    v = C.c_int(0)
    check(lib().lb_read_device_status(ws.data_ptr(), int(clear), C.byref(v)),
          "lb_read_device_status")
    return v.value


def _bf16_2d(t, name):
    if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D bf16 tensor with a contiguous last dim")


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
         accumulate_fp32: bool = False, splits: int = 1) -> torch.Tensor:
    """``out = a @ b.T`` (bf16) or ``out += a @ b.T`` (fp32 ``out``, split-K allowed)."""
    _bf16_2d(a, "a")
    _bf16_2d(b, "b")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = (torch.zeros if accumulate_fp32 else torch.empty)(
            M, N, dtype=torch.float32 if accumulate_fp32 else torch.bfloat16, device=a.device)
    ws = workspace(256, a.device, "gemm")
    rc = lib().lb_gemm_bf16(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(),
                            out.stride(0), M, N, K, int(accumulate_fp32), splits, ws.data_ptr(),
                            stream_ptr())
    check(rc, "lb_gemm_bf16")
    return out


def router_topk(logits: torch.Tensor, k: int):
    """Top-k of softmax(logits) with lowest-index ties; returns (ids i32, w f32, w bf16)."""
    _bf16_2d(logits, "logits")
    T, E = logits.shape
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    wf = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    wb = torch.empty(T, k, dtype=torch.bfloat16, device=logits.device)
    check(lib().lb_router_topk(logits.data_ptr(), logits.stride(0), T, E, k, ids.data_ptr(),
                               wf.data_ptr(), wb.data_ptr(), stream_ptr()), "lb_router_topk")
    return ids, wf, wb


def moe_permute(ids: torch.Tensor, expert_base: int, num_local_experts: int):
    """Expert-major permutation; returns (row_start [G+1], perm_token [T+T*k], row_of [T,k])."""
    T, k = ids.shape
    ids = ids.to(torch.int32).contiguous()
    G = num_local_experts + 1
    dev = ids.device
    row_start = torch.empty(G + 1, dtype=torch.int32, device=dev)
    perm_token = torch.full((T + T * k,), -1, dtype=torch.int32, device=dev)
    row_of = torch.empty(T, k, dtype=torch.int32, device=dev)
    nbytes = lib().lb_moe_permute_workspace_size(T, k, num_local_experts)
    ws = workspace(nbytes, dev, "permute")
    check(lib().lb_moe_permute(ids.data_ptr(), T, k, expert_base, num_local_experts,
                               row_start.data_ptr(), perm_token.data_ptr(), row_of.data_ptr(),
                               ws.data_ptr(), ws.numel(), stream_ptr()), "lb_moe_permute")
    return row_start, perm_token, row_of


def moe_forward(x, router, gate_up, down, sh_gate, sh_up, sh_down, sh_gate_w, top_k,
                out=None, expert_base=0, return_routing=False, ws_tag="moe", events=None,
                topk_ids=None, topk_weights=None, pair_rows=None, pair_index=None,
                num_experts=None):
    """The MoE block (router -> experts -> shared expert -> combine) on the GPU.

    Expert-parallel building blocks (all optional):
    * ``topk_ids`` [T,k] int32 global expert ids and ``topk_weights`` [T,k] fp32 given:
      the router is skipped (``router`` may be None; pass ``num_experts``);
    * ``sh_gate=None``: no shared expert;
    * ``gate_up``/``down`` with 0 local experts (shape [0, ...]) or None: no routed compute;
    * ``pair_rows`` [*, H] bf16 + ``pair_index`` [T, k] int32: rows computed elsewhere that
      the combine adds into ``out[t]`` (-1 = none).
    """
    T, H = x.shape
    given = topk_ids is not None
    E = num_experts if num_experts is not None else router.shape[0]
    nl = 0 if gate_up is None else gate_up.shape[0]
    I = (down.shape[2] if down is not None and nl else sh_down.shape[1])
    shared = sh_gate is not None
    if out is None:
        out = torch.empty_like(x)
    for name, t in (("x", x), ("router", router), ("gate_up", gate_up), ("down", down),
                    ("sh_gate", sh_gate), ("sh_up", sh_up), ("sh_down", sh_down),
                    ("sh_gate_w", sh_gate_w), ("out", out), ("pair_rows", pair_rows)):
        if t is None:
            continue
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError(f"{name} must be a contiguous CUDA bf16 tensor")
    logits = ids = wb = None
    if return_routing and not given:
        logits = torch.empty(T, E, dtype=torch.bfloat16, device=x.device)
        ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
        wb = torch.empty(T, top_k, dtype=torch.bfloat16, device=x.device)
    if given:
        ids = topk_ids.to(torch.int32).contiguous()
        topk_weights = topk_weights.to(torch.float32).contiguous()
    if pair_index is not None:
        pair_index = pair_index.to(torch.int32).contiguous()
    a = LbMoeArgs(num_tokens=T, hidden=H, num_experts=E, top_k=top_k, inter=I,
                  shared_inter=sh_gate.shape[0] if shared else 0, expert_base=expert_base,
                  num_local_experts=nl, x=x.data_ptr(), w_router=ptr(router),
                  w_gate_up=ptr(gate_up) if nl else None, w_down=ptr(down) if nl else None,
                  w_shared_gate=ptr(sh_gate), w_shared_up=ptr(sh_up), w_shared_down=ptr(sh_down),
                  w_shared_expert_gate=ptr(sh_gate_w), out=out.data_ptr(),
                  router_logits=ptr(logits), topk_ids=ptr(ids), topk_weights=ptr(wb),
                  routing_given=int(given), topk_weights_f32=ptr(topk_weights),
                  no_shared=int(not shared), pair_rows=ptr(pair_rows), pair_index=ptr(pair_index))
    _events(a, events)
    need = C.c_size_t(0)
    check(lib().lb_moe_workspace_size(C.byref(a), C.byref(need)), "lb_moe_workspace_size")
    ws = workspace(need.value, x.device, ws_tag)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    check(lib().lb_moe_forward(C.byref(a), stream_ptr()), "lb_moe_forward")
    if return_routing and not given:
        return out, logits, ids, wb
    return out


def store_kvcache(k, v, k_cache, v_cache, slot_mapping):
    """``k_cache/v_cache[slot] = k/v`` for slot != -1 (reference attention.py:71-80)."""
    N = k.shape[0]
    row = k_cache.shape[-2] * k_cache.shape[-1]
    if k.stride(-1) != 1 or k.stride(-2) != k.shape[-1] or v.stride(-2) != v.shape[-1]:
        raise ValueError("k/v heads must be packed ([N, Hkv, D] with D contiguous)")
    slots = k_cache.numel() // row
    sm = slot_mapping.to(torch.int32)
    check(lib().lb_store_kvcache(k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                 k_cache.data_ptr(), v_cache.data_ptr(), sm.data_ptr(), N, slots,
                                 row, stream_ptr()), "lb_store_kvcache")


def prologue_args(q_in, k_in, v_in, q_norm_w, k_norm_w, cos_sin_cache, positions,
                  slot_mapping, k_cache, v_cache, eps, q_out, status=None):
    """``LbPrologueArgs`` of one prologue call, and the tensors it points to (keep them
    alive until the call is enqueued)."""
    N, Hq, D = q_in.shape
    Hkv = k_in.shape[1]
    for t, name in ((k_in, "k_in"), (v_in, "v_in")):
        if t.stride(-1) != 1 or t.stride(-2) != D:
            raise ValueError(f"{name} must be [N, Hkv, D] with packed heads")
    if q_in.stride(-1) != 1:
        raise ValueError("q_in must have a contiguous last dim")
    cs = cos_sin_cache.reshape(cos_sin_cache.shape[0], -1)
    if cs.dtype != torch.float32 or not cs.is_contiguous():
        raise ValueError("cos_sin_cache must be a contiguous fp32 [max_position, rotary_dim]")
    pos = positions.to(torch.int64)
    sm = slot_mapping.to(torch.int32)
    row = k_cache.shape[-2] * k_cache.shape[-1]
    a = LbPrologueArgs(
        num_tokens=N, num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, rotary_dim=cs.shape[1],
        eps=float(eps), q_in=q_in.data_ptr(), q_in_stride_tok=q_in.stride(0),
        q_in_stride_head=q_in.stride(1), k_in=k_in.data_ptr(), k_in_stride_tok=k_in.stride(0),
        v_in=v_in.data_ptr(), v_in_stride_tok=v_in.stride(0), q_norm_w=q_norm_w.data_ptr(),
        k_norm_w=k_norm_w.data_ptr(), cos_sin_cache=cs.data_ptr(), max_position=cs.shape[0],
        positions=pos.data_ptr(), slot_mapping=sm.data_ptr(), k_cache=k_cache.data_ptr(),
        v_cache=v_cache.data_ptr(), num_slots=k_cache.numel() // row, q_out=q_out.data_ptr(),
        q_out_stride_tok=q_out.stride(0), q_out_stride_head=q_out.stride(1),
        status=ptr(status))
    return a, (cs, pos, sm)


def attn_prologue(q_in, k_in, v_in, q_norm_w, k_norm_w, cos_sin_cache, positions, slot_mapping,
                  k_cache, v_cache, eps, q_out=None, status=None):
    """Fused (1+w) RMSNorm + partial RoPE of query and key, and the K/V cache store
    (reference qwen3_5.py:730-736 and attention.py:50-80).

    ``q_in [N, Hq, D]`` may be a strided view (the query half of q_proj's output);
    ``k_in``/``v_in`` are ``[N, Hkv, D]`` with packed heads; ``cos_sin_cache`` is the
    rotary module's fp32 ``[max_position, (1,) rotary_dim]`` buffer.  Returns ``q_out``
    ``[N, Hq, D]`` (allocated when not given).
    """
    N, Hq, D = q_in.shape
    if q_out is None:
        q_out = torch.empty(N, Hq, D, dtype=q_in.dtype, device=q_in.device)
    a, keep = prologue_args(q_in, k_in, v_in, q_norm_w, k_norm_w, cos_sin_cache, positions,
                            slot_mapping, k_cache, v_cache, eps, q_out, status)
    check(lib().lb_attn_prologue(C.byref(a), stream_ptr()), "lb_attn_prologue")
    del keep
    return q_out


def gated_attention_layer(x, w_qkv, num_heads, num_kv_heads, q_norm_w, k_norm_w,
                          cos_sin_cache, eps, positions, slot_mapping, k_cache, v_cache,
                          block_tables, context_lens, cu_seqlens_q, w_o, scale, out=None,
                          max_q_len=None, work_hint=None, events=None, qkv=None, q=None,
                          attn_out=None, ws_tag="pod", tp=None, tp_phases=0,
                          stage_events=None, fuse_prologue=False, prologue="gemm"):
    """The whole gated full-attention layer from its hidden states
    (``Qwen3_5FullAttention.forward``, nanovllm/models/qwen3_5.py:705-746):

    1. one GEMM for the three projections: ``qkv = x @ w_qkv.T`` with ``w_qkv`` =
       ``[q_proj.weight; k_proj.weight; v_proj.weight]`` (``[Hq*2D + 2*Hkv*D, H]``);
    2. the prologue: (1+w) RMSNorm and partial RoPE of query and key, the K/V of the new
       tokens stored into the paged cache at ``slot_mapping``;
    3. ``lb_pod_attn_oproj``: attention over the cache for every sequence of the batch,
       ``* sigmoid(gate)`` (the gate read in place from q_proj's output) and o_proj.

    Where step 2 runs (``prologue``), all giving the same bits:
    ``"gemm"`` (default; head_dim 256 with rotary_dim 64, else "kernel"): in the epilogue
    of the projection GEMM (``lb_qkv_prologue_gemm``), so only the gate columns of
    ``qkv`` are written; ``"kernel"``: its own ``lb_attn_prologue`` launch after the
    GEMM; ``"pod"`` (or ``fuse_prologue=True``): inside the attention kernel of step 3
    (``LbPodArgs.prologue``: the kernel's CTAs first do the prologue rows, each attention
    item waits for its own sequence's rows).

    ``qkv`` ``[N, Hq*2D + 2*Hkv*D]`` and ``q`` ``[N, Hq, D]`` may be given as preallocated
    buffers (CUDA-graph capture); ``attn_out`` ``[N, Hq*D]`` optionally receives the
    attention output before the gate.  The prologue reports bad positions or slots in the
    status word of the workspace tagged ``ws_tag + "_prologue"``.  ``stage_events`` (up to
    two ``torch.cuda.Event``) are recorded after the GEMM and after the prologue.
    """
    N = x.shape[0]
    Hq, Hkv = num_heads, num_kv_heads
    D = k_cache.shape[-1]
    if w_qkv.shape[0] != Hq * 2 * D + 2 * Hkv * D:
        raise ValueError("w_qkv must stack q_proj [Hq*2D], k_proj [Hkv*D] and v_proj [Hkv*D] rows")
    stage_events = list(stage_events or []) + [None, None]
    if fuse_prologue:
        prologue = "pod"
    if prologue not in ("gemm", "kernel", "pod"):
        raise ValueError("prologue must be 'gemm', 'kernel' or 'pod'")
    rot = cos_sin_cache.reshape(cos_sin_cache.shape[0], -1).shape[1]
    if prologue == "gemm" and (D != 256 or rot != 64):
        prologue = "kernel"
    _bf16_2d(x, "x")
    _bf16_2d(w_qkv, "w_qkv")
    if qkv is None:
        qkv = torch.empty(N, w_qkv.shape[0], dtype=torch.bfloat16, device=x.device)
    q3 = qkv[:, :Hq * 2 * D].view(N, Hq, 2 * D)
    k_in = qkv[:, Hq * 2 * D:Hq * 2 * D + Hkv * D].view(N, Hkv, D)
    v_in = qkv[:, Hq * 2 * D + Hkv * D:].view(N, Hkv, D)
    status = workspace(256, x.device, ws_tag + "_prologue").view(torch.int32)[:1]
    if q is None:
        q = torch.empty(N, Hq, D, dtype=x.dtype, device=x.device)
    pro = None
    if prologue == "gemm":
        a, keep = prologue_args(q3[..., :D], k_in, v_in, q_norm_w, k_norm_w, cos_sin_cache,
                                positions, slot_mapping, k_cache, v_cache, eps, q, status)
        ws = workspace(256, x.device, "gemm")
        check(lib().lb_qkv_prologue_gemm(x.data_ptr(), x.stride(0), w_qkv.data_ptr(),
                                         w_qkv.stride(0), qkv.data_ptr(), qkv.stride(0),
                                         x.shape[1], C.byref(a), ws.data_ptr(), stream_ptr()),
              "lb_qkv_prologue_gemm")
        del keep
        for e in stage_events[:2]:
            if e is not None:
                e.record()
    else:
        gemm(x, w_qkv, out=qkv)
        if stage_events[0] is not None:
            stage_events[0].record()
        if prologue == "pod":
            pro, keep = prologue_args(q3[..., :D], k_in, v_in, q_norm_w, k_norm_w,
                                      cos_sin_cache, positions, slot_mapping, k_cache, v_cache,
                                      eps, q, status)
        else:
            attn_prologue(q3[..., :D], k_in, v_in, q_norm_w, k_norm_w, cos_sin_cache, positions,
                          slot_mapping, k_cache, v_cache, eps, q_out=q, status=status)
        if stage_events[1] is not None:
            stage_events[1].record()
    return pod_attn_oproj(q, q3[..., D:], k_cache, v_cache, block_tables, context_lens,
                          cu_seqlens_q, w_o, scale, out=out, attn_out=attn_out,
                          max_q_len=max_q_len, ws_tag=ws_tag, events=events,
                          work_hint=work_hint, tp=tp, tp_phases=tp_phases, prologue=pro)


def pod_args(q, gate, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, w_o, scale,
             out, attn_out=None, max_q_len=None, kv_split_pages=0) -> LbPodArgs:
    N, Hq, D = q.shape
    B = context_lens.numel()
    nb, ps, Hkv, _ = k_cache.shape
    if max_q_len is None:
        max_q_len = N
    return LbPodArgs(
        num_seqs=B, num_tokens=N, max_q_len=max_q_len, num_q_heads=Hq, num_kv_heads=Hkv,
        head_dim=D, page_size=ps, num_pages=nb, max_pages_per_seq=block_tables.shape[1],
        hidden=w_o.shape[0] if w_o is not None else 0, sm_scale=float(scale),
        kv_split_pages=kv_split_pages,
        q=q.data_ptr(), q_stride_tok=q.stride(0), q_stride_head=q.stride(1),
        gate=ptr(gate), gate_stride_tok=gate.stride(0) if gate is not None else 0,
        gate_stride_head=gate.stride(1) if gate is not None else 0,
        k_cache=k_cache.data_ptr(), v_cache=v_cache.data_ptr(),
        block_tables=block_tables.data_ptr(), context_lens=context_lens.data_ptr(),
        cu_seqlens_q=cu_seqlens_q.data_ptr(), w_o=ptr(w_o), attn_out=ptr(attn_out),
        out=ptr(out), out_fp32=int(out is not None and out.dtype == torch.float32))


def pod_work_hint(ctx_list, qlen_list):
    """(prefill query-key pairs, decode context tokens) of a batch, from host lists."""
    pairs = sum(L * (c - L) + L * (L + 1) // 2 for c, L in zip(ctx_list, qlen_list) if L > 1)
    dec = sum(c for c, L in zip(ctx_list, qlen_list) if L == 1)
    return pairs, dec


def pod_attn_oproj(q, gate, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, w_o,
                   scale, out=None, attn_out=None, max_q_len=None, kv_split_pages=0,
                   ws_tag="pod", events=None, work_hint=None, tp=None, tp_phases=0,
                   prologue=None):
    """Fused paged attention (prefill + decode mixed) -> sigmoid gate -> o_proj.

    ``gate`` may be None (no output gate).  With ``w_o=None`` only the attention runs and
    ``attn_out`` [N, Hq*D] receives it; the function then returns ``attn_out``.
    ``out`` may be fp32 to receive the o_proj partial sums unrounded (tensor parallel).
    ``tp`` (an ``engine.peer.TPExchange``): this rank holds a head slice and W_o's matching
    columns; the o_proj partials are reduced over the group through peer memory inside
    the call and ``out`` (bf16) receives the all-reduced result.
    ``prologue`` (an ``LbPrologueArgs`` from ``prologue_args`` whose ``q_out`` is ``q``): the
    prologue of the call's tokens runs inside the attention kernel.
    """
    N, Hq, D = q.shape
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != torch.bfloat16 or not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA bf16 tensor")
    if w_o is None:
        if attn_out is None:
            attn_out = torch.empty(N, Hq * D, dtype=torch.bfloat16, device=q.device)
    elif out is None:
        out = torch.empty(N, w_o.shape[0], dtype=torch.bfloat16, device=q.device)
    bt = block_tables.to(torch.int32)
    cl = context_lens.to(torch.int32)
    cu = cu_seqlens_q.to(torch.int32)
    a = pod_args(q, gate, k_cache, v_cache, bt, cl, cu, w_o, scale, out, attn_out, max_q_len,
                 kv_split_pages)
    if work_hint is not None:
        a.prefill_pairs_hint, a.decode_tokens_hint = int(work_hint[0]), int(work_hint[1])
    if tp is not None and tp.world > 1:
        a.tp_rank, a.tp_size, a.tp_capacity = tp.rank, tp.world, tp.capacity
        for r, p in enumerate(tp.peers):
            a.tp_bufs[r] = p
        a.tp_phases = tp_phases
    _events(a, events)
    if prologue is not None:
        a.prologue = C.pointer(prologue)
    need = C.c_size_t(0)
    check(lib().lb_pod_workspace_size(C.byref(a), C.byref(need)), "lb_pod_workspace_size")
    ws = workspace(need.value, q.device, ws_tag)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    check(lib().lb_pod_attn_oproj(C.byref(a), stream_ptr()), "lb_pod_attn_oproj")
    return out if w_o is not None else attn_out
