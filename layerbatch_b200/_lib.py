"""ctypes binding of ``liblb_b200.so`` (declared in ``include/layerbatch_b200.h``).

The library is the only compute path: if it is missing or no CUDA device is present,
``lib()`` raises; nothing falls back to PyTorch or the CPU.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblb_b200.so")

LB_OK = 0
ERRORS = {1: "invalid argument", 2: "unsupported", 3: "workspace", 4: "CUDA error",
          5: "device status"}

# Every symbol the header declares (checked by the CPU test suite).
EXPORTS = [
    "lb_get_last_error_string", "lb_version", "lb_kernel_launch_count", "lb_device_info",
    "lb_read_device_status",
    "lb_gemm_workspace_size", "lb_gemm_bf16", "lb_router_topk",
    "lb_moe_permute_workspace_size", "lb_moe_permute", "lb_moe_permute_noalloc",
    "lb_moe_workspace_size",
    "lb_moe_forward", "lb_ep_buffer_size", "lb_ep_buffer_alloc", "lb_ep_buffer_open",
    "lb_ep_buffer_close", "lb_ep_buffer_free", "lb_ep_workspace_size", "lb_ep_moe_forward",
    "lb_store_kvcache", "lb_attn_prologue", "lb_qkv_prologue_gemm", "lb_tp_buffer_size",
    "lb_pod_workspace_size",
    "lb_pod_attn_oproj",
]

LB_EP_MAX_RANKS = 8
LB_EP_IPC_HANDLE_BYTES = 64
LB_EP_PHASE_DISPATCH, LB_EP_PHASE_EXPERTS, LB_EP_PHASE_COMBINE = 1, 2, 4
LB_TP_PHASE_ATTN, LB_TP_PHASE_REDUCE, LB_TP_PHASE_GATHER = 1, 2, 4

vp = C.c_void_p
i64 = C.c_int64
i32 = C.c_int32


class LbMoeArgs(C.Structure):
    _fields_ = [
        ("num_tokens", i64), ("hidden", i64), ("num_experts", i64), ("top_k", i64),
        ("inter", i64), ("shared_inter", i64), ("expert_base", i64),
        ("num_local_experts", i64),
        ("x", vp), ("w_router", vp), ("w_gate_up", vp), ("w_down", vp),
        ("w_shared_gate", vp), ("w_shared_up", vp), ("w_shared_down", vp),
        ("w_shared_expert_gate", vp), ("out", vp), ("router_logits", vp),
        ("topk_ids", vp), ("topk_weights", vp), ("workspace", vp),
        ("workspace_bytes", C.c_size_t), ("timing_events", vp * 4),
        ("routing_given", i32), ("topk_weights_f32", vp), ("no_shared", i32),
        ("pair_rows", vp), ("pair_index", vp),
    ]


class LbEpArgs(C.Structure):
    _fields_ = [
        ("num_tokens", i64), ("capacity", i64), ("hidden", i64), ("num_experts", i64),
        ("top_k", i64), ("inter", i64), ("rank", i32), ("world", i32),
        ("x", vp), ("w_router", vp), ("w_gate_up", vp), ("w_down", vp),
        ("w_shared_gate", vp), ("w_shared_up", vp), ("w_shared_down", vp),
        ("w_shared_expert_gate", vp), ("out", vp), ("peer_bufs", vp * LB_EP_MAX_RANKS),
        ("workspace", vp), ("workspace_bytes", C.c_size_t), ("phases", i32),
        ("timing_events", vp * 4), ("expert_slot", vp),
    ]


class LbPrologueArgs(C.Structure):
    _fields_ = [
        ("num_tokens", i64), ("num_q_heads", i64), ("num_kv_heads", i64), ("head_dim", i64),
        ("rotary_dim", i64), ("eps", C.c_float),
        ("q_in", vp), ("q_in_stride_tok", i64), ("q_in_stride_head", i64),
        ("k_in", vp), ("k_in_stride_tok", i64), ("v_in", vp), ("v_in_stride_tok", i64),
        ("q_norm_w", vp), ("k_norm_w", vp), ("cos_sin_cache", vp), ("max_position", i64),
        ("positions", vp), ("slot_mapping", vp), ("k_cache", vp), ("v_cache", vp),
        ("num_slots", i64), ("q_out", vp), ("q_out_stride_tok", i64),
        ("q_out_stride_head", i64), ("status", vp),
    ]


class LbPodArgs(C.Structure):
    _fields_ = [
        ("num_seqs", i64), ("num_tokens", i64), ("max_q_len", i64), ("num_q_heads", i64),
        ("num_kv_heads", i64), ("head_dim", i64), ("page_size", i64), ("num_pages", i64),
        ("max_pages_per_seq", i64), ("hidden", i64), ("sm_scale", C.c_float),
        ("kv_split_pages", i32),
        ("q", vp), ("q_stride_tok", i64), ("q_stride_head", i64),
        ("gate", vp), ("gate_stride_tok", i64), ("gate_stride_head", i64),
        ("k_cache", vp), ("v_cache", vp), ("block_tables", vp), ("context_lens", vp),
        ("cu_seqlens_q", vp), ("w_o", vp), ("attn_out", vp), ("out", vp),
        ("out_fp32", i32), ("workspace", vp), ("workspace_bytes", C.c_size_t),
        ("timing_events", vp * 4), ("prefill_pairs_hint", i64), ("decode_tokens_hint", i64),
        ("tp_rank", i32), ("tp_size", i32), ("tp_capacity", i64),
        ("tp_bufs", vp * LB_EP_MAX_RANKS), ("tp_phases", i32),
        ("prologue", C.POINTER(LbPrologueArgs)),
    ]


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the shared library without touching the GPU (used by CPU symbol tests)."""
    if not os.path.exists(path):
        raise RuntimeError(f"layerbatch_b200 CUDA library not built: {path} is missing "
                           "(run `python -m layerbatch_b200.build`)")
    L = C.CDLL(path)
    L.lb_get_last_error_string.restype = C.c_char_p
    L.lb_gemm_workspace_size.restype = C.c_size_t
    L.lb_kernel_launch_count.restype = C.c_ulonglong
    L.lb_moe_permute_workspace_size.restype = C.c_size_t
    L.lb_moe_permute_workspace_size.argtypes = [i64, i64, i64]
    L.lb_gemm_bf16.argtypes = [vp, i64, vp, i64, vp, i64, i64, i64, i64, C.c_int, C.c_int, vp, vp]
    L.lb_router_topk.argtypes = [vp, i64, i64, i64, i64, vp, vp, vp, vp]
    L.lb_moe_permute.argtypes = [vp, i64, i64, i64, i64, vp, vp, vp, vp, C.c_size_t, vp]
    L.lb_moe_permute_noalloc.argtypes = [vp, i64, i64, i64, i64, vp, vp, vp, vp]
    L.lb_moe_workspace_size.argtypes = [C.POINTER(LbMoeArgs), C.POINTER(C.c_size_t)]
    L.lb_moe_forward.argtypes = [C.POINTER(LbMoeArgs), vp]
    L.lb_ep_buffer_size.restype = C.c_size_t
    L.lb_ep_buffer_size.argtypes = [i64, i64, i64, i64]
    L.lb_ep_buffer_alloc.argtypes = [C.c_size_t, C.POINTER(vp), vp]
    L.lb_ep_buffer_open.argtypes = [vp, C.POINTER(vp)]
    L.lb_ep_buffer_close.argtypes = [vp]
    L.lb_ep_buffer_free.argtypes = [vp]
    L.lb_ep_workspace_size.argtypes = [C.POINTER(LbEpArgs), C.POINTER(C.c_size_t)]
    L.lb_ep_moe_forward.argtypes = [C.POINTER(LbEpArgs), vp]
    L.lb_tp_buffer_size.restype = C.c_size_t
    L.lb_tp_buffer_size.argtypes = [i64, i64, i64]
    L.lb_attn_prologue.argtypes = [C.POINTER(LbPrologueArgs), vp]
    L.lb_qkv_prologue_gemm.argtypes = [vp, i64, vp, i64, vp, i64, i64, C.POINTER(LbPrologueArgs),
                                       vp, vp]
    L.lb_store_kvcache.argtypes = [vp, i64, vp, i64, vp, vp, vp, i64, i64, i64, vp]
    L.lb_pod_workspace_size.argtypes = [C.POINTER(LbPodArgs), C.POINTER(C.c_size_t)]
    L.lb_pod_attn_oproj.argtypes = [C.POINTER(LbPodArgs), vp]
    L.lb_read_device_status.argtypes = [vp, C.c_int, C.POINTER(C.c_int)]
    L.lb_device_info.argtypes = [C.POINTER(C.c_int), C.POINTER(C.c_int)]
    return L


def lib() -> C.CDLL:
    """The loaded library, after checking that a CUDA device is present."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                import torch
                if not torch.cuda.is_available():
                    raise RuntimeError("layerbatch_b200 needs a CUDA device (sm_100a); "
                                       "there is no CPU fallback")
                torch.cuda.init()
                _lib = load()
    return _lib


class LbError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != LB_OK:
        msg = lib().lb_get_last_error_string().decode(errors="replace")
        raise LbError(f"{what}: {ERRORS.get(rc, rc)}: {msg}")


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()
