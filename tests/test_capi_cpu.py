"""C-ABI checks that need no GPU: the library loads and exports every function that
``include/layerbatch_b200.h`` declares, and the Python binding knows all of them."""
import os
import re

import pytest

from layerbatch_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "layerbatch_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lb_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_binding_list():
    assert header_functions() == sorted(_lib.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built (python -m layerbatch_b200.build)")
    L = _lib.load()
    for name in header_functions():
        assert hasattr(L, name), name
    assert L.lb_version() >= 100
    # pure host-side validation paths run without a device
    assert L.lb_moe_permute_workspace_size(16, 2, 8) > 0
    assert L.lb_gemm_workspace_size() >= 4


def _lib_or_skip():
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built (python -m layerbatch_b200.build)")
    return _lib.load()


def _moe_args(**kw):
    """Shape-valid MoE arguments with stand-in (16-byte aligned, never dereferenced)
    pointers: the size query and the argument checks read no device memory."""
    fake = 0x10000
    a = _lib.LbMoeArgs(num_tokens=64, hidden=2048, num_experts=64, top_k=8, inter=512,
                       shared_inter=512, expert_base=0, num_local_experts=64,
                       x=fake, w_router=fake, w_gate_up=fake, w_down=fake,
                       w_shared_gate=fake, w_shared_up=fake, w_shared_down=fake,
                       w_shared_expert_gate=fake, out=fake)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_argument_checks_fail_with_a_message_and_no_device():
    import ctypes as C
    L = _lib_or_skip()
    fake = 0x10000
    # K must be a multiple of 64 and pointers non-null
    rc = L.lb_gemm_bf16(fake, 128, fake, 128, fake, 128, 16, 128, 100, 0, 1, fake, None)
    assert rc == 1 and b"multiple of 64" in L.lb_get_last_error_string()
    rc = L.lb_gemm_bf16(None, 128, fake, 128, fake, 128, 16, 128, 128, 0, 1, fake, None)
    assert rc == 1 and b"null" in L.lb_get_last_error_string()
    n = C.c_size_t(0)
    for bad, word in ((dict(hidden=100), b"hidden"), (dict(top_k=40), b"top_k"),
                      (dict(inter=100), b"inter"), (dict(x=None), b"null"),
                      (dict(x=fake + 8), b"aligned")):
        rc = L.lb_moe_workspace_size(C.byref(_moe_args(**bad)), C.byref(n))
        assert rc == 1, bad
        assert word in L.lb_get_last_error_string(), (bad, L.lb_get_last_error_string())


def test_moe_workspace_grows_with_the_tokens():
    import ctypes as C
    L = _lib_or_skip()
    sizes = []
    for T in (1, 64, 4096):
        n = C.c_size_t(0)
        assert L.lb_moe_workspace_size(C.byref(_moe_args(num_tokens=T)), C.byref(n)) == 0
        sizes.append(n.value)
    assert 0 < sizes[0] < sizes[1] < sizes[2]
    # at least the packed rows of the routed pairs and the shared rows, in and out
    assert sizes[2] >= (4096 * 8 + 4096) * 2048 * 2 * 2
