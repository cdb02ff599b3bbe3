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
