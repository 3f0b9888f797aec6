"""CPU checks of the C-ABI library: it loads without a GPU, exports every
symbol include/cyfa.h declares, and rejects bad arguments on the host before
launching anything."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cyfa.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|size_t)\s+(cyfa_\w+)\(", text, re.M)))


def test_library_loads_and_exports_header_symbols():
    from cyclic_flow_attention import _lib

    handle = _lib.lib()
    names = _declared()
    assert len(names) >= 8
    for name in names:
        assert hasattr(handle, name), name
    assert handle.cyfa_version() >= 1


def test_host_side_argument_checks():
    from cyclic_flow_attention import _lib

    L = _lib.lib()
    # null pointers are rejected before any CUDA call
    st = L.cyfa_decode_step(*([None] * 16), 1, 1, 256, 256, 0, 1e-6, 1e-6, 0.0625, None)
    assert st == 2
    assert "null" in L.cyfa_strerror(st).decode()
    # unsupported head size
    buf = ctypes.c_void_p(16)
    st = L.cyfa_decode_step(*([buf] * 16), 1, 1, 96, 256, 0, 1e-6, 1e-6, 0.1, None)
    assert st == 1
    st = L.cyfa_gates_fwd(*([buf] * 8), 0, 4, 1, None)
    assert st == 1
    st = L.cyfa_token_fwd(*([buf] * 11), 1, 4, 1, 64, 1e-6, 1e-6, None)
    assert st == 1


def test_ops_refuse_cpu_tensors():
    import torch

    from cyclic_flow_attention import _lib

    with pytest.raises(RuntimeError, match="no CPU path"):
        _lib.require_cuda(torch.zeros(2))
