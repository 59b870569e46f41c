"""The C-ABI library loads, exports every declared symbol and refuses bad arguments without a GPU."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            names |= set(re.findall(r"CLM_API\s+[\w\s\*]+?\b(clm_b200_\w+)\s*\(", text))
    return sorted(names)


def test_every_declared_symbol_is_exported():
    from clusterlm_b200 import _native

    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(_native.lib, n), n
    # and the Python binding binds every declared symbol
    assert set(names) <= set(_native.exported_symbols())


def test_library_is_sm100a_only_build():
    from clusterlm_b200 import _native

    assert _native.lib.clm_b200_abi_version() == 1


def test_refusals_without_gpu():
    import torch

    from clusterlm_b200 import _native

    lib = _native.lib
    assert lib.clm_b200_tensor_bytes(3, 256) == 144
    assert lib.clm_b200_tensor_bytes(3, 100) == 0
    assert lib.clm_b200_tensor_bytes(2, 64) == 68
    assert lib.clm_b200_tensor_bytes(1, 64) == 72
    assert lib.clm_b200_tensor_bytes(9, 64) == 0
    n = C.c_int(-1)
    assert lib.clm_b200_device_count(C.byref(n)) == 0
    if not torch.cuda.is_available():
        assert n.value == 0
        h = C.c_void_p()
        st = lib.clm_b200_ctx_create(0, C.byref(h))
        assert st == 19  # kHardwareUnavailable
        assert b"device" in lib.clm_b200_last_error()
    # null context is an invalid argument, never a crash
    assert lib.clm_b200_ctx_synchronize(None) == 1
