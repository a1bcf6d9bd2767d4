"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before touching a device."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "smallmind_cuda.h")


def header_symbols():
    return re.findall(r"SM_API\s+int\s+(sm_\w+)\s*\(", open(HEADER).read())


def test_header_declares_the_boundary():
    syms = header_symbols()
    for name in ("sm_weight_upload", "sm_matmul", "sm_dequant", "sm_model_create", "sm_kv_create", "sm_prefill",
                 "sm_decode", "sm_last_error"):
        assert name in syms


def test_library_exports_every_header_symbol():
    import smallmind_b200 as sm
    L = sm.lib()
    for name in header_symbols():
        assert hasattr(L, name), name
    from smallmind_b200._lib import SIGNATURES
    assert set(header_symbols()) == set(SIGNATURES)


def test_host_side_argument_checks():
    import smallmind_b200 as sm
    L = sm.lib()
    assert L.sm_version() >= 1
    # null handles are rejected without touching a device
    assert L.sm_matmul(None, None, None, 1, 1, 1, 0) == -1
    assert L.sm_dequant(None, None, 0) == -1
    assert L.sm_weight_upload(None, 6, 1, 256, 0, None, 0, None, 0, 0, None) == -1
    assert L.sm_prefill(None, None, 0, None, 0, None, None) == -1
    assert L.sm_decode(None, None, None, None, 0, None, None, 0) == -1
    assert "null" in sm.last_error()
    # zero or non-dividing head counts are shape errors, checked before anything is dereferenced
    for nh, nkv in ((4, 0), (0, 2), (5, 2)):
        assert L.sm_attention_decode(None, None, None, None, None, None, 1, 16, nh, nkv, 64) == -2
        assert L.sm_attention_decode_noalloc(None, None, None, None, None, None, 1, 16, nh, nkv, 64) == -2
    assert "bad shape" in sm.last_error()
    assert L.sm_weight_destroy(None) == 0 and L.sm_ctx_destroy(None) == 0
    n = C.c_int(-1)
    rc = L.sm_device_count(C.byref(n))
    assert rc in (0, -3)


def test_shape_errors_surface_as_value_error(monkeypatch):
    import smallmind_b200._lib as L
    with pytest.raises(ValueError):
        L.check(-2, "MatMul")
    with pytest.raises(RuntimeError):
        L.check(-3, "cuda")
