"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes
import os
import re

from tests.conftest import ROOT


def header_symbols():
    src = open(os.path.join(ROOT, "include", "wisp_b200.h")).read()
    return sorted(set(re.findall(r"WISP_API\s+[\w\s\*]*?\b(wisp_\w+)\s*\(", src)))


def test_header_declares_the_abi():
    syms = header_symbols()
    for must in ("wisp_layer_create", "wisp_layer_destroy", "wisp_moe_forward",
                 "wisp_ensure_resident", "wisp_pager_step", "wisp_get_state"):
        assert must in syms


def test_library_exports_every_header_symbol():
    from wisp_b200 import _lib
    L = _lib.lib()
    for s in header_symbols():
        assert hasattr(L, s), s
    assert sorted(_lib.SIGNATURES) == header_symbols()
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for s in header_symbols():
        assert ctypes.cast(getattr(raw, s), ctypes.c_void_p).value


def test_version_and_argument_errors_need_no_gpu():
    from wisp_b200 import _lib
    L = _lib.lib()
    assert b"sm_100a" in L.wisp_version()
    rc = L.wisp_moe_forward(None, None, None, None, 0, 1, 8, None, None)
    assert rc == _lib.WISP_ERR_INVALID
    assert b"NULL layer" in L.wisp_last_error()
    out = ctypes.c_void_p()
    rc = L.wisp_layer_create(8, 16, 0, 0, 16, 16, None, None, 0, 0, ctypes.byref(out))
    assert rc == _lib.WISP_ERR_INVALID and out.value is None


def test_error_mapping():
    import pytest
    from wisp_b200 import _lib
    _lib.lib().wisp_moe_forward(None, None, None, None, 0, 1, 8, None, None)
    with pytest.raises(_lib.WispError) as ei:
        _lib.check(_lib.WISP_ERR_INVALID, "x")
    assert ei.value.code == _lib.WISP_ERR_INVALID
    with pytest.raises(RuntimeError, match="sub-batch"):
        _lib.check(_lib.WISP_ERR_OVERFLOW)
