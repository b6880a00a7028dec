"""The C ABI library: it loads, exports what the header declares, and its
argument checks answer without a GPU."""
import ctypes

import pytest

from elffuss_engine_b200 import _lib


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = _lib.header_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the Python binding declares a signature for each
    assert set(syms) == set(_lib._SIGS)


def test_version_and_type_info():
    L = _lib.lib()
    assert L.ef_version() == 1
    be, bb = ctypes.c_int(), ctypes.c_int()
    for t, want in ((8, (32, 34)), (12, (256, 144)), (14, (256, 210)), (16, (256, 66)), (19, (256, 50))):
        assert L.ef_type_info(t, ctypes.byref(be), ctypes.byref(bb)) == 0
        assert (be.value, bb.value) == want
    assert L.ef_type_info(3, ctypes.byref(be), ctypes.byref(bb)) == -2   # no decoder: EF_ERR_TYPE


def test_null_arguments_are_rejected():
    L = _lib.lib()
    assert L.ef_ctx_create(0, None) == -1
    assert L.ef_ctx_destroy(None) == -1
    assert L.ef_gemv(None, None, None, 1, None) == -1
    assert L.ef_stream_sync(None) == -1
    assert L.ef_last_error(None) == b"null context"


def test_check_raises_on_negative_status():
    with pytest.raises(_lib.EfError) as e:
        _lib.check(-3)
    assert e.value.code == -3
    assert _lib.check(_lib.EF_NOT_APPLICABLE) == 1
