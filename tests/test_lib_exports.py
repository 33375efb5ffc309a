"""libkvq.so loads on a CPU-only host and exports every symbol of include/kvq.h.

No compute call is made here (no GPU); only host-side argument validation,
which returns an error status before any CUDA call.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "kvq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(kvq_[a-z_0-9]+)\s*\(", src, re.M)))


def test_header_declares_boundary():
    names = header_functions()
    for must in ("kvq_append", "kvq_sdpa_decode", "kvq_sdpa_prefill", "kvq_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from kvq import _lib
    L = _lib.lib()
    for n in header_functions():
        assert hasattr(L, n), n
    assert set(_lib.EXPORTS) >= set(header_functions())


def test_version_and_error_convention():
    from kvq import _lib
    L = _lib.lib()
    assert L.kvq_version() == 100
    h = ctypes.c_void_p()
    bad = _lib.Desc(1, 1, 128, 3, 64, 9, 0, 0, 0)  # bits 3 is unsupported
    assert L.kvq_cache_create(ctypes.byref(bad), ctypes.byref(h)) == _lib.ERR_ARG
    assert b"bits" in L.kvq_last_error()
    bad = _lib.Desc(1, 1, 100, 8, 64, 9, 0, 0, 0)  # D not a multiple of gs
    assert L.kvq_cache_create(ctypes.byref(bad), ctypes.byref(h)) == _lib.ERR_ARG
    bad = _lib.Desc(1, 1, 128, 8, 64, 10, 0, 0, 0)  # f32 dtype is not a cache dtype
    assert L.kvq_cache_create(ctypes.byref(bad), ctypes.byref(h)) == _lib.ERR_ARG
    with pytest.raises(_lib.KvqError):
        _lib.check(L.kvq_cache_create(None, ctypes.byref(h)))


def test_empty_cache_host_logic():
    """Creation without a reservation touches no device; mask/state/trim are host logic."""
    from kvq import _lib
    L = _lib.lib()
    h = ctypes.c_void_p()
    d = _lib.Desc(1, 2, 64, 8, 32, 12, 64, 0, 0)
    assert L.kvq_cache_create(ctypes.byref(d), ctypes.byref(h)) == 0
    vals = [ctypes.c_int64() for _ in range(4)]
    assert L.kvq_cache_state(h, *[ctypes.byref(v) for v in vals]) == 0
    assert [v.value for v in vals] == [0, 0, 0, 0]
    mode, win = ctypes.c_int32(), ctypes.c_int32()
    assert L.kvq_cache_make_mask(h, 1, 0, ctypes.byref(mode), ctypes.byref(win)) == 0
    assert (mode.value, win.value) == (0, 0)
    assert L.kvq_cache_make_mask(h, 100, 0, ctypes.byref(mode), ctypes.byref(win)) == 0
    assert (mode.value, win.value) == (1, 64)  # 0 + 100 > window 64 -> windowed causal
    assert L.kvq_cache_trim(h, 3, 0) == 0
    qk, qv = _lib.QTensor(), _lib.QTensor()
    assert L.kvq_cache_fetch(h, ctypes.byref(qk), ctypes.byref(qv)) == _lib.ERR_STATE
    assert L.kvq_cache_free(h) == 0
