"""The C ABI without a GPU: the library loads and exports every function include/owsm_dec.h declares,
and the ctypes binding declares exactly those."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared() -> set[str]:
    text = (ROOT / "include" / "owsm_dec.h").read_text()
    return set(re.findall(r"\b(owsm_(?:dec|xkv)_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from owsm_trt_b200 import _lib
    from owsm_trt_b200.build import build

    build()
    return _lib.lib()


def test_header_declares_the_api():
    names = declared()
    for n in ("owsm_dec_create", "owsm_dec_plan", "owsm_dec_step", "owsm_dec_beam_step", "owsm_dec_get_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_binding_matches_header():
    from owsm_trt_b200 import _lib

    assert set(_lib.SIGNATURES) == declared()


def test_error_codes_without_gpu(lib):
    """Argument errors are reported as codes, not crashes (no CUDA call is made for them)."""
    import ctypes as C

    from owsm_trt_b200 import _lib

    out = C.c_void_p()
    assert lib.owsm_dec_create(None, None, 0, 0, C.byref(out)) == _lib.ERR_ARG
    assert b"null" in lib.owsm_dec_last_error()
    dims = _lib.Dims(2, 100, 2, 64, 10, 16, 1e-12, 10.0)  # head size 50: refused
    w = _lib.Weights()
    assert lib.owsm_dec_create(C.byref(dims), C.byref(w), 0, 0, C.byref(out)) == _lib.ERR_LIMIT
    assert lib.owsm_dec_plan(None, 1, 1, 1, 1, 1, 0, C.byref(out)) == _lib.ERR_ARG
    assert lib.owsm_dec_get_error(None) == _lib.ERR_ARG


def test_cross_kv_error_codes_without_gpu(lib):
    """The K/V projection's argument checks run before any CUDA call."""
    import ctypes as C

    from owsm_trt_b200 import _lib

    out = C.c_void_p()
    assert lib.owsm_xkv_create(2, 256, 4, _lib.F32, None, 0, C.byref(out)) == _lib.ERR_ARG
    layers = (_lib.XkvLayer * 2)()
    assert lib.owsm_xkv_create(2, 100, 2, _lib.F32, layers, 0, C.byref(out)) == _lib.ERR_LIMIT  # heads of 50
    assert lib.owsm_xkv_run(None, None, None, 1, 1, 1, None, None) == _lib.ERR_ARG
    assert lib.owsm_xkv_get_error(None) == _lib.ERR_ARG
