"""ctypes binding of ``libowsmdec.so`` (the C ABI in ``include/owsm_dec.h``).

The library is the only compute path: if it is missing or fails to load, :func:`lib` raises. There is
no CPU or PyTorch fallback."""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libowsmdec.so"

OK, ERR_ARG, ERR_CUDA, ERR_TIMEOUT, ERR_LIMIT = 0, -1, -2, -3, -4
F32, F16 = 0, 1

# every function the header declares, with its ctypes signature
vp, i32, i64, u32 = C.c_void_p, C.c_int, C.c_int64, C.c_uint32


class Dims(C.Structure):
    _fields_ = [("L", i32), ("D", i32), ("H", i32), ("F", i32), ("V", i32), ("max_pos", i32),
                ("eps", C.c_float), ("xscale", C.c_float)]  # fmt: skip


class Layer(C.Structure):
    _fields_ = [(n, vp) for n in ("wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo", "wcq", "bcq", "wco", "bco",
                                  "w1", "b1", "w2", "b2", "ln1_g", "ln1_b", "ln2_g", "ln2_b", "ln3_g", "ln3_b")]  # fmt: skip


class XkvLayer(C.Structure):
    _fields_ = [("wk", vp), ("wv", vp), ("bk", vp), ("bv", vp)]


class Weights(C.Structure):
    _fields_ = [("weight_dtype", i32), ("emb", vp), ("pe", vp), ("layers", C.POINTER(Layer)), ("lnf_g", vp),
                ("lnf_b", vp), ("wout", vp), ("bout", vp)]  # fmt: skip


SIGNATURES = {
    "owsm_dec_create": (i32, [C.POINTER(Dims), C.POINTER(Weights), i32, i32, C.POINTER(vp)]),
    "owsm_dec_destroy": (None, [vp]),
    "owsm_dec_plan": (i32, [vp, i32, i32, i32, i32, i32, i32, C.POINTER(vp)]),
    "owsm_dec_plan_destroy": (None, [vp]),
    "owsm_dec_step": (i32, [vp, vp, vp, i64, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32]),
    "owsm_dec_step_verify": (i32, [vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "owsm_dec_beam_step": (i32, [vp, vp, vp, i64, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "owsm_dec_get_error": (i32, [vp]),
    "owsm_dec_plan_reset": (i32, [vp]),
    "owsm_dec_plan_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i64)]),
    "owsm_dec_plan_trace": (i32, [vp, vp]),
    "owsm_dec_plan_trace_from": (i32, [vp, i32]),
    "owsm_dec_plan_stages": (i32, [vp, i32]),
    "owsm_dec_set_max_spin": (i32, [vp, u32]),
    "owsm_dec_set_path": (i32, [vp, i32]),
    "owsm_dec_plan_kernel": (i32, [vp]),
    "owsm_dec_plan_launches": (i32, [vp]),
    "owsm_dec_step_static": (i32, [vp, vp, i32, i32, i32, i32, vp, i64, vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                   i32, i32]),  # fmt: skip
    "owsm_dec_last_error": (C.c_char_p, []),
    "owsm_xkv_create": (i32, [i32, i32, i32, i32, C.POINTER(XkvLayer), i32, C.POINTER(vp)]),
    "owsm_xkv_run": (i32, [vp, vp, vp, i32, i32, i32, vp, vp]),
    "owsm_xkv_get_error": (i32, [vp]),
    "owsm_xkv_destroy": (None, [vp]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built: run `python -m owsm_trt_b200.build` (nvcc, sm_100a)")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


class OwsmDecError(RuntimeError):
    def __init__(self, code: int, what: str):
        msg = lib().owsm_dec_last_error().decode(errors="replace")
        super().__init__(f"{what} failed ({code}): {msg}")
        self.code = code


def check(code: int, what: str) -> None:
    if code != OK:
        raise OwsmDecError(code, what)
