"""ctypes binding of ``libuttt_b200.so`` (the C ABI declared in include/uttt_b200.h).

The library is loaded from the package directory (built in-tree by
``python -m utttcompanion_b200.build``).  There is no fallback: if it is
missing, every op raises.  Status codes map to the reference's error
classes: invalid arguments / unsupported shapes -> ``ValueError`` (the
server maps those to HTTP 422, ``server/app.py:271-272``), runtime and
device-wait failures -> ``RuntimeError``.
"""

from __future__ import annotations

import ctypes as C
import os
import re
from typing import Dict, Optional

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libuttt_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "uttt_b200.h")

UTTT_OK = 0
UTTT_ERR_INVALID = 1
UTTT_ERR_UNSUPPORTED = 2
UTTT_ERR_CUDA = 3
UTTT_ERR_TIMEOUT = 4
UTTT_ERR_WORKSPACE = 5
DTYPE_F32 = 0
DTYPE_BF16 = 1
ENGINE_RING = 8
ROW_IDLE, ROW_RUNNING, ROW_FINISHED = 0, 1, 2

vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t

# argtypes per exported symbol; kept in the same order as include/uttt_b200.h
# uttt_partial_sum_fn: int (*)(float* data, size_t count, void* ctx, void* stream)
PARTIAL_SUM_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)

SIGNATURES: Dict[str, tuple] = {
    "uttt_version": (i32, []),
    "uttt_status_string": (C.c_char_p, [i32]),
    "uttt_last_cuda_error": (i32, []),
    "uttt_read_status": (i32, [vp, i32, vp]),
    "uttt_profile_enable": (i32, [i32]),
    "uttt_profile_read": (i32, [vp, vp]),
    "uttt_selftest_gemm": (i32, [i32, i32, i32, i32, vp, vp, vp, vp, sz, vp]),
    "uttt_selftest_wait": (i32, [i32, C.c_uint, vp, sz, vp]),
    "uttt_chunk_write_workspace": (sz, [i32, i32, i32, i32]),
    "uttt_chunk_write": (i32, [i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                               vp, vp, f32, f32, i32, f32, vp, i32, vp, vp, i32, vp, vp, vp, vp, sz, vp]),
    "uttt_chunk_write_guarded": (i32, [i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                       vp, vp, vp, vp, f32, f32, i32, f32, vp, i32, vp, vp, vp, vp, f32, vp, vp, vp,
                                       sz, vp]),
    "uttt_chunk_write_noalloc": (i32, [i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                       vp, vp, vp, vp, f32, f32, i32, f32, vp, i32, vp, vp, vp]),
    "uttt_chunk_write_noalloc_status": (i32, [i32, vp]),
    "uttt_fast_readout_workspace": (sz, [i32, i32, i32, i32]),
    "uttt_fast_readout": (i32, [i32, i32, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, f32, vp, i32, vp, sz, vp]),
    "uttt_fast_readout_partial": (i32, [i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, sz, vp]),
    "uttt_readout_finish": (i32, [i32, i32, vp, vp, vp, vp, f32, vp, i32, i32, vp]),
    "uttt_split_exchange_bytes": (sz, [i32, i32, i32]),
    "uttt_ipc_alloc": (i32, [sz, vp, vp]),
    "uttt_ipc_open": (i32, [vp, vp]),
    "uttt_ipc_close": (i32, [vp]),
    "uttt_ipc_free": (i32, [vp]),
    "uttt_split_exchange_finish": (i32, [i32, i32, vp, vp, vp, vp, f32, vp, i32, i32, i32, i32, i32, vp, C.c_uint,
                                         vp, sz, vp]),
    "uttt_linear_workspace": (sz, [i32, i32]),
    "uttt_linear": (i32, [i32, i32, i32, vp, vp, i32, vp, f32, vp, sz, vp]),
    "uttt_attn_decode": (i32, [i32, i32, i32, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, vp, i32, vp]),
    "uttt_attn_prefill": (i32, [i32, i32, i32, i32, i32, i32, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, vp]),
    "uttt_kv_ring_fill": (i32, [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]),
    "uttt_rmsnorm": (i32, [i32, i32, vp, C.c_longlong, vp, f32, vp, C.c_longlong, vp]),
    "uttt_embed": (i32, [i32, i32, i32, vp, vp, vp, vp]),
    "uttt_greedy_argmax": (i32, [i32, i32, vp, i32, C.c_longlong, i32, i32, vp, vp, vp]),
    "uttt_engine_step": (i32, [i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, vp]),
    "uttt_engine_admit": (i32, [i32, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, vp]),
    "uttt_pack_read_copies": (i32, [i32, i32, i32, vp, vp, vp, vp, vp, vp]),
    "uttt_apply_rope": (i32, [C.c_longlong, i32, i32, vp, vp, vp, vp, vp]),
    "uttt_guard_workspace": (sz, [i32]),
    "uttt_elastic_pull": (i32, [i32, i32, i32, vp, vp, vp, vp, vp, vp, f32, f32, vp, sz, vp]),
    "uttt_drift_sums": (i32, [i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
}


class Segment(C.Structure):
    """``UtttSegment`` of include/uttt_b200.h."""
    _fields_ = [("start", C.c_int), ("len", C.c_int), ("op", C.c_int), ("out_f32", C.c_int),
                ("out", C.c_void_p), ("out_ld", C.c_longlong), ("aux", C.c_void_p), ("aux_ld", C.c_longlong),
                ("scale", C.c_float), ("aux2", C.c_void_p)]


SEG_STORE, SEG_RESID, SEG_RMSNORM, SEG_SIGMOID, SEG_NORM = 0, 1, 2, 3, 4

_lib: Optional[C.CDLL] = None


class UtttError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m utttcompanion_b200.build` "
            "(there is no CPU fallback for the uTTT B200 ops)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        try:
            fn = getattr(lib, name)
        except AttributeError:      # reported by tests/test_capi.py
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def header_symbols() -> list:
    """Function names declared in include/uttt_b200.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(uttt_[a-z0-9_]+)\s*\(", text)))


def check(status: int, what: str = "uttt op") -> None:
    if status == UTTT_OK:
        return
    lib = load()
    msg = lib.uttt_status_string(status).decode()
    if status in (UTTT_ERR_INVALID, UTTT_ERR_UNSUPPORTED, UTTT_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    cuda = lib.uttt_last_cuda_error()
    raise UtttError(f"{what}: {msg}" + (f" (cudaError {cuda})" if cuda else ""))
