"""ctypes binding of libqwa.so (the C ABI in include/qwa.h).

There is no fallback: if the library is missing or cannot be loaded, every
call raises. Build it with ``build.build()`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwa.so")

QWA_OK, QWA_ERR_INVALID_ARG, QWA_ERR_UNSUPPORTED, QWA_ERR_CUDA, QWA_ERR_TIMEOUT, \
    QWA_ERR_NO_DEVICE = range(6)
MODE_AUTO, MODE_FULL, MODE_SPARSE = 0, 1, 2

P = ctypes.c_void_p
I32, I64, F32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float
I32P = ctypes.POINTER(ctypes.c_int32)
I64P = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); the exported surface of include/qwa.h
SIGNATURES = {
    "qwa_create": (I32, [I32, ctypes.POINTER(P)]),
    "qwa_destroy": (I32, [P]),
    "qwa_last_error": (ctypes.c_char_p, [P]),
    "qwa_status_string": (ctypes.c_char_p, [I32]),
    "qwa_version": (ctypes.c_char_p, []),
    "qwa_qk_norm_rope": (I32, [P, P, I64, P, P, P, P, I32P, I32, F32, F32, P, P]),
    "qwa_qk_norm_rope_padded": (I32, [P, P, I64, P, P, P, P, I32, I32, F32, F32, P, P]),
    "qwa_attention": (I32, [P, P, P, P, I64, I64, P, I32P, I32, I32, I32, I32, P]),
    "qwa_attention_padded": (I32, [P, P, P, P, P, I32, I32, I32, I32, I64, I64, P]),
    "qwa_prefill_attention_layer": (I32, [P, P, I64, P, P, P, P, P, I32P, I32, I32, I32, I32, F32,
                                          F32, P]),
    "qwa_check": (I32, [P, P]),
    "qwa_set_debug": (I32, [P, I64, I32]),
    "qwa_attention_work": (I32, [I32P, I32, I32, I32, I32, I64P, I64P]),
    "qwa_selftest_tile": (I32, [P, P, P, P, P, P, P]),
    "qwa_attention_noalloc": (I32, [P, P, P, I64, I64, P, I32P, I32, I32, I32, I32, P]),
    "qwa_matmul": (I32, [P, P, P, P, I32, I32, I32, P]),
    "qwa_matmul_swiglu": (I32, [P, P, P, P, I32, I32, I32, P]),
    "qwa_q40_dequantize": (I32, [P, P, I32, I32, P, P]),
    "qwa_q40_matmul": (I32, [P, P, P, P, I32, I32, I32, P]),
    "qwa_q40_forget": (I32, [P, P]),
    "qwa_qkv_projection": (I32, [P, P, P, I32, P, P, P, P, P, I32P, I32, F32, F32, P, P]),
    "qwa_q40_qkv_projection": (I32, [P, P, P, I32, P, P, P, P, P, I32P, I32, F32, F32, P, P]),
    "qwa_rms_norm": (I32, [P, P, P, P, P, I32, I32, F32, I32, P]),
    "qwa_swiglu": (I32, [P, P, P, I32, I32, P]),
    "qwa_embedding_lookup_q6k": (I32, [P, P, P, I32, P, I32, I32, P]),
    "qwa_last_token_pool": (I32, [P, P, I32, P, I32P, I32, P]),
    "qwa_last_token_pool_padded": (I32, [P, P, P, P, I32, I32, I32, P]),
}

_lib = None


class QwaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"qwa status {status}: {message}")
        self.status = status


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run the package's build.build() first")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().qwa_status_string(status).decode()


def check(status: int, ctx=None) -> None:
    if status != QWA_OK:
        msg = load().qwa_last_error(ctx).decode() if ctx else ""
        raise QwaError(status, msg or status_string(status))


def cu_array(cu_seqlens) -> ctypes.Array:
    vals = [int(x) for x in cu_seqlens]
    return (ctypes.c_int32 * len(vals))(*vals)
