"""ctypes binding of the C ABI in ``include/nibblegemm_b200.h``.

The shared library is built in-tree (``python -m nibblegemm_b200.build``) and
loaded from the package directory.  There is no fallback: if the library is
missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libnibblegemm_b200.so")

NG_OK = 0
NG_DTYPE_F16 = 0
NG_DTYPE_BF16 = 1

#: Every symbol the header declares, with (restype, argtypes).
_P, _I = ctypes.c_void_p, ctypes.c_int
SIGNATURES = {
    "ng_abi_version": (_I, []),
    "ng_status_string": (ctypes.c_char_p, [_I]),
    "ng_device_status": (_I, [_P]),
    "ng_dequant_w4": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "ng_gemv_w4a16": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, ctypes.c_size_t, _P]),
    "ng_gemv_workspace_bytes": (ctypes.c_size_t, [_I, _I]),
    "ng_gemv_w4a16_noalloc": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ng_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P]),
    "ng_rope_append": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P]),
    "ng_rope_prefill": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P]),
    "ng_attn_prefill": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _P]),
    "ng_attn_workspace_bytes": (ctypes.c_size_t, [_I, _I, _I]),
    "ng_attn_decode": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float, _P,
                            ctypes.c_size_t, _P]),
    "ng_silu_mul": (_I, [_P, _P, _I, _I, _I, _P]),
    "ng_gemv_w4a16_rmsnorm": (_I, [_P, _P, _P, _P, ctypes.c_float, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ng_attn_decode_rope": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, ctypes.c_float,
                                 ctypes.c_float, _P, ctypes.c_size_t, _P]),
    "ng_argmax": (_I, [_P, _I, _I, _I, ctypes.c_longlong, _P, _P, _P, _P]),
    "ng_allreduce_buffer_bytes": (ctypes.c_size_t, [_I, ctypes.c_size_t]),
    "ng_allreduce_sum": (_I, [_P, _I, ctypes.c_size_t, _P, _I, _I, ctypes.c_size_t, _P, _P]),
    "ng_ipc_alloc": (_I, [ctypes.c_size_t, _P, _P]),
    "ng_ipc_free": (_I, [_P]),
    "ng_ipc_open": (_I, [_P, _P]),
    "ng_ipc_close": (_I, [_P]),
    "ng_gemm_w4a16": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P, ctypes.c_size_t, _P]),
    "ng_gemm_workspace_bytes": (ctypes.c_size_t, [_I, _I]),
    "ng_gemv_w4a16_silu": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ng_gemv_w4a16_attn": (_I, [_P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ng_gemv_allreduce_buffer_bytes": (ctypes.c_size_t, [_I, _I]),
    "ng_gemv_w4a16_allreduce": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _I, _P]),
    "ng_lm_head_argmax": (_I, [_P, _P, _I, _I, _I, _I, ctypes.c_longlong, _P, _P, _P]),
    "ng_embed_tokens": (_I, [_P, _P, _P, _P, _I, _I, _I, ctypes.c_longlong, _P, _P, _P]),
}

_lib = None
_lock = threading.Lock()


class NibbleError(RuntimeError):
    """A non-zero status from the C ABI."""


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m nibblegemm_b200.build` "
                    "(there is no CPU fallback)")
            L = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != NG_OK:
        msg = load().ng_status_string(status).decode()
        raise NibbleError(f"{what}: {msg} (status {status})")
