"""ctypes wrapper over ``oracle/_build/libnibble_oracle.so`` (the C restatement).

TEST INFRASTRUCTURE ONLY.  Builds the library on first use if ``make`` and a C
compiler exist (both do, here and on the GPU box).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libnibble_oracle.so")
_lib = None
_lock = threading.Lock()


def build() -> str:
    src = os.path.join(_HERE, "nibble_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                L = ctypes.CDLL(build())
                P = ctypes.c_void_p
                I = ctypes.c_int
                L.ngo_dequantize_f16.argtypes = [P, P, P, I, I, I]
                L.ngo_dequantize_f16.restype = None
                L.ngo_matmul_f32.argtypes = [P, I, P, P, P, I, I, I, I, I]
                L.ngo_matmul_f32.restype = None
                _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequantize_f16(qweight: np.ndarray, scales: np.ndarray, group_size: int, K: int) -> np.ndarray:
    q = np.ascontiguousarray(qweight).view(np.uint32)
    s = np.ascontiguousarray(scales, dtype=np.float16).view(np.uint16)
    N = q.shape[1]
    out = np.empty((K, N), dtype=np.uint16)
    lib().ngo_dequantize_f16(_ptr(q), _ptr(s), _ptr(out), K, N, group_size)
    return out.view(np.float16)


def matmul_f32(x: np.ndarray, qweight: np.ndarray, scales: np.ndarray, group_size: int,
               K: int, x_kind: str = "f16", threads: int = 0) -> np.ndarray:
    """fp32 ``x @ dequant(W)``; ``x_kind`` in {'f16', 'bf16' (uint16 bits), 'f32'}."""
    kind = {"f16": 0, "bf16": 1, "f32": 2}[x_kind]
    if kind == 0:
        xa = np.ascontiguousarray(x, dtype=np.float16).view(np.uint16)
    elif kind == 1:
        xa = np.ascontiguousarray(x, dtype=np.uint16)
    else:
        xa = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(qweight).view(np.uint32)
    s = np.ascontiguousarray(scales, dtype=np.float16).view(np.uint16)
    M = xa.shape[0]
    N = q.shape[1]
    y = np.empty((M, N), dtype=np.float32)
    lib().ngo_matmul_f32(_ptr(xa), kind, _ptr(q), _ptr(s), _ptr(y), M, K, N, group_size, threads)
    return y
