"""The C ABI library: it loads, exports every symbol the header declares, and
rejects bad arguments with the documented status before touching the GPU.

No kernel is launched here (these run on machines without a GPU): every call
below fails validation, which happens before any CUDA call.
"""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from nibblegemm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_symbols():
    syms = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        syms |= set(re.findall(r"\b(ng_[a-z0-9_]+)\s*\(", text))
    return sorted(syms)


def status_codes():
    codes = {}
    for h in HEADERS:
        for m in re.finditer(r"#define\s+(NG_(?:OK|ERR_[A-Z_]+))\s+(\d+)", open(h).read()):
            codes[m.group(1)] = int(m.group(2))
    return codes


def test_library_builds_and_loads():
    lib = _lib.load()
    assert lib.ng_abi_version() == 3


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    syms = declared_symbols()
    assert set(syms) == set(_lib.SIGNATURES), "python binding and header disagree"
    for name in syms:
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr), name


def test_status_strings_cover_every_code():
    lib = _lib.load()
    codes = status_codes()
    assert codes["NG_OK"] == 0 and len(codes) >= 10
    for name, v in codes.items():
        s = lib.ng_status_string(v).decode()
        assert s and s != "unknown status", name
    assert lib.ng_status_string(999).decode() == "unknown status"


FAKE = 0x1000  # a 16-byte-aligned non-null address; never dereferenced (validation fails first)


def test_null_pointers_rejected():
    lib = _lib.load()
    c = status_codes()
    assert lib.ng_gemv_w4a16(None, 0, FAKE, FAKE, FAKE, 1, 256, 128, 128, 0, 0, 0, None, 0, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_gemm_w4a16(FAKE, 0, None, FAKE, FAKE, 32, 256, 128, 128, 0, None, 0, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_dequant_w4(FAKE, None, FAKE, 0, 256, 128, 128, 1, None) == c["NG_ERR_NULL_POINTER"]


@pytest.mark.parametrize("M,K,N,G", [
    (0, 256, 128, 128),    # empty batch
    (17, 256, 128, 128),   # above the decode limit
    (1, 256, 130, 128),    # N % 4 != 0
    (1, 192, 128, 128),    # K % G != 0
    (1, 256, 128, 32),     # unsupported group
    (1, 0, 128, 128),
])
def test_gemv_shape_validation(M, K, N, G):
    lib = _lib.load()
    assert lib.ng_gemv_w4a16(FAKE, 0, FAKE, FAKE, FAKE, M, K, N, G, 0, 0, 0, None, 0, None) == status_codes()["NG_ERR_BAD_SHAPE"]


def test_gemv_option_validation():
    lib = _lib.load()
    c = status_codes()
    assert lib.ng_gemv_w4a16(FAKE, 7, FAKE, FAKE, FAKE, 1, 256, 128, 128, 0, 0, 0, None, 0, None) == c["NG_ERR_BAD_DTYPE"]
    assert lib.ng_gemv_w4a16(FAKE, 0, FAKE, FAKE, FAKE, 1, 256, 128, 128, 17, 0, 0, None, 0, None) == c["NG_ERR_BAD_ARGUMENT"]
    assert lib.ng_gemv_w4a16(FAKE, 0, FAKE, FAKE, FAKE, 1, 256, 128, 128, 0, 96, 0, None, 0, None) == c["NG_ERR_BAD_ARGUMENT"]
    assert lib.ng_gemv_w4a16(FAKE, 1, FAKE, FAKE, FAKE, 1, 256, 128, 128, 0, 0, 1, None, 0, None) == c["NG_ERR_BAD_ARGUMENT"]
    assert lib.ng_gemv_w4a16(FAKE + 8, 0, FAKE, FAKE, FAKE, 1, 256, 128, 128, 0, 0, 0, None, 0, None) == c["NG_ERR_MISALIGNED"]


def test_dequant_validation():
    lib = _lib.load()
    c = status_codes()
    assert lib.ng_dequant_w4(FAKE, FAKE, FAKE, 3, 256, 128, 128, 1, None) == c["NG_ERR_BAD_DTYPE"]
    assert lib.ng_dequant_w4(FAKE, FAKE, FAKE, 0, 100, 128, 128, 1, None) == c["NG_ERR_BAD_SHAPE"]
    assert lib.ng_dequant_w4(FAKE, FAKE, FAKE, 0, 256, 128, 96, 1, None) == c["NG_ERR_BAD_SHAPE"]
