"""numpy restatement of the reference's packed-INT4 format and its CPU oracle.

TEST INFRASTRUCTURE ONLY -- imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs, never by the ``nibblegemm_b200`` package.

Every function names the reference lines (arvindcr4/nibblegemm,
``python/nibblegemm/quant.py``) whose behaviour it restates.  The arithmetic is
the same; the code is written independently (vectorised over the slot table
instead of a per-slot loop, numpy instead of torch where torch adds nothing).

Format recap (``quant.py:8-39``): ``W[K, N]`` is consumed as ``Y = X @ W``;
eight 4-bit codes along K share one uint32 in the slot order
``SLOT_FOR_K = [0, 4, 1, 5, 2, 6, 3, 7]`` (even k in slots 0..3, odd k in
slots 4..7); a code ``u`` in ``[0, 15]`` means ``(u - 8) * scale[k // G, n]``
with one fp16 scale per (group of G rows, column).
"""
from __future__ import annotations

import numpy as np

# quant.py:47-54
SLOT_FOR_K = np.array([0, 4, 1, 5, 2, 6, 3, 7], dtype=np.int64)
K_FOR_SLOT = np.argsort(SLOT_FOR_K)
QMIN, QMAX = -8, 7
ZERO_POINT = 8
PACK_FACTOR = 8

_SHIFTS = (4 * SLOT_FOR_K).astype(np.uint32)  # bit offset of logical k within a word


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """uint8 ``[K, N]`` codes in 0..15 -> int32 ``[K/8, N]`` (quant.py:164-182).

    Raises ``ValueError`` for K % 8 != 0 or a code above 15, as the reference does.
    """
    codes = np.asarray(codes)
    K, N = codes.shape
    if K % PACK_FACTOR:
        raise ValueError(f"K={K} is not a multiple of {PACK_FACTOR}")
    if codes.size and codes.max() > 15:
        raise ValueError("codes must fit in 4 bits")
    blk = codes.reshape(K // PACK_FACTOR, PACK_FACTOR, N).astype(np.uint32) & np.uint32(0xF)
    words = np.bitwise_or.reduce(blk << _SHIFTS[None, :, None], axis=1).astype(np.uint32)
    return words.view(np.int32)


def unpack_nibbles(packed: np.ndarray, K: int) -> np.ndarray:
    """int32 ``[K/8, N]`` -> uint8 ``[K, N]`` (quant.py:185-196)."""
    w = np.ascontiguousarray(packed).view(np.uint32)
    rows, N = w.shape
    if rows * PACK_FACTOR != K:
        raise ValueError(f"{rows} packed rows do not hold K={K}")
    codes = (w[:, None, :] >> _SHIFTS[None, :, None]) & np.uint32(0xF)
    return codes.astype(np.uint8).reshape(K, N)


def dequantize_np(qweight: np.ndarray, scales: np.ndarray, group_size: int, K: int) -> np.ndarray:
    """fp16 ``[K, N]`` = fp16((u - 8) * float32(scale)), one rounding (quant.py:199-204).

    The product of a 4-bit integer and an 11-bit fp16 significand is exact in
    fp32, so the only rounding is the final cast -- the property the
    bit-exactness tests rely on.
    """
    u = unpack_nibbles(qweight, K).astype(np.float32) - np.float32(ZERO_POINT)
    s = np.repeat(np.asarray(scales, dtype=np.float16).astype(np.float32), group_size, axis=0)
    return (u * s).astype(np.float16)


def dequantize_bf16_np(qweight: np.ndarray, scales: np.ndarray, group_size: int, K: int) -> np.ndarray:
    """bf16 (as uint16 bit patterns) of the same exact fp32 product, one round-to-nearest-even.

    The reference has no bf16 path; this is the weight value a bf16-operand
    kernel must hold, derived the same way as ``dequantize_np``.
    """
    u = unpack_nibbles(qweight, K).astype(np.float32) - np.float32(ZERO_POINT)
    s = np.repeat(np.asarray(scales, dtype=np.float16).astype(np.float32), group_size, axis=0)
    return f32_to_bf16_bits(u * s)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even); returns uint16 bit patterns."""
    xf = np.ascontiguousarray(x, dtype=np.float32)
    b = xf.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(xf)] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def reference_matmul_f32(x: np.ndarray, qweight: np.ndarray, scales: np.ndarray,
                         group_size: int, K: int) -> np.ndarray:
    """fp32 ``X @ dequant(W)`` before the final fp16 cast (quant.py:207-215).

    ``x`` is any float array (fp16 or fp32 of bf16 values).  The weight is the
    fp16-rounded dequantised matrix, exactly as the reference builds it.
    """
    W = dequantize_np(qweight, scales, group_size, K).astype(np.float32)
    return np.asarray(x, dtype=np.float32) @ W


def reference_matmul(x: np.ndarray, qweight: np.ndarray, scales: np.ndarray,
                     group_size: int, K: int) -> np.ndarray:
    """fp16 result of the reference oracle (quant.py:207-215)."""
    return reference_matmul_f32(x, qweight, scales, group_size, K).astype(np.float16)


def quantize_np(W: np.ndarray, group_size: int = 128):
    """Round-to-nearest symmetric INT4 (quant.py:127-161, ``clip_search=False``).

    scale = max|w| / 7 over each group of ``group_size`` rows (clamped to >= 1e-8),
    q = clamp(round_half_even(w / scale), -8, 7) + 8.  Returns
    ``(qweight int32 [K/8, N], scales fp16 [K/G, N])``.
    """
    W = np.asarray(W, dtype=np.float32)
    if W.ndim != 2:
        raise ValueError(f"expected a 2-D weight, got shape {W.shape}")
    K, N = W.shape
    if K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    if group_size % PACK_FACTOR:
        raise ValueError(f"group_size={group_size} is not a multiple of {PACK_FACTOR}")
    g = W.reshape(K // group_size, group_size, N)
    scale = np.maximum(np.abs(g).max(axis=1) / np.float32(QMAX), np.float32(1e-8)).astype(np.float32)
    q = np.clip(np.rint(g / scale[:, None, :]), QMIN, QMAX)
    codes = (q + ZERO_POINT).reshape(K, N).astype(np.uint8)
    return pack_nibbles(codes), scale.astype(np.float16)


# ---------------------------------------------------------------------------
# BASELINE synthetic inputs (configs 1-3): seeded, CPU-generated.
# ---------------------------------------------------------------------------
def synthetic_case(M: int, K: int, N: int, group_size: int = 128, seed: int = 0,
                   act: str = "f16"):
    """Codes uniform in 0..15, scales |N(0,1)|*0.02 + 1e-3 (fp16), X ~ N(0,1).

    Returns ``(x, qweight, scales)``; ``x`` is float16 for ``act='f16'`` and
    uint16 bf16 bit patterns for ``act='bf16'``.
    """
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((K // group_size, N), dtype=np.float32)) * 0.02
              + 1e-3).astype(np.float16)
    xf = rng.standard_normal((M, K), dtype=np.float32)
    x = xf.astype(np.float16) if act == "f16" else f32_to_bf16_bits(xf)
    return x, pack_nibbles(codes), scales
