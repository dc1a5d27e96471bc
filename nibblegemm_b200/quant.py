"""The packed INT4 weight format and the host-side (offline) quantiser / packer.

The format is the reference's, byte for byte (arvindcr4/nibblegemm
``python/nibblegemm/quant.py:8-54``), so checkpoints and GPTQ output produced for
it load unchanged:

* ``W[K, N]`` is consumed as ``Y = X @ W`` (K is the reduction axis).
* ``qweight`` int32 ``[K/8, N]``: eight 4-bit codes along K per word.  Logical
  offset k of a word sits in nibble slot ``SLOT_FOR_K[k]`` = 0,4,1,5,2,6,3,7,
  so slots s and s+4 (16 bits apart) hold the adjacent pair (2s, 2s+1) -- the
  property the device decode uses to produce packed pairs with one AND/OR.
* ``scales`` fp16 ``[K/G, N]``; a code u means ``(u - 8) * scale`` (symmetric,
  implicit zero point 8).

Quantisation is round-to-nearest max-abs (``scale = max|w| / 7`` per group),
the reference's default.  It runs with torch on whatever device the weight is
on; packing runs wherever the codes are.  None of this is on the kernel path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

SLOT_FOR_K = np.array([0, 4, 1, 5, 2, 6, 3, 7], dtype=np.int64)
K_FOR_SLOT = np.argsort(SLOT_FOR_K)
QMIN, QMAX = -8, 7
ZERO_POINT = 8
PACK_FACTOR = 8

_BIT_OFFSET = 4 * SLOT_FOR_K  # bit position of logical k inside its word


@dataclass(frozen=True)
class QuantizedWeight:
    """Packed INT4 weights plus their fp16 group scales (reference quant.py:60-78)."""

    qweight: torch.Tensor  # int32 [K // 8, N], nibble-interleaved
    scales: torch.Tensor  # fp16  [K // G, N]
    group_size: int
    K: int
    N: int

    def to(self, device) -> "QuantizedWeight":
        return QuantizedWeight(self.qweight.to(device), self.scales.to(device), self.group_size,
                               self.K, self.N)

    @property
    def weight_bytes(self) -> int:
        """Bytes a perfect kernel must read for the weight: packed codes + scales."""
        return self.qweight.numel() * 4 + self.scales.numel() * 2

    def shard_columns(self, n0: int, n1: int) -> "QuantizedWeight":
        """Columns ``[n0, n1)`` -- a valid weight on its own (groups run along K)."""
        return QuantizedWeight(self.qweight[:, n0:n1].contiguous(),
                               self.scales[:, n0:n1].contiguous(), self.group_size, self.K, n1 - n0)

    def shard_rows(self, k0: int, k1: int) -> "QuantizedWeight":
        """Rows ``[k0, k1)`` of K; both ends must be multiples of the group size."""
        G = self.group_size
        if k0 % G or k1 % G:
            raise ValueError(f"row shard [{k0}, {k1}) is not aligned to group_size={G}")
        return QuantizedWeight(self.qweight[k0 // 8:k1 // 8].contiguous(),
                               self.scales[k0 // G:k1 // G].contiguous(), G, k1 - k0, self.N)


def pack_nibbles(qu: np.ndarray) -> np.ndarray:
    """uint8 codes ``[K, N]`` in 0..15 -> int32 ``[K // 8, N]`` in the interleaved layout."""
    qu = np.asarray(qu)
    K, N = qu.shape
    if K % PACK_FACTOR:
        raise ValueError(f"K={K} must be divisible by {PACK_FACTOR}")
    if qu.size and int(qu.max()) > 15:
        raise ValueError("quantised values must fit in 4 bits")
    words = np.zeros((K // PACK_FACTOR, N), dtype=np.uint32)
    blk = qu.reshape(K // PACK_FACTOR, PACK_FACTOR, N)
    for k in range(PACK_FACTOR):
        words |= (blk[:, k, :].astype(np.uint32) & np.uint32(0xF)) << np.uint32(_BIT_OFFSET[k])
    return words.view(np.int32)


def unpack_nibbles(packed: np.ndarray, K: int) -> np.ndarray:
    """Inverse of :func:`pack_nibbles`: uint8 ``[K, N]``."""
    words = np.ascontiguousarray(packed).view(np.uint32)
    rows, N = words.shape
    if rows * PACK_FACTOR != K:
        raise ValueError(f"packed rows={rows} inconsistent with K={K}")
    out = np.empty((rows, PACK_FACTOR, N), dtype=np.uint8)
    for k in range(PACK_FACTOR):
        out[:, k, :] = (words >> np.uint32(_BIT_OFFSET[k])) & np.uint32(0xF)
    return out.reshape(K, N)


def pack_nibbles_torch(codes: torch.Tensor) -> torch.Tensor:
    """Device-agnostic packer: integer codes ``[K, N]`` (0..15) -> int32 ``[K // 8, N]``."""
    K, N = codes.shape
    if K % PACK_FACTOR:
        raise ValueError(f"K={K} must be divisible by {PACK_FACTOR}")
    blk = codes.reshape(K // PACK_FACTOR, PACK_FACTOR, N).to(torch.int64) & 0xF
    shifts = torch.as_tensor(_BIT_OFFSET, dtype=torch.int64, device=codes.device).view(1, 8, 1)
    words = (blk << shifts).sum(dim=1)  # disjoint bit fields: sum == bitwise or
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def quantize(W: torch.Tensor, group_size: int = 128, clip_search: bool = False) -> QuantizedWeight:
    """Round-to-nearest symmetric INT4 of a ``[K, N]`` weight (reference quant.py:127-161).

    Returns CPU tensors, like the reference.  ``clip_search=True`` picks each
    group's scale among clipped max-abs candidates by the smallest squared
    reconstruction error (reference quant.py:81-125, off by default there too,
    because lower weight error did not mean a better model).
    """
    if W.ndim != 2:
        raise ValueError(f"expected a 2-D weight, got shape {tuple(W.shape)}")
    K, N = W.shape
    if K % group_size:
        raise ValueError(f"K={K} must be divisible by group_size={group_size}")
    if group_size % PACK_FACTOR:
        raise ValueError(f"group_size={group_size} must be divisible by {PACK_FACTOR}")
    return quantize_on_device(W, group_size, clip_search).to("cpu")


#: Clip ratios the scale search tries, largest first (the first of equally good
#: candidates wins): 1.0, 0.975, ..., 0.55.
CLIP_CANDIDATES = torch.linspace(1.0, 0.55, 19)


def _clip_scales(w: torch.Tensor, cols_per_pass: int = 4096) -> torch.Tensor:
    """Per-(group, column) scale of ``w`` [groups, G, N] minimising
    sum((round(w / s) clamped to [-8, 7]) * s - w)^2 over the candidates
    s = max|w| * r / 7; processed a column block at a time to bound memory."""
    ng, _, N = w.shape
    best = torch.empty(ng, N, dtype=w.dtype, device=w.device)
    ratios = CLIP_CANDIDATES.to(w.device, w.dtype)
    for c0 in range(0, N, cols_per_pass):
        blk = w[:, :, c0:c0 + cols_per_pass]
        amax = blk.abs().amax(dim=1)
        pick = (amax / QMAX).clamp(min=1e-8)
        pick_err = torch.full_like(amax, float("inf"))
        for r in ratios:
            s = (amax * r / QMAX).clamp(min=1e-8)
            recon = torch.round(blk / s[:, None, :]).clamp(QMIN, QMAX) * s[:, None, :]
            err = (recon - blk).square().sum(dim=1)
            take = err < pick_err
            pick = torch.where(take, s, pick)
            pick_err = torch.where(take, err, pick_err)
        best[:, c0:c0 + cols_per_pass] = pick
    return best


def quantize_on_device(W: torch.Tensor, group_size: int = 128, clip_search: bool = False) -> QuantizedWeight:
    """:func:`quantize` leaving the packed weight on ``W``'s device (the same RTN
    arithmetic, run by torch on a CUDA tensor: quantising a model's 224
    projections on the GPU takes seconds)."""
    K, N = W.shape
    if K % group_size or group_size % PACK_FACTOR:
        raise ValueError(f"K={K} / group_size={group_size} not supported")
    w = W.detach().float().reshape(K // group_size, group_size, N)
    scale = _clip_scales(w) if clip_search else (w.abs().amax(dim=1) / QMAX).clamp(min=1e-8)
    codes = (torch.round(w / scale.unsqueeze(1)).clamp(QMIN, QMAX) + ZERO_POINT).reshape(K, N)
    return QuantizedWeight(qweight=pack_nibbles_torch(codes).contiguous(),
                           scales=scale.to(torch.float16).contiguous(), group_size=group_size,
                           K=K, N=N)
