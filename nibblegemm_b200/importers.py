"""Checkpoint importers: GPTQ-style packed INT4 tensors -> ``QuantizedWeight``.

The format here is the reference's (arvindcr4/nibblegemm ``python/nibblegemm/
quant.py:8-54``): ``qweight`` int32 ``[K/8, N]`` with the eight codes of a word
in the interleaved slot order 0,4,1,5,2,6,3,7 (``quant.py:28-38``), a fixed
zero point 8, fp16 ``scales [K/G, N]``.  The reference's own GPTQ
(``gptq.py:131-138``) already emits exactly that, so its output loads as is.

AutoGPTQ-style checkpoints differ in two ways, handled here:

* nibble order: word ``r`` holds ``k = 8r + j`` at bits ``4j..4j+3``
  (sequential) -- repacked to the interleaved order, on the tensor's device;
* zero points: ``qzeros int32 [K/G, N/8]``, eight 4-bit zeros per word along N
  (sequential), stored as ``zero - 1`` by the original ("gptq", v1) format and
  as ``zero`` by the "gptq_v2" format.  Only symmetric checkpoints (every zero
  equal to 8) map onto the fixed zero point; anything else raises, since the
  kernels have no per-group offset term.

Act-order checkpoints (``g_idx`` other than ``k // G``) permute K and are
rejected as well: the kernels assume contiguous groups.
"""
from __future__ import annotations

from typing import Optional

import torch

from .quant import QuantizedWeight

# slot of logical k within a word (quant.py:47-54)
_SLOT_FOR_K = (0, 4, 1, 5, 2, 6, 3, 7)


def _unpack_sequential(words: torch.Tensor) -> torch.Tensor:
    """int32 ``[R, C]`` with sequential nibbles -> int64 codes ``[R, 8, C]``."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, device=words.device, dtype=torch.int64).mul_(4).view(1, 8, 1)
    return (w.unsqueeze(1) >> shifts) & 0xF


def _to_int32(words64: torch.Tensor) -> torch.Tensor:
    return torch.where(words64 >= 2**31, words64 - 2**32, words64).to(torch.int32)


def repack_sequential_to_interleaved(qweight_seq: torch.Tensor) -> torch.Tensor:
    """AutoGPTQ nibble order -> this library's (and the reference's) slot order."""
    codes = _unpack_sequential(qweight_seq)  # [K/8, 8 (k offset), N]
    slot_shift = torch.as_tensor([4 * s for s in _SLOT_FOR_K], device=codes.device,
                                 dtype=torch.int64).view(1, 8, 1)
    return _to_int32((codes << slot_shift).sum(dim=1))


def repack_interleaved_to_sequential(qweight: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`repack_sequential_to_interleaved` (for export / tests)."""
    w = qweight.to(torch.int64) & 0xFFFFFFFF
    slot_shift = torch.as_tensor([4 * s for s in _SLOT_FOR_K], device=qweight.device,
                                 dtype=torch.int64).view(1, 8, 1)
    codes = (w.unsqueeze(1) >> slot_shift) & 0xF  # [K/8, 8 (k offset), N]
    seq_shift = torch.arange(8, device=qweight.device, dtype=torch.int64).mul_(4).view(1, 8, 1)
    return _to_int32((codes << seq_shift).sum(dim=1))


def from_autogptq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                  g_idx: Optional[torch.Tensor] = None, group_size: int = 128, bits: int = 4,
                  checkpoint_format: str = "gptq") -> QuantizedWeight:
    """Load one AutoGPTQ-style linear layer (``qweight [K/8, N]``, ``qzeros
    [K/G, N/8]``, ``scales [K/G, N]``, optional ``g_idx [K]``).

    Raises ``ValueError`` for anything this format cannot hold exactly: other
    bit widths, asymmetric zero points, act-order group indices, or shapes that
    do not match.
    """
    if bits != 4:
        raise ValueError(f"only 4-bit checkpoints are supported, got bits={bits}")
    if checkpoint_format not in ("gptq", "gptq_v2"):
        raise ValueError(f"unknown checkpoint_format {checkpoint_format!r}")
    if qweight.dim() != 2 or scales.dim() != 2 or qzeros.dim() != 2:
        raise ValueError("qweight, qzeros and scales must be 2-D")
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    if K % group_size or scales.shape != (K // group_size, N) or qzeros.shape != (K // group_size, N // 8):
        raise ValueError(f"inconsistent shapes: qweight {tuple(qweight.shape)}, qzeros "
                         f"{tuple(qzeros.shape)}, scales {tuple(scales.shape)}, group_size {group_size}")
    zeros = _unpack_sequential(qzeros).permute(0, 2, 1).reshape(K // group_size, N)
    if checkpoint_format == "gptq":
        zeros = zeros + 1  # the v1 format stores zero - 1
    if not bool((zeros == 8).all()):
        raise ValueError("asymmetric zero points are not supported (the format's zero point is 8); "
                         "requantize symmetrically")
    if g_idx is not None:
        expect = torch.arange(K, device=g_idx.device) // group_size
        if not torch.equal(g_idx.to(torch.int64), expect):
            raise ValueError("act-order checkpoints (permuted g_idx) are not supported")
    return QuantizedWeight(qweight=repack_sequential_to_interleaved(qweight).contiguous(),
                           scales=scales.to(torch.float16).contiguous(), group_size=group_size,
                           K=K, N=N)


def to_autogptq(qw: QuantizedWeight, checkpoint_format: str = "gptq"):
    """Export ``qw`` as AutoGPTQ-style ``(qweight, qzeros, scales, g_idx)``."""
    K, N, G = qw.K, qw.N, qw.group_size
    if N % 8:
        raise ValueError("AutoGPTQ packs zeros 8 per word along N: N must be a multiple of 8")
    stored = 8 - (1 if checkpoint_format == "gptq" else 0)
    word = sum(stored << (4 * j) for j in range(8))
    word = word - 2**32 if word >= 2**31 else word
    qzeros = torch.full((K // G, N // 8), word, dtype=torch.int32, device=qw.qweight.device)
    g_idx = torch.arange(K, dtype=torch.int32, device=qw.qweight.device) // G
    return repack_interleaved_to_sequential(qw.qweight), qzeros, qw.scales.clone(), g_idx
