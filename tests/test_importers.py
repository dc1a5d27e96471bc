"""AutoGPTQ-style checkpoint import (nibble repack, zero-point and act-order
checks) against the oracle's packer and dequantiser -- CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from nibblegemm_b200 import importers
from nibblegemm_b200.quant import QuantizedWeight
from oracle import quant_oracle as qo


def _sequential_pack(codes: np.ndarray) -> np.ndarray:
    """Independent restatement of the AutoGPTQ packing: k = 8r + j at bits 4j."""
    K, N = codes.shape
    blk = codes.reshape(K // 8, 8, N).astype(np.uint64)
    words = np.zeros((K // 8, N), dtype=np.uint64)
    for j in range(8):
        words |= blk[:, j, :] << np.uint64(4 * j)
    return words.astype(np.uint32).view(np.int32)


def _zeros_word(z: int) -> int:
    w = sum(z << (4 * j) for j in range(8))
    return w - 2**32 if w >= 2**31 else w


@pytest.mark.parametrize("K,N,G", [(256, 64, 128), (1024, 136, 64), (512, 8, 256)])
@pytest.mark.parametrize("fmt", ["gptq", "gptq_v2"])
def test_import_matches_interleaved_pack_and_dequant(K, N, G, fmt):
    rng = np.random.default_rng(K + N + G)
    codes = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((K // G, N))) * 0.02 + 1e-3).astype(np.float16)
    stored = 7 if fmt == "gptq" else 8
    qzeros = torch.full((K // G, N // 8), _zeros_word(stored), dtype=torch.int32)
    qw = importers.from_autogptq(torch.from_numpy(_sequential_pack(codes)), qzeros,
                                 torch.from_numpy(scales), torch.arange(K) // G, group_size=G,
                                 checkpoint_format=fmt)
    assert np.array_equal(qw.qweight.numpy(), qo.pack_nibbles(codes))
    assert np.array_equal(qo.dequantize_np(qw.qweight.numpy(), qw.scales.numpy(), G, K),
                          ((codes.astype(np.float32) - 8) * np.repeat(scales.astype(np.float32), G, 0)
                           ).astype(np.float16))


def test_round_trip_export_import():
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 16, size=(512, 64), dtype=np.uint8)
    qw = QuantizedWeight(torch.from_numpy(qo.pack_nibbles(codes)),
                         torch.rand(4, 64).half(), 128, 512, 64)
    for fmt in ("gptq", "gptq_v2"):
        qweight, qzeros, scales, g_idx = importers.to_autogptq(qw, fmt)
        assert np.array_equal(qweight.numpy(), _sequential_pack(codes))
        back = importers.from_autogptq(qweight, qzeros, scales, g_idx, 128, checkpoint_format=fmt)
        assert torch.equal(back.qweight, qw.qweight) and torch.equal(back.scales, qw.scales)


def test_rejects_what_the_format_cannot_hold():
    K, N, G = 256, 16, 128
    qweight = torch.zeros(K // 8, N, dtype=torch.int32)
    scales = torch.ones(K // G, N, dtype=torch.float16)
    ok = torch.full((K // G, N // 8), _zeros_word(7), dtype=torch.int32)
    with pytest.raises(ValueError, match="asymmetric"):
        importers.from_autogptq(qweight, torch.full_like(ok, _zeros_word(3)), scales, group_size=G)
    with pytest.raises(ValueError, match="act-order"):
        importers.from_autogptq(qweight, ok, scales, torch.arange(K).flip(0) // G, group_size=G)
    with pytest.raises(ValueError, match="4-bit"):
        importers.from_autogptq(qweight, ok, scales, group_size=G, bits=8)
    with pytest.raises(ValueError, match="inconsistent"):
        importers.from_autogptq(qweight, ok, scales[:1], group_size=G)
