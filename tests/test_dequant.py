"""Bit-exactness of the device decode (``dequant_w4``) against the oracle.

Everything demands exact equality.  The fp16 product (u - 8) * scale of a 4-bit
integer and an 11-bit significand is exact before its single rounding, so the
lop3 path, the shift/mask path and the oracle must round the same real number
the same way; any difference is a wrong mask, magic, bias or slot.
Cases follow the reference's tests/test_dequant.py:27-123 (every (slot, value)
pair isolated on a 0xF background, uniform words, random words; unit, 2**[-10,
10] and per-group 2**g scales) and are also pinned to the reference's own
dequantize output through the golden fixtures.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import nibblegemm_b200 as ng
from oracle import quant_oracle as qo
from tests.golden.make_golden import SWEEPS, sweep_nibbles

pytestmark = pytest.mark.gpu


def make_qw(qu: np.ndarray, scales: np.ndarray, G: int) -> ng.QuantizedWeight:
    K, N = qu.shape
    return ng.QuantizedWeight(torch.from_numpy(qo.pack_nibbles(qu)),
                              torch.from_numpy(np.ascontiguousarray(scales).astype(np.float16)),
                              G, K, N).to("cuda")


@pytest.mark.parametrize("name,K,extra,nseed,kind,sseed", SWEEPS)
@pytest.mark.parametrize("G", [64, 128])
@pytest.mark.parametrize("fast", [True, False])
def test_decode_matches_reference_golden(name, K, extra, nseed, kind, sseed, G, fast, golden):
    qu = sweep_nibbles(K, extra, nseed)
    qw = make_qw(qu, golden[f"sweep_{name}_g{G}_scales"], G)
    out = ng.dequant(qw, fast=fast)
    assert out.shape == (K, qu.shape[1]) and out.dtype == torch.float16
    ref = golden[f"sweep_{name}_g{G}_deq"].view(np.uint16)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref)


@pytest.mark.parametrize("N", [4, 132, 260, 1000, 1003])
@pytest.mark.parametrize("G", [64, 128])
def test_fast_equals_scalar_equals_oracle(N, G):
    rng = np.random.default_rng(N + G)
    K = 512
    qu = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    scales = (2.0 ** rng.uniform(-10, 10, size=(K // G, N))).astype(np.float32)
    qw = make_qw(qu, scales, G)
    fast = ng.dequant(qw, fast=True)
    slow = ng.dequant(qw, fast=False)
    assert torch.equal(fast, slow)
    ref = qo.dequantize_np(qw.qweight.cpu().numpy(), qw.scales.cpu().numpy(), G, K)
    assert np.array_equal(fast.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    # codebook range: |out| <= 8 * s * (1 + 2**-11)
    out = fast.float().cpu()
    s = qw.scales.float().cpu().repeat_interleave(G, dim=0)
    assert torch.all(out <= 7.0 * s * (1 + 2**-11)) and torch.all(out >= -8.0 * s * (1 + 2**-11))


@pytest.mark.parametrize("fast", [True, False])
def test_bf16_output_rounds_the_exact_product(fast):
    rng = np.random.default_rng(3)
    K, N, G = 256, 264, 128
    qu = sweep_nibbles(K, N - 144, 9)
    scales = (np.abs(rng.standard_normal((K // G, N))) * 0.02 + 1e-3).astype(np.float32)
    qw = make_qw(qu, scales, G)
    out = ng.dequant(qw, fast=fast, dtype=torch.bfloat16)
    ref = qo.dequantize_bf16_np(qw.qweight.cpu().numpy(), qw.scales.cpu().numpy(), G, K)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


def test_full_size_decode_is_bit_exact():
    """BASELINE config 1 weight (4096 x 14336), checked against the C oracle."""
    from oracle import c_oracle
    _, q, s = qo.synthetic_case(1, 4096, 14336, seed=0)
    qw = ng.QuantizedWeight(torch.from_numpy(q), torch.from_numpy(s), 128, 4096, 14336).to("cuda")
    out = ng.dequant(qw).cpu().numpy()
    ref = c_oracle.dequantize_f16(q, s, 128, 4096)
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))
