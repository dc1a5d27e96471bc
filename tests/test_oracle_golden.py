"""Pin the CPU oracle (and the host-side packer) to the reference's own outputs.

``tests/golden/golden.npz`` was produced by running the reference module
``nibblegemm.quant`` (see ``tests/golden/make_golden.py``).  Every comparison
here is exact: pack/unpack and dequantisation are integer / single-rounding
work, and the golden matmul outputs are compared after the same final fp16 cast.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import quant_oracle as qo
from tests.golden.make_golden import (MM_CASES, PACK_SHAPES, SWEEPS, mm_inputs, sweep_nibbles,
                                      sweep_scales)
import nibblegemm_b200 as ng
from nibblegemm_b200 import quant as pq

EXPECTED_SLOT_FOR_K = [0, 4, 1, 5, 2, 6, 3, 7]  # reference tests/test_pack.py:17-21


def test_slot_table_literal():
    assert list(qo.SLOT_FOR_K) == EXPECTED_SLOT_FOR_K
    assert list(pq.SLOT_FOR_K) == EXPECTED_SLOT_FOR_K
    assert [(4 + (k >> 1)) if (k & 1) else (k >> 1) for k in range(8)] == EXPECTED_SLOT_FOR_K


@pytest.mark.parametrize("pack", [qo.pack_nibbles, pq.pack_nibbles])
def test_golden_word(pack):
    """Packing k = 0..7 gives 0x75316420 (reference tests/test_pack.py:30-42)."""
    word = int(pack(np.arange(8, dtype=np.uint8).reshape(8, 1)).view(np.uint32)[0, 0])
    assert word == 0x75316420


def test_golden_word_torch_packer():
    codes = torch.arange(8, dtype=torch.int32).reshape(8, 1)
    assert int(pq.pack_nibbles_torch(codes)[0, 0]) & 0xFFFFFFFF == 0x75316420


@pytest.mark.parametrize("K,N", PACK_SHAPES)
def test_pack_matches_reference(K, N, golden):
    qu = np.random.default_rng(K * 31 + N).integers(0, 16, size=(K, N), dtype=np.uint8)
    ref = golden[f"pack_{K}x{N}"]
    for pack in (qo.pack_nibbles, pq.pack_nibbles):
        got = pack(qu)
        assert got.dtype == np.int32 and got.shape == (K // 8, N)
        assert np.array_equal(got, ref)
    assert np.array_equal(pq.pack_nibbles_torch(torch.from_numpy(qu)).numpy(), ref)
    assert np.array_equal(qo.unpack_nibbles(ref, K), qu)
    assert np.array_equal(pq.unpack_nibbles(ref, K), qu)


@pytest.mark.parametrize("pack", [qo.pack_nibbles, pq.pack_nibbles])
def test_pack_rejections(pack):
    bad = np.zeros((8, 4), dtype=np.uint8)
    bad[5, 2] = 16
    with pytest.raises(ValueError):
        pack(bad)
    with pytest.raises(ValueError):
        pack(np.zeros((12, 4), dtype=np.uint8))


@pytest.mark.parametrize("unpack", [qo.unpack_nibbles, pq.unpack_nibbles])
def test_unpack_rejects_inconsistent_k(unpack):
    with pytest.raises(ValueError):
        unpack(qo.pack_nibbles(np.zeros((16, 4), dtype=np.uint8)), 24)


@pytest.mark.parametrize("K,G", [(192, 128), (100, 64), (8, 128), (130, 128)])
def test_quantize_rejects_bad_group(K, G):
    with pytest.raises(ValueError):
        ng.quantize(torch.randn(K, 8), group_size=G)
    with pytest.raises(ValueError):
        qo.quantize_np(np.zeros((K, 8), np.float32), group_size=G)


def test_quantize_rejects_non_2d():
    with pytest.raises(ValueError):
        ng.quantize(torch.randn(4, 128, 8), group_size=128)


@pytest.mark.parametrize("name,K,extra,nseed,kind,sseed", SWEEPS)
@pytest.mark.parametrize("G", [64, 128])
def test_dequantize_matches_reference(name, K, extra, nseed, kind, sseed, G, golden):
    """Bit-exact: both oracles vs the reference's dequantize on the nibble sweeps."""
    qu = sweep_nibbles(K, extra, nseed)
    scales = golden[f"sweep_{name}_g{G}_scales"]
    assert np.array_equal(scales, sweep_scales(kind, K // G, qu.shape[1], sseed).astype(np.float16))
    ref = golden[f"sweep_{name}_g{G}_deq"].view(np.uint16)
    q = qo.pack_nibbles(qu)
    assert np.array_equal(qo.dequantize_np(q, scales, G, K).view(np.uint16), ref)
    assert np.array_equal(c_oracle.dequantize_f16(q, scales, G, K).view(np.uint16), ref)


@pytest.mark.parametrize("G", [64, 128])
def test_quantize_matches_reference(G, golden):
    W = golden[f"quant_g{G}_W"]
    q_ref, s_ref = golden[f"quant_g{G}_qweight"], golden[f"quant_g{G}_scales"]
    q, s = qo.quantize_np(W, G)
    assert np.array_equal(q, q_ref) and np.array_equal(s.view(np.uint16), s_ref.view(np.uint16))
    qw = ng.quantize(torch.from_numpy(W), group_size=G)
    assert np.array_equal(qw.qweight.numpy(), q_ref)
    assert np.array_equal(qw.scales.numpy().view(np.uint16), s_ref.view(np.uint16))


@pytest.mark.parametrize("M,K,N,G,seed", MM_CASES)
def test_reference_matmul_matches_reference(M, K, N, G, seed, golden):
    codes, scales, x = mm_inputs(M, K, N, G, seed)
    ref = golden[f"mm_{M}x{K}x{N}_g{G}_s{seed}"].astype(np.float32)
    q = qo.pack_nibbles(codes)
    y_np = qo.reference_matmul(x, q, scales, G, K).astype(np.float32)
    y_c = c_oracle.matmul_f32(x, q, scales, G, K).astype(np.float16).astype(np.float32)
    # Same fp32 products; the summation order of the reference's BLAS differs,
    # which can move a result across an fp16 rounding boundary: allow 1 ulp.
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(y_np - ref) <= ulp)
    assert np.all(np.abs(y_c - ref) <= ulp)
    assert np.mean(y_c == ref) > 0.97


def test_c_oracle_matches_numpy_oracle_on_synthetic_case():
    x, q, s = qo.synthetic_case(3, 1024, 520, seed=7)
    a = c_oracle.matmul_f32(x, q, s, 128, 1024)
    b = qo.reference_matmul_f32(x, q, s, 128, 1024)
    assert np.abs(a - b).max() / np.abs(b).max() < 1e-5
    xb, q, s = qo.synthetic_case(2, 512, 256, group_size=64, seed=8, act="bf16")
    a = c_oracle.matmul_f32(xb, q, s, 64, 512, x_kind="bf16")
    b = qo.reference_matmul_f32(qo.bf16_bits_to_f32(xb), q, s, 64, 512)
    assert np.abs(a - b).max() / np.abs(b).max() < 1e-5


def test_bf16_rounding_helper():
    vals = np.array([1.0, 1.00390625, 1.01171875, -3.5, 0.0, 65504.0, 1e-30], dtype=np.float32)
    got = qo.bf16_bits_to_f32(qo.f32_to_bf16_bits(vals))
    ref = torch.from_numpy(vals).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("G", [64, 128])
def test_quantize_clip_search_matches_reference_golden(golden, G):
    """quantize(clip_search=True): the per-group MSE search over clipped max-abs
    scales reproduces the reference's choice (and packing) bit for bit on
    weights with planted outliers, where most groups pick a clipped scale."""
    W = torch.from_numpy(golden[f"clip_g{G}_W"])
    qw = ng.quantize(W, G, clip_search=True)
    assert np.array_equal(qw.qweight.numpy(), golden[f"clip_g{G}_qweight"])
    assert np.array_equal(qw.scales.numpy(), golden[f"clip_g{G}_scales"])
    rtn = ng.quantize(W, G)
    assert (rtn.scales.numpy() != golden[f"clip_g{G}_scales"]).mean() > 0.5
