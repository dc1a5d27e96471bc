"""Parity of the decode GEMV (``gemv_w4a16``) with the CPU oracle.

Gate: max|y - ref| / max|ref| <= 5e-3 against the oracle's fp32 result, where
ref = X @ dequant(W) with the reference's fp16-rounded weights (quant.py:207-215).
Expected error, derived per path:
  * algo 1 (fp16 activations): half2 accumulation of 16 products per lane per
    32-value window, then fp32.  CPU emulation of this scheme on config 1 gives
    ~7e-4; the fp16 output rounding alone is 2**-11 ~ 4.9e-4 of max|ref|.
  * algo 2 / bf16: exact fp32 weights and fp32 accumulation: only summation
    order (~1e-6) and the output rounding (fp16 4.9e-4, bf16 3.9e-3 of max|ref|).
The reference suite's own metric (max|err| / mean|ref| < 5e-2, tests/test_gemv.py)
is checked as well.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import nibblegemm_b200 as ng
from oracle import c_oracle
from oracle import quant_oracle as qo
from tests.conftest import max_rel, mean_rel

pytestmark = pytest.mark.gpu

GATE = 5e-3
REF_TOL = 5e-2


def make_case(M, K, N, G=128, seed=0, act="f16"):
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=seed, act=act)
    qw = ng.QuantizedWeight(torch.from_numpy(q), torch.from_numpy(s), G, K, N).to("cuda")
    if act == "f16":
        X = torch.from_numpy(x).cuda()
        ref = c_oracle.matmul_f32(x, q, s, G, K)
    else:
        X = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
        ref = c_oracle.matmul_f32(x, q, s, G, K, x_kind="bf16")
    return X, qw, ref


def check(y, ref, dtype):
    assert y.dtype == dtype
    yf = y.float().cpu().numpy()
    assert np.isfinite(yf).all()
    err = max_rel(yf, ref)
    assert err <= GATE, err
    assert mean_rel(yf, ref) < REF_TOL
    return err


CASES = [(1, 512, 256), (2, 256, 132), (3, 1024, 260), (4, 512, 512), (5, 2048, 132),
         (8, 512, 256), (9, 1024, 388), (13, 256, 128), (16, 512, 1028)]


@pytest.mark.parametrize("M,K,N", CASES)
@pytest.mark.parametrize("G", [64, 128])
@pytest.mark.parametrize("act,algo", [("f16", 0), ("f16", 1), ("f16", 2), ("bf16", 0), ("bf16", 2)])
def test_gemv_matches_oracle(M, K, N, G, act, algo):
    X, qw, ref = make_case(M, K, N, G, seed=M * 7 + N, act=act)
    y = ng.gemv(X, qw, algo=algo)
    assert y.shape == (M, N)
    check(y, ref, X.dtype)


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("splits", [1, 2, 4, 5, 16])
@pytest.mark.parametrize("threads", [128, 256])
def test_split_and_block_invariance(M, splits, threads):
    """Any K split / block width gives the same answer to fp32 summation order."""
    X, qw, ref = make_case(M, 1024, 256, 64, seed=2)
    y = ng.gemv(X, qw, splits=splits, block_threads=threads)
    check(y, ref, torch.float16)
    base = ng.gemv(X, qw, splits=1, block_threads=256)
    d = (y.float() - base.float()).abs().max().item() / base.float().abs().max().item()
    assert d < 2e-3


def test_version3_is_one_split():
    X, qw, _ = make_case(4, 1024, 256, 64, seed=3)
    assert torch.equal(ng.gemv(X, qw, version=4, splits=1), ng.gemv(X, qw, version=3))


def test_deterministic():
    X, qw, _ = make_case(4, 4096, 1024, 128, seed=4)
    a = ng.gemv(X, qw)
    for _ in range(3):
        assert torch.equal(a, ng.gemv(X, qw))


def test_rejects_m_above_16():
    X, qw, _ = make_case(17, 256, 132, 128, seed=5)
    with pytest.raises(RuntimeError):
        ng.gemv(X, qw)


def test_rejects_bad_inputs():
    X, qw, _ = make_case(2, 256, 132, 128, seed=6)
    with pytest.raises(RuntimeError):
        ng.gemv(X.float(), qw)
    with pytest.raises(RuntimeError):
        ng.gemv(X[:, :128], qw)


def test_matmul_dispatch_and_k_mismatch():
    X, qw, _ = make_case(ng.DECODE_MAX_M, 512, 256, 128, seed=7)
    assert torch.equal(ng.matmul(X, qw), ng.gemv(X, qw, version=4))
    with pytest.raises(ValueError):
        ng.matmul(torch.randn(1, 256, device="cuda", dtype=torch.float16), qw)


def test_output_fully_written():
    """A poisoned output buffer must be completely overwritten."""
    X, qw, ref = make_case(3, 1024, 1028, 128, seed=8)
    out = torch.full((3, 1028), float("nan"), dtype=torch.float16, device="cuda")
    ng.extension().gemv_w4a16(X, qw.qweight, qw.scales, 128, out=out)
    check(out, ref, torch.float16)


# BASELINE config 1 and the config 2 sweep shapes at full size.
FULL = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096), (8192, 8192)]


@pytest.mark.parametrize("K,N", FULL)
@pytest.mark.parametrize("M", [1, 16])
def test_full_size_shapes(K, N, M):
    X, qw, ref = make_case(M, K, N, 128, seed=K + N + M)
    check(ng.gemv(X, qw), ref, torch.float16)


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
def test_config1_every_path(M):
    X, qw, ref = make_case(M, 4096, 14336, 128, seed=11, act="bf16")
    check(ng.gemv(X, qw), ref, torch.bfloat16)
    check(ng.gemv(X, qw, algo=2), ref, torch.bfloat16)
    X, qw, ref = make_case(M, 4096, 14336, 128, seed=12)
    for algo in (0, 1, 2, 3):
        check(ng.gemv(X, qw, algo=algo), ref, torch.float16)


def test_workspace_counters_left_zero():
    ext = ng.extension()
    for (M, K, N) in [(1, 4096, 14336), (16, 1024, 4100), (3, 14336, 4096)]:
        X, qw, ref = make_case(M, K, N, 128, seed=N)
        check(ext.gemv_w4a16(X, qw.qweight, qw.scales, 128), ref, torch.float16)
        ws = ext.workspace(N, X.device, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        sm = torch.cuda.get_device_properties(X.device).multi_processor_count
        off = 2 * 4 * sm * 16 * 64 * 4  # counters follow the partial-sum slots
        assert int(ws[off:off + 4 * ((N + 63) // 64)].count_nonzero()) == 0


@pytest.mark.parametrize("M,K,N,G", [(1, 4096, 14336, 128), (3, 14336, 4096, 128), (16, 1024, 132, 64),
                                     (2, 256, 4, 128), (1, 320, 1024, 64), (8, 8192, 8192, 256),
                                     (16, 14336, 4096, 128)])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_heuristic_split_matches_oracle_and_fixed_splits(M, K, N, G, act):
    """Default schedule vs the oracle and vs an explicit split count, including
    tiny N, K that is not a multiple of the 8-row chunk per slice, and M=16 at
    K=14336 where the split count is raised so activations fit on chip."""
    X, qw, ref = make_case(M, K, N, G, seed=M + K + N, act=act)
    ext = ng.extension()
    y = ext.gemv_w4a16(X, qw.qweight, qw.scales, G)
    check(y, ref, X.dtype)
    yc = ext.gemv_w4a16(X, qw.qweight, qw.scales, G, splits_override=3)
    d = (y.float() - yc.float()).abs().max().item() / yc.float().abs().max().item()
    assert d < 4e-3
    for _ in range(2):
        assert torch.equal(y, ext.gemv_w4a16(X, qw.qweight, qw.scales, G))
    assert ext.device_status() == 0


# ---------------------------------------------------------------------------
# Bulk-copy ring schedule (algo 4, M <= 8)
# ---------------------------------------------------------------------------
RING_CASES = [(1, 512, 256), (2, 256, 132), (3, 1024, 260), (4, 512, 512), (5, 2048, 132),
              (8, 512, 256), (1, 320, 1024), (2, 256, 4), (7, 8192, 388)]


@pytest.mark.parametrize("M,K,N", RING_CASES)
@pytest.mark.parametrize("G", [64, 128, 256])
@pytest.mark.parametrize("act", ["f16", "bf16"])
@pytest.mark.parametrize("algo", [4, 5])
def test_ring_matches_oracle(M, K, N, G, act, algo):
    if K % G:
        pytest.skip("K not a multiple of G")
    X, qw, ref = make_case(M, K, N, G, seed=M * 5 + N + G, act=act)
    check(ng.gemv(X, qw, algo=algo), ref, X.dtype)
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("K,N", FULL + [(2048, 4096), (4096, 3072), (4096, 7168), (7168, 4096)])
@pytest.mark.parametrize("M", [1, 8])
@pytest.mark.parametrize("algo", [4, 5])
def test_ring_full_size_shapes(K, N, M, algo):
    """BASELINE config 1 / config 2 shapes and the tensor-parallel Llama-3-8B
    shards (o / qkv / gate-up / down at TP=2), including multi-wave stage reuse."""
    X, qw, ref = make_case(M, K, N, 128, seed=K + N + M)
    check(ng.gemv(X, qw, algo=algo), ref, torch.float16)
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("algo", [4, 5])
def test_ring_split_invariance(splits, algo):
    X, qw, ref = make_case(2, 4096, 1028, 128, seed=splits)
    y = ng.gemv(X, qw, splits=splits, algo=algo)
    check(y, ref, torch.float16)
    assert torch.equal(y, ng.gemv(X, qw, splits=splits, algo=algo))


def test_ring_output_fully_written_and_rejects_m_above_8():
    X, qw, ref = make_case(3, 1024, 1028, 128, seed=8)
    out = torch.full((3, 1028), float("nan"), dtype=torch.float16, device="cuda")
    for algo in (4, 5):
        out.fill_(float("nan"))
        ng.extension().gemv_w4a16(X, qw.qweight, qw.scales, 128, algo=algo, out=out)
        check(out, ref, torch.float16)
    X9, qw9, _ = make_case(9, 256, 128, 128)
    with pytest.raises(Exception):
        ng.gemv(X9, qw9, algo=4)


@pytest.mark.parametrize("algo", [4, 5])
def test_ring_back_to_back_in_graph(algo):
    """A chain of ring GEMVs captured in one CUDA graph (programmatic dependent
    launch between them): each output still matches its own oracle."""
    cases = [make_case(1, K, N, 128, seed=K + N) for K, N in [(4096, 14336), (14336, 4096), (4096, 4096)]]
    ext = ng.extension()
    outs = [torch.empty(1, qw.N, dtype=torch.float16, device="cuda") for _, qw, _ in cases]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for (X, qw, _), o in zip(cases, outs):
                ext.gemv_w4a16(X, qw.qweight, qw.scales, 128, algo=algo, out=o)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for (_, _, ref), o in zip(cases, outs):
        check(o, ref, torch.float16)
    assert ext.device_status() == 0


@pytest.mark.parametrize("M,K,N,G", [(1, 4096, 14336, 128), (2, 14336, 4096, 128), (4, 4096, 4096, 64),
                                     (1, 2048, 4100, 256), (3, 1024, 132, 128), (1, 8192, 8192, 128)])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_ring_stream_k_matches_oracle_and_leaves_flags_zero(M, K, N, G, act):
    """The stream-K ring (algo 5, no explicit split, M <= 4): parity, run-to-run
    determinism, and the per-CTA flags in the workspace back at zero."""
    X, qw, ref = make_case(M, K, N, G, seed=M + K + N + G, act=act)
    ext = ng.extension()
    y = ext.gemv_w4a16(X, qw.qweight, qw.scales, G, algo=5)
    check(y, ref, X.dtype)
    for _ in range(3):
        assert torch.equal(y, ext.gemv_w4a16(X, qw.qweight, qw.scales, G, algo=5))
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    ws = ext.workspace(N, X.device, torch.cuda.current_stream().cuda_stream)
    total = ext.lib.ng_gemv_workspace_bytes(1, N)
    sm = torch.cuda.get_device_properties(X.device).multi_processor_count
    assert int(ws[total - 8 * sm: total].count_nonzero()) == 0  # 2 x SMs flags at the end


@pytest.mark.parametrize("M,K,N", [(9, 1024, 388), (12, 4096, 1028), (16, 4096, 14336), (16, 14336, 4096),
                                   (13, 2048, 132), (16, 8192, 8192)])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_ring_tensor_pipe_two_token_tiles(M, K, N, act):
    """algo 5 at M = 9..16 (two 8-token MMA tiles), and the default schedule
    that routes there."""
    X, qw, ref = make_case(M, K, N, 128, seed=M * 3 + N, act=act)
    check(ng.gemv(X, qw, algo=5), ref, X.dtype)
    check(ng.gemv(X, qw), ref, X.dtype)
    assert ng.extension().device_status() == 0


# More column tiles than SMs (the Llama gate|up and 70B widths): the default
# routing takes the ring with its own K split there, not one slice per tile.
@pytest.mark.parametrize("K,N", [(4096, 28672), (8192, 28672), (4096, 57344)])
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_wide_shapes_default_routing(K, N, M):
    X, qw, ref = make_case(M, K, N, 128, seed=K + N + 3 * M)
    y = ng.gemv(X, qw)
    check(y, ref, torch.float16)
    assert torch.equal(y, ng.gemv(X, qw, algo=5))


# ---------------------------------------------------------------------------
# Register-streamed tensor-pipe schedule (algo 6, M <= 16)
# ---------------------------------------------------------------------------
STREAM_CASES = [(1, 512, 256), (2, 256, 132), (3, 1024, 260), (4, 512, 512), (5, 2048, 132),
                (8, 512, 256), (1, 320 * 4, 1024), (2, 256, 4), (7, 8192, 388), (9, 1024, 388),
                (13, 2048, 132), (16, 512, 1028), (16, 4096, 4096)]


@pytest.mark.parametrize("M,K,N", STREAM_CASES)
@pytest.mark.parametrize("G", [64, 128, 256])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_stream_matches_oracle(M, K, N, G, act):
    if K % G:
        pytest.skip("K not a multiple of G")
    X, qw, ref = make_case(M, K, N, G, seed=M * 7 + N + G, act=act)
    check(ng.gemv(X, qw, algo=6), ref, X.dtype)
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("K,N", FULL + [(2048, 4096), (4096, 3072), (4096, 7168), (7168, 4096),
                                        (4096, 28672), (8192, 28672), (28672, 8192)])
@pytest.mark.parametrize("M", [1, 4, 8, 16])
def test_stream_full_size_shapes(K, N, M):
    X, qw, ref = make_case(M, K, N, 128, seed=K + N + M)
    check(ng.gemv(X, qw, algo=6), ref, torch.float16)
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8, 16])
def test_stream_split_invariance(splits):
    X, qw, ref = make_case(3, 4096, 1028, 128, seed=splits)
    y = ng.gemv(X, qw, splits=splits, algo=6)
    check(y, ref, torch.float16)
    assert torch.equal(y, ng.gemv(X, qw, splits=splits, algo=6))


@pytest.mark.parametrize("scale", [1e-4, 1.0, 300.0])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_stream_activation_magnitudes(scale, act):
    """The offsets removed per group (sum x * (offset + 8)) scale with X, so the
    relative error must not depend on the activations' magnitude."""
    x, q, s = qo.synthetic_case(4, 4096, 1024, group_size=128, seed=11, act="f16")
    xf = x.astype(np.float32) * scale
    qw = ng.QuantizedWeight(torch.from_numpy(q), torch.from_numpy(s), 128, 4096, 1024).to("cuda")
    dt = torch.float16 if act == "f16" else torch.bfloat16
    X = torch.from_numpy(xf).to(dt).cuda()
    xr = X.float().cpu().numpy()
    ref = xr @ qo.dequantize_np(q, s, 128, 4096).astype(np.float32)
    check(ng.gemv(X, qw, algo=6), ref, dt)


def test_stream_output_fully_written_and_back_to_back_in_graph():
    cases = [make_case(1, K, N, 128, seed=K + N) for K, N in [(4096, 14336), (14336, 4096), (4096, 4100)]]
    ext = ng.extension()
    outs = [torch.full((1, qw.N), float("nan"), dtype=torch.float16, device="cuda") for _, qw, _ in cases]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for (X, qw, _), o in zip(cases, outs):
                ext.gemv_w4a16(X, qw.qweight, qw.scales, 128, algo=6, out=o)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for (_, _, ref), o in zip(cases, outs):
        check(o, ref, torch.float16)
    assert ext.device_status() == 0
