"""Parity of the tcgen05 prefill GEMM (``gemm_w4a16``) with the CPU oracle.

The A operand the tensor cores read is the fp16 value ``fp16((u - 8) * s)`` --
bit-identical to the reference's ``dequantize`` -- so against the oracle
(fp32 X @ fp32(dequantize(W))) only fp32 summation order and the final output
rounding differ: expected max|err| / max|ref| ~ 2**-11 ~ 5e-4 (fp16 out) and
~ 2**-8 ~ 3.9e-3 (bf16 out, whose weights are also bf16-rounded, adding
~2**-9 / sqrt(K)-averaged noise).  Gate: 5e-3, plus the reference suite's own
max|err| / mean|ref| < 3e-2 (tests/test_gemm.py:27-34).

Edge cases follow the reference's tests/test_gemm.py: M of 1, 17, 64, 65, 128,
1000 (fractions of, exact multiples of and remainders past a tile) and
N = 128, 132 (a masked partial column tile), G = 64 / 128.
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
REF_TOL = 3e-2


def make_case(M, K, N, G=128, seed=0, act="f16"):
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=seed, act=act)
    qw = ng.QuantizedWeight(torch.from_numpy(q), torch.from_numpy(s), G, K, N).to("cuda")
    if act == "f16":
        X = torch.from_numpy(x).cuda()
    else:
        X = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    return x, q, s, X, qw


def oracle(x, q, s, G, K, act, rows=None):
    if rows is not None:
        x = x[rows]
    return c_oracle.matmul_f32(x, q, s, G, K, x_kind=act)


def check(y, ref, dtype):
    assert y.dtype == dtype
    yf = y.float().cpu().numpy()
    assert np.isfinite(yf).all()
    err = max_rel(yf, ref)
    assert err <= GATE, err
    assert mean_rel(yf, ref) < REF_TOL
    return err


@pytest.mark.parametrize("M", [1, 17, 64, 65, 128, 1000])
@pytest.mark.parametrize("N", [128, 132])
@pytest.mark.parametrize("G", [64, 128])
def test_gemm_edges_match_oracle(M, N, G):
    K = 256
    x, q, s, X, qw = make_case(M, K, N, G, seed=M + N + G)
    y = ng.gemm(X, qw)
    assert y.shape == (M, N)
    check(y, oracle(x, q, s, G, K, "f16"), torch.float16)


@pytest.mark.parametrize("bt", [16, 32, 64, 128, 192, 224, 240, 256])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_every_token_tile(bt, act):
    M, K, N, G = 300, 1024, 392, 128
    x, q, s, X, qw = make_case(M, K, N, G, seed=bt, act=act)
    y = ng.extension().gemm_w4a16(X, qw.qweight, qw.scales, G, tile_tokens=bt)
    check(y, oracle(x, q, s, G, K, act), X.dtype)


@pytest.mark.parametrize("M", [16, 128, 512, 2048])
@pytest.mark.parametrize("K,N", [(4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_config3_shapes_sampled_rows(M, K, N, act):
    """BASELINE config 3 shapes; rows sampled so the C oracle stays fast."""
    x, q, s, X, qw = make_case(M, K, N, 128, seed=M + K, act=act)
    y = ng.gemm(X, qw)
    rows = np.unique(np.linspace(0, M - 1, num=min(M, 12)).astype(int))
    check(y[torch.from_numpy(rows).cuda()], oracle(x, q, s, 128, K, act, rows), X.dtype)


def test_large_m_against_torch_fp32():
    """M = 8192: whole output vs fp32 torch matmul of the bit-exact dequantised weight."""
    M, K, N = 8192, 4096, 14336
    x, q, s, X, qw = make_case(M, K, N, 128, seed=5)
    y = ng.gemm(X, qw).float()
    ref = X.float() @ ng.dequant(qw).float()
    err = ((y - ref).abs().max() / ref.abs().max()).item()
    assert err <= GATE, err


def test_deterministic_and_poisoned_output():
    x, q, s, X, qw = make_case(333, 512, 260, 64, seed=9)
    out = torch.full((333, 260), float("nan"), dtype=torch.float16, device="cuda")
    ng.extension().gemm_w4a16(X, qw.qweight, qw.scales, 64, out=out)
    check(out, oracle(x, q, s, 64, 512, "f16"), torch.float16)
    assert torch.equal(out, ng.gemm(X, qw))
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("M", [17, 64, 512])
def test_matmul_dispatches_to_gemm_above_the_crossover(M):
    _, _, _, X, qw = make_case(M, 256, 128, 128, seed=1)
    assert M > ng.DECODE_MAX_M
    assert torch.equal(ng.matmul(X, qw), ng.gemm(X, qw))


def test_gemm_rejects_bad_shapes():
    _, _, _, X, qw = make_case(32, 256, 132, 128, seed=2)
    with pytest.raises(RuntimeError):
        ng.extension().gemm_w4a16(X[:, :192].contiguous(), qw.qweight[:24], qw.scales[:1].contiguous().expand(1, 132).contiguous(), 192)
    with pytest.raises(RuntimeError):
        ng.extension().gemm_w4a16(X, qw.qweight, qw.scales, 128, tile_tokens=48)


@pytest.mark.parametrize("M,K,N", [(16, 14336, 4096), (100, 14336, 4096), (128, 4096, 1024), (40, 8192, 2048),
                                   (16, 1024, 128), (200, 14336, 1028)])
@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_split_k_matches_oracle_deterministic_and_reusable(M, K, N, act):
    """Grids with fewer tiles than SMs are split along K through the workspace:
    parity, bit-identical repeats (the per-tile counters are re-armed), and the
    same answer as the unsplit kernel (no workspace) to summation order."""
    x, q, s, X, qw = make_case(M, K, N, 128, seed=M + K + N, act=act)
    ext = ng.extension()
    y = ext.gemm_w4a16(X, qw.qweight, qw.scales, 128)
    rows = np.unique(np.linspace(0, M - 1, num=min(M, 16)).astype(int))
    check(y[torch.from_numpy(rows).cuda()], oracle(x, q, s, 128, K, act, rows), X.dtype)
    for _ in range(3):
        assert torch.equal(y, ext.gemm_w4a16(X, qw.qweight, qw.scales, 128))
    y1 = torch.empty_like(y)
    st = ext.lib.ng_gemm_w4a16(X.data_ptr(), 1 if act == "bf16" else 0, qw.qweight.data_ptr(),
                               qw.scales.data_ptr(), y1.data_ptr(), M, K, N, 128, 0, None, 0,
                               torch.cuda.current_stream().cuda_stream)
    assert st == 0
    d = (y.float() - y1.float()).abs().max().item() / y1.float().abs().max().item()
    assert d < (1e-2 if act == "bf16" else 2e-3)  # ~two output ulps: only the fp32 summation order differs
    assert ext.device_status() == 0


def test_split_k_workspace_shared_across_shapes():
    """One workspace serves calls of different shapes in any order (the
    counters sit at a fixed place, partials never overlap them)."""
    ext = ng.extension()
    cases = [make_case(M, K, N, 128, seed=i, act=act) for i, (M, K, N, act) in
             enumerate([(300, 1024, 392, "bf16"), (16, 14336, 4096, "f16"), (40, 8192, 2048, "bf16"),
                        (128, 4096, 1024, "f16")])]
    first = [ext.gemm_w4a16(X, qw.qweight, qw.scales, 128, tile_tokens=32) for _, _, _, X, qw in cases]
    for _ in range(2):
        for (x, q, s, X, qw), y0 in zip(reversed(cases), reversed(first)):
            assert torch.equal(y0, ext.gemm_w4a16(X, qw.qweight, qw.scales, 128, tile_tokens=32))
    for (x, q, s, X, qw), y in zip(cases, first):
        M, K = X.shape
        rows = np.unique(np.linspace(0, M - 1, num=min(M, 8)).astype(int))
        act = "bf16" if X.dtype == torch.bfloat16 else "f16"
        check(y[torch.from_numpy(rows).cuda()], oracle(x, q, s, 128, K, act, rows), X.dtype)
