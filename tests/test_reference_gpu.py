"""The reference's own CUDA kernels, recompiled for the B200, beside this
library's on the same inputs.

``oracle/build_ref_cuda.py`` compiles the reference's unmodified
``csrc/{bindings.cpp,gemv_w4a16.cu,gemm_w4a16.cu,dequant_kernel.cu}`` (its
Ampere-era ``mma.sync`` / ``wmma`` kernels) for sm_100a into ``oracle/_ref/``.
These tests check that both implementations agree with the CPU oracle, and
print both timings on BASELINE config 1 (decode GEMV, the reference's
default ladder rung v4) and config 3 (prefill GEMM at M = 2048, its default
v6).  Timings are CUDA-graph replays over weights rotated past L2; run with
``-s`` to see them.  Skipped when the module has not been built.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import nibblegemm_b200 as ng
from oracle import build_ref_cuda, c_oracle
from oracle import quant_oracle as qo

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not build_ref_cuda.module_path(), reason="reference CUDA module not built")]

GATE = 5e-3


def _graph_us(fn, n=20):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(n):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        a.record(s)
        g.replay()
        b.record(s)
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / n


@pytest.mark.parametrize("workload,M,K,N", [("gemv", 1, 4096, 14336), ("gemm", 2048, 4096, 14336)])
def test_reference_kernels_on_b200_match_oracle_and_are_timed(workload, M, K, N):
    ref = build_ref_cuda.load_module()
    x, q, s = qo.synthetic_case(M, K, N, group_size=128, seed=11)
    X = torch.from_numpy(x).cuda()
    copies = 8  # 8 x 30 MB of packed weights: every launch reads HBM
    Ws = [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for _ in range(copies)]
    ext = ng.extension()
    if workload == "gemv":
        theirs = lambda i: ref.gemv_w4a16(X, Ws[i % copies][0], Ws[i % copies][1], 128, 4, 0, 0)  # noqa: E731
        ours = lambda i: ext.gemv_w4a16(X, Ws[i % copies][0], Ws[i % copies][1], 128)  # noqa: E731
    else:
        theirs = lambda i: ref.gemm_w4a16(X, Ws[i % copies][0], Ws[i % copies][1], 128, 6)  # noqa: E731
        ours = lambda i: ext.gemm_w4a16(X, Ws[i % copies][0], Ws[i % copies][1], 128)  # noqa: E731
    oracle = c_oracle.matmul_f32(x, q, s, 128, K)
    for name, fn in (("reference", theirs), ("nibblegemm_b200", ours)):
        y = fn(0).float().cpu().numpy()
        err = float(np.abs(y - oracle).max() / np.abs(oracle).max())
        assert err <= GATE, (name, err)
    t_ref, t_ours = _graph_us(theirs), _graph_us(ours)
    row = {"workload": workload, "M": M, "K": K, "N": N, "reference_us": round(t_ref, 2),
           "ours_us": round(t_ours, 2), "speedup": round(t_ref / t_ours, 2)}
    if workload == "gemv":
        nbytes = K * N // 2 + (K // 128) * N * 2 + M * K * 2 + M * N * 2
        row.update(reference_gbs=round(nbytes / t_ref / 1e3, 1), ours_gbs=round(nbytes / t_ours / 1e3, 1))
    else:
        row.update(reference_tflops=round(2 * M * K * N / t_ref / 1e6, 1),
                   ours_tflops=round(2 * M * K * N / t_ours / 1e6, 1))
    print("\nREFERENCE_ON_B200 " + json.dumps(row))
    assert ext.device_status() == 0
