"""The allocation-free GEMV entry point (``ng_gemv_w4a16_noalloc``).

It serves callers that cannot allocate device memory when they call the GEMV
(code running inside an allocator or memory hook, plugins whose host owns all
allocation, allocation-free inference loops): instead of a caller-provided
workspace it uses a fixed array in the library's device data.  Here it is
called through the C ABI and compared with the regular entry point
(``ng_gemv_w4a16``, tensor-pipe schedule, caller workspace) on the same
inputs, twice in a row, within the GEMV suite's 5e-3 gate -- the second call
checks that the state the first call leaves in the shared array does not leak.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import nibblegemm_b200 as ng
from nibblegemm_b200 import _lib
from oracle import c_oracle
from oracle import quant_oracle as qo

pytestmark = pytest.mark.gpu

GATE = 5e-3  # max|y - y_ref| / max|y_ref|, the tolerance of tests/test_gemv.py


@pytest.mark.parametrize("M,K,N,G,act", [(1, 4096, 14336, 128, "f16"), (5, 1024, 4100, 64, "f16"),
                                         (16, 2048, 1028, 128, "bf16")])
def test_noalloc_matches_regular_entry_point_twice(M, K, N, G, act):
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=M + K + N, act=act)
    qw = ng.QuantizedWeight(torch.from_numpy(q), torch.from_numpy(s), G, K, N).to("cuda")
    if act == "f16":
        X, code = torch.from_numpy(x).cuda(), _lib.NG_DTYPE_F16
    else:
        X, code = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(), _lib.NG_DTYPE_BF16
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream

    # regular entry point: tensor-pipe schedule with a caller-provided workspace
    ref = torch.empty((M, N), dtype=X.dtype, device="cuda")
    ws = torch.zeros(lib.ng_gemv_workspace_bytes(M, N), dtype=torch.uint8, device="cuda")
    st = lib.ng_gemv_w4a16(X.data_ptr(), code, qw.qweight.data_ptr(), qw.scales.data_ptr(),
                           ref.data_ptr(), M, K, N, G, 0, 0, 3, ws.data_ptr(), ws.numel(), stream)
    assert st == _lib.NG_OK, lib.ng_status_string(st)

    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=X.dtype, device="cuda")
        st = lib.ng_gemv_w4a16_noalloc(X.data_ptr(), code, qw.qweight.data_ptr(),
                                       qw.scales.data_ptr(), y.data_ptr(), M, K, N, G, stream)
        assert st == _lib.NG_OK, lib.ng_status_string(st)
        assert lib.ng_device_status(stream) == _lib.NG_OK
        a, b = y.float(), ref.float()
        assert torch.isfinite(a).all(), f"call {call}"
        err = ((a - b).abs().max() / b.abs().max()).item()
        assert err <= GATE, (call, err)
    # and against the CPU oracle directly, so a fault shared by both GPU paths shows
    oracle = c_oracle.matmul_f32(x, q, s, G, K, x_kind=act)
    y32 = y.float().cpu().numpy()
    assert float(np.abs(y32 - oracle).max() / np.abs(oracle).max()) <= GATE


def test_noalloc_rejects_bad_arguments():
    lib = _lib.load()
    FAKE = 0x1000
    assert lib.ng_gemv_w4a16_noalloc(None, 0, FAKE, FAKE, FAKE, 1, 256, 128, 128, None) == 1
    assert lib.ng_gemv_w4a16_noalloc(FAKE, 0, FAKE, FAKE, FAKE, 17, 256, 128, 128, None) == 3
