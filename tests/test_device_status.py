"""Failure reporting without a GPU fault: a kernel whose bounded wait runs out
records NG_ERR_DEVICE_TIMEOUT in the device error word, and the Python surface
turns it into an exception.

The wait is made to run out on the host's terms: the peer all-reduce is run in
one process with world = 2, its "peer" buffer is a second local allocation, and
no second rank ever raises the flag the kernel waits for.  The kernel gives up
after its 1 s limit, finishes with the data it has, and returns; the context
stays usable.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import nibblegemm_b200 as ng
from nibblegemm_b200 import _lib

pytestmark = pytest.mark.gpu


def _ipc_buffer(lib, nbytes):
    base, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    _lib.check(lib.ng_ipc_alloc(nbytes, ctypes.byref(base), handle), "ng_ipc_alloc")
    return base.value


def test_bounded_wait_timeout_reaches_python_and_clears():
    ext = ng.extension()
    lib = ext.lib
    ng.check_device()  # start clean
    n = 256
    nbytes = lib.ng_allreduce_buffer_bytes(2, n)
    mine, fake_peer = _ipc_buffer(lib, nbytes), _ipc_buffer(lib, nbytes)
    try:
        data = torch.ones(n, dtype=torch.float16, device="cuda")
        epochs = torch.zeros(16, dtype=torch.int32, device="cuda")
        peers = (ctypes.c_void_p * 2)(mine, fake_peer)
        st = lib.ng_allreduce_sum(data.data_ptr(), _lib.NG_DTYPE_F16, n, peers, 0, 2, n,
                                  epochs.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert st == _lib.NG_OK
        with pytest.raises(_lib.NibbleError, match="bounded pipeline wait"):
            ng.check_device()
        ng.check_device()  # reported once, then cleared
        # the context is still usable
        x = torch.randn(4, 4, device="cuda")
        assert torch.isfinite(x @ x).all()
    finally:
        torch.cuda.synchronize()
        lib.ng_ipc_free(fake_peer)
        lib.ng_ipc_free(mine)


def test_debug_checks_raise_on_bad_index_at_the_op():
    """With debug checks on, an op that flags the error word raises right away."""
    ext = ng.extension()
    table = torch.randn(10, 64, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 64, dtype=torch.float16, device="cuda")
    bad = torch.tensor([10], dtype=torch.int64, device="cuda")
    st = ext.lib.ng_embed_tokens(bad.data_ptr(), None, None, table.data_ptr(), 0, 1, 64, 10, out.data_ptr(),
                                 None, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    with pytest.raises(_lib.NibbleError, match="outside its table"):
        ng.check_device()
    ng.set_debug_checks(True)
    try:
        x, q, s = (torch.randn(1, 256, dtype=torch.float16, device="cuda"),
                   torch.zeros(32, 128, dtype=torch.int32, device="cuda"),
                   torch.ones(2, 128, dtype=torch.float16, device="cuda"))
        y = ng.extension().gemv_w4a16(x, q, s, 128)  # a clean op passes the check
        assert y.shape == (1, 128)
    finally:
        ng.set_debug_checks(False)
