"""The tensor-parallel reduction (``ng_allreduce_sum`` / ``PeerAllReduce``).

CPU: the buffer-size arithmetic and argument validation (no launch).
GPU (two devices): the one-shot peer-memory sum against an fp32 sum in rank
order rounded once -- bit-exact, since the kernel computes exactly that --
over message sizes that exercise the vector and scalar copy paths and the
CTA split, repeated calls (both slot parities), and CUDA-graph replay.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from nibblegemm_b200 import _lib

FAKE = 1 << 20


def _codes():
    from tests.test_capi import status_codes
    return status_codes()


def test_buffer_bytes():
    lib = _lib.load()
    # 2 parities x 16 CTAs x world slots of ceil(n/16) rounded to 8 elems, 2 B each,
    # then 2 x 16 x 8 uint32 flags.
    for world, n in [(2, 4096), (8, 4096), (4, 1), (2, 14336 * 4)]:
        slot = ((n + 15) // 16 + 7) // 8 * 8
        assert lib.ng_allreduce_buffer_bytes(world, n) == 2 * 16 * world * slot * 2 + 2 * 16 * 8 * 4
    assert lib.ng_allreduce_buffer_bytes(0, 4096) == 0
    assert lib.ng_allreduce_buffer_bytes(9, 4096) == 0


def test_argument_validation():
    lib = _lib.load()
    c = _codes()
    ptrs = (ctypes.c_void_p * 2)(FAKE, FAKE)
    assert lib.ng_allreduce_sum(None, 0, 16, ptrs, 0, 2, 64, FAKE, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_allreduce_sum(FAKE, 0, 16, None, 0, 2, 64, FAKE, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_allreduce_sum(FAKE, 0, 16, ptrs, 0, 2, 64, None, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_allreduce_sum(FAKE, 5, 16, ptrs, 0, 2, 64, FAKE, None) == c["NG_ERR_BAD_DTYPE"]
    assert lib.ng_allreduce_sum(FAKE, 0, 16, ptrs, 2, 2, 64, FAKE, None) == c["NG_ERR_BAD_ARGUMENT"]
    assert lib.ng_allreduce_sum(FAKE, 0, 16, ptrs, 0, 9, 64, FAKE, None) == c["NG_ERR_BAD_ARGUMENT"]
    assert lib.ng_allreduce_sum(FAKE, 0, 0, ptrs, 0, 2, 64, FAKE, None) == c["NG_ERR_BAD_SHAPE"]
    assert lib.ng_allreduce_sum(FAKE, 0, 65, ptrs, 0, 2, 64, FAKE, None) == c["NG_ERR_BAD_SHAPE"]
    assert lib.ng_allreduce_sum(FAKE + 1, 0, 16, ptrs, 0, 2, 64, FAKE, None) == c["NG_ERR_MISALIGNED"]
    assert lib.ng_ipc_open(None, None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_ipc_close(None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_ipc_free(None) == c["NG_ERR_NULL_POINTER"]
    assert lib.ng_ipc_alloc(64, None, None) == c["NG_ERR_NULL_POINTER"]


def _rank_input(n, dtype, rank, call):
    g = torch.Generator().manual_seed(1000 * call + 7 * rank + n)
    return torch.randn(n, generator=g).to(dtype)


def _expected(n, dtype, world, call):
    acc = torch.zeros(n, dtype=torch.float32)
    for r in range(world):
        acc += _rank_input(n, dtype, r, call).float()
    return acc.to(dtype)


SIZES = [4096, 14336, 1, 8, 333, 4096 * 16 + 24]
MAX_N = max(SIZES)


def _ar_worker(rank, world, port, q):
    import torch.distributed as dist
    from nibblegemm_b200.comm import PeerAllReduce
    from nibblegemm_b200 import ops
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    fails = []
    try:
        ar = PeerAllReduce(MAX_N)
        call = 0
        for dtype in (torch.float16, torch.bfloat16):
            for n in SIZES:
                for _ in range(3):  # both parities, then the first again
                    t = _rank_input(n, dtype, rank, call).cuda()
                    ar(t)
                    if not torch.equal(t.cpu(), _expected(n, dtype, world, call)):
                        fails.append((str(dtype), n, call))
                    call += 1
        # graph replay: inputs refreshed in place between replays
        n = 14336
        buf = torch.empty(n, dtype=torch.float16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                ar(buf)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(4):
            buf.copy_(_rank_input(n, torch.float16, rank, call).cuda())
            g.replay()
            if not torch.equal(buf.cpu(), _expected(n, torch.float16, world, call)):
                fails.append(("graph", n, call))
            call += 1
        torch.cuda.synchronize()
        status = ops.extension().device_status()
        q.put((rank, fails, status))
        dist.barrier()
        ar.close()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, [repr(e)], -1))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ar_worker, args=(r, world, 29723 + world, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=150) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, fails, status in results:
        assert not fails, (rank, fails[:5])
        assert status == 0, (rank, status)


def _fused_worker(rank, world, port, q):
    """ng_gemv_w4a16_allreduce against ng_gemv_w4a16 + an NCCL all-reduce of the
    partials, and every rank's Y bit-identical, over several calls (graph too)."""
    import ctypes
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import nibblegemm_b200 as ng
        from nibblegemm_b200 import _lib
        from nibblegemm_b200.comm import PeerBuffers
        lib = _lib.load()
        fails = []
        for (M, K, N, mode) in [(1, 14336, 4096, 0), (3, 4096, 4096, 0), (2, 1792, 4096, 2), (16, 1024, 1028, 0)]:
            g = torch.Generator().manual_seed(K + N + M)
            Kr = K // world
            W = torch.randn(K, N, generator=g) * 0.02
            qw = ng.quantize(W[rank * Kr:(rank + 1) * Kr].contiguous(), 128 if Kr % 128 == 0 else 64).to("cuda")
            xin = torch.randn(M, (2 * K if mode == 2 else K), generator=g).half().cuda()
            if mode == 2:  # gate | up of this rank's slice
                x_full = torch.cat([xin[:, rank * Kr:(rank + 1) * Kr], xin[:, K + rank * Kr:K + (rank + 1) * Kr]], 1).contiguous()
                act = torch.empty(M, Kr, dtype=torch.float16, device="cuda")
                lib.ng_silu_mul(x_full.data_ptr(), act.data_ptr(), 0, M, Kr, torch.cuda.current_stream().cuda_stream)
                x_gemv = act
            else:
                x_full = xin[:, rank * Kr:(rank + 1) * Kr].contiguous()
                x_gemv = x_full
            ref = ng.extension().gemv_w4a16(x_gemv, qw.qweight, qw.scales, qw.group_size, algo=1).float()
            dist.all_reduce(ref)
            bufs = PeerBuffers(lib.ng_gemv_allreduce_buffer_bytes(world, N))
            for call in range(3):
                y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
                st = lib.ng_gemv_w4a16_allreduce(x_full.data_ptr(), 0, qw.qweight.data_ptr(), qw.scales.data_ptr(),
                                                 y.data_ptr(), M, Kr, N, qw.group_size, mode, bufs.ptrs, rank, world,
                                                 torch.cuda.current_stream().cuda_stream)
                if st != 0:
                    fails.append(("status", M, K, N, st))
                    break
                torch.cuda.synchronize()
                err = float((y.float() - ref).abs().max() / ref.abs().max())
                if not err <= 5e-3:
                    fails.append(("err", M, K, N, call, err))
                allys = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(allys, y)
                if not all(torch.equal(a, allys[0]) for a in allys):
                    fails.append(("ranks differ", M, K, N, call))
            # CUDA-graph replays: the per-slice call counters live on the device
            y = torch.empty((M, N), dtype=torch.float16, device="cuda")
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=s):
                    lib.ng_gemv_w4a16_allreduce(x_full.data_ptr(), 0, qw.qweight.data_ptr(), qw.scales.data_ptr(),
                                                y.data_ptr(), M, Kr, N, qw.group_size, mode, bufs.ptrs, rank,
                                                world, s.cuda_stream)
            torch.cuda.current_stream().wait_stream(s)
            dist.barrier()
            for _ in range(4):
                gr.replay()
                torch.cuda.synchronize()
                err = float((y.float() - ref).abs().max() / ref.abs().max())
                if not err <= 5e-3:
                    fails.append(("graph err", M, K, N, err))
            dist.barrier()
            bufs.close()
        status = ng.extension().device_status()
        q.put((rank, fails, status))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, [repr(e)], -1))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gemv_allreduce(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, 29823 + world, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, fails, status in results:
        assert not fails, (rank, fails[:5])
        assert status == 0, (rank, status)
