"""The INT4 projection stack of a Llama-3-8B-shaped decode step on the GPU.

* TP = 1: every projection of two full-width layers against the CPU oracle
  (5e-3 max/max gate), and the step replayed from a CUDA graph gives the same
  outputs as eager execution.
* TP = 2 (needs two GPUs; skipped otherwise): NCCL ranks, each holding its
  Megatron shard, reproduce the TP = 1 outputs after the all-reduce.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from nibblegemm_b200.decode_step import LLAMA3_8B, ProjectionStackStep
from oracle import c_oracle
from tests.conftest import max_rel

pytestmark = pytest.mark.gpu


def _oracle(p):
    w = p.weight
    return c_oracle.matmul_f32(p.x.cpu().numpy(), w.qweight.cpu().numpy(), w.scales.cpu().numpy(),
                               w.group_size, w.K)


def test_tp1_projections_match_oracle_and_graph_replay():
    step = ProjectionStackStep(LLAMA3_8B, batch=1, layers=2)
    step.step()
    torch.cuda.synchronize()
    eager = [p.y.clone() for layer in step.proj for p in layer]
    for layer in step.proj:
        for p in layer:
            assert max_rel(p.y.float().cpu().numpy(), _oracle(p)) <= 5e-3, p.name
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        step.step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step.step()
    for p in (p for layer in step.proj for p in layer):
        p.y.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, p in zip(eager, (p for layer in step.proj for p in layer)):
        assert torch.equal(a, p.y), p.name


def _tp_worker(rank, world, port, q, reduce):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        step = ProjectionStackStep(LLAMA3_8B, batch=2, layers=1, rank=rank, world=world, reduce=reduce)
        step.step()
        torch.cuda.synchronize()
        outs = {}
        for p in step.proj[0]:
            y = p.y
            if p.style == "col":
                parts = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(parts, y)
                y = torch.cat(parts, dim=1)
            outs[p.name] = y.float().cpu()
        if rank == 0:
            ref = ProjectionStackStep(LLAMA3_8B, batch=2, layers=1)
            ref.step()
            torch.cuda.synchronize()
            errs = {p.name: float((outs[p.name] - p.y.float().cpu()).abs().max() / p.y.float().cpu().abs().max())
                    for p in ref.proj[0]}
            q.put(errs)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put({"worker error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("reduce,port", [("peer", 29711), ("nccl", 29713)])
def test_tp_matches_tp1(world, reduce, port):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port + 10 * world, q, reduce)) for r in range(world)]
    for p in procs:
        p.start()
    errs = q.get(timeout=150)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert "worker error" not in errs, errs
    for name, e in errs.items():
        assert e <= 5e-3, (name, e)
