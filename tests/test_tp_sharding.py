"""Tensor-parallel sharding of the decode step (host logic, CPU, gloo).

Two ranks split a projection Megatron-style with the same helpers the decode
step uses (``shard_weight`` / ``shard_input``); each rank computes its partial
with the CPU oracle, the row-parallel partials are summed with an all-reduce,
and the gathered result must equal the unsharded oracle result.  No GPU.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nibblegemm_b200.decode_step import layer_projections, shard_input, shard_weight, LLAMA3_8B
from nibblegemm_b200.quant import QuantizedWeight
from oracle import c_oracle
from oracle import quant_oracle as qo


def _worker(rank, world, port, K, N, G, style, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, qweight, scales = qo.synthetic_case(3, K, N, group_size=G, seed=K + N)
        full = QuantizedWeight(torch.from_numpy(qweight), torch.from_numpy(scales), G, K, N)
        w = shard_weight(full, style, rank, world)
        xs = shard_input(torch.from_numpy(x), style, rank, world).numpy()
        part = torch.from_numpy(c_oracle.matmul_f32(xs, w.qweight.numpy(), w.scales.numpy(), G, w.K))
        if style == "row":
            dist.all_reduce(part)
            out = part
        else:
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            out = torch.cat(parts, dim=1)
        if rank == 0:
            ref = c_oracle.matmul_f32(x, qweight, scales, G, K)
            q.put(float(np.abs(out.numpy() - ref).max() / np.abs(ref).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("style,K,N", [("col", 512, 256), ("row", 1024, 128)])
def test_two_rank_shards_reassemble_the_full_product(style, K, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (K + N) % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, K, N, 128, style, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=10) < 1e-5


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_llama3_8b_shapes_shard_evenly(world):
    for name, K, N, style in layer_projections(LLAMA3_8B):
        if style == "col":
            assert N % (world * 4) == 0, name
        else:
            assert (K // world) % 128 == 0, name
