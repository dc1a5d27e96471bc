"""The INT4 projection stack of a Llama-shaped decode step, optionally tensor-parallel.

The reference's model-level measurement (arvindcr4/nibblegemm
``bench/bench_model.py:43-125``, "layers" mode) runs the seven decoder
projections -- q, k, v, o, gate, up, down -- of every layer at batch 1 through
``ng.matmul`` and times the whole step eagerly and under a CUDA graph.  This
module does the same with this library's kernels, with three differences that
the B200 setting requires:

* every layer has its own weights (the reference replays one layer's 109 MB,
  which would sit in B200's 126 MB L2 and turn an HBM benchmark into an L2 one);
* weights are generated on the device as random INT4 codes and fp16 scales with
  the BASELINE distributions (random-init model; no checkpoint exists offline);
* Megatron-style tensor parallelism over ``torch.distributed`` (NCCL): q/k/v/
  gate/up are column-parallel (each rank holds N/TP output columns), o/down are
  row-parallel (each rank holds K/TP input rows, a valid packed weight because
  quantisation groups run along K) and their partial outputs are summed with
  one all-reduce each -- two per layer.

As in the reference, the projections read preallocated activations (no data
dependency between them), so the step measures weight streaming plus, under
TP, the all-reduce latency.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .ops import extension
from .quant import QuantizedWeight

LLAMA3_8B = dict(layers=32, hidden=4096, kv=1024, intermediate=14336)
LLAMA3_70B = dict(layers=80, hidden=8192, kv=1024, intermediate=28672)

#: (name, K, N, parallel style) of one decoder layer; "col" shards N, "row" shards K.
def layer_projections(cfg) -> List[tuple]:
    h, kv, inter = cfg["hidden"], cfg["kv"], cfg["intermediate"]
    return [("q", h, h, "col"), ("k", h, kv, "col"), ("v", h, kv, "col"), ("o", h, h, "row"),
            ("gate", h, inter, "col"), ("up", h, inter, "col"), ("down", inter, h, "row")]


def random_weight(K: int, N: int, group_size: int, generator: torch.Generator,
                  device) -> QuantizedWeight:
    """Packed INT4 weight with codes uniform in 0..15 and scales |N(0,1)|*0.02+1e-3."""
    words = torch.randint(-2**31, 2**31, (K // 8, N), dtype=torch.int64, generator=generator,
                          device=device).to(torch.int32)
    scales = (torch.randn(K // group_size, N, generator=generator, device=device).abs() * 0.02
              + 1e-3).to(torch.float16)
    return QuantizedWeight(words, scales, group_size, K, N)


def shard_weight(full: QuantizedWeight, style: str, rank: int, world: int) -> QuantizedWeight:
    """This rank's Megatron shard: N/world columns ("col") or K/world rows ("row")."""
    if style == "col":
        n = full.N // world
        return full.shard_columns(rank * n, (rank + 1) * n)
    k = full.K // world
    return full.shard_rows(rank * k, (rank + 1) * k)


def shard_input(x: torch.Tensor, style: str, rank: int, world: int) -> torch.Tensor:
    """Input a rank multiplies: the whole activation ("col") or its K slice ("row")."""
    if style == "col":
        return x
    k = x.size(1) // world
    return x[:, rank * k:(rank + 1) * k].contiguous()


@dataclass
class Projection:
    name: str
    style: str
    weight: QuantizedWeight  # this rank's shard
    x: torch.Tensor          # [M, K_shard] input
    y: torch.Tensor          # [M, N_shard] output


class ProjectionStackStep:
    """One decode step through every INT4 projection of a Llama-shaped model.

    ``rank`` / ``world`` select this process's tensor-parallel shard; with
    ``world > 1`` a ``torch.distributed`` process group (NCCL) must already be
    initialised.  ``step()`` enqueues the whole token on the current stream and
    is capturable into one CUDA graph.
    """

    def __init__(self, cfg=LLAMA3_8B, batch: int = 1, group_size: int = 128, rank: int = 0,
                 world: int = 1, device: Optional[torch.device] = None, seed: int = 0,
                 dtype: torch.dtype = torch.float16, layers: Optional[int] = None,
                 reduce: str = "peer"):
        if reduce not in ("peer", "nccl"):
            raise ValueError(f"reduce must be 'peer' or 'nccl', not {reduce!r}")
        self.cfg, self.batch, self.rank, self.world = cfg, batch, rank, world
        self.reduce = reduce
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.layers = layers if layers is not None else cfg["layers"]
        self.ext = extension()
        gen = torch.Generator(device=self.device)
        self.proj: List[List[Projection]] = []
        x_full = {}
        projs = layer_projections(cfg)
        for li in range(self.layers):
            layer = []
            for pi, (name, K, N, style) in enumerate(projs):
                if style == "col" and N % (world * 4):
                    raise ValueError(f"{name}: N={N} does not split into {world} column shards")
                if style == "row" and K % (world * group_size):
                    raise ValueError(f"{name}: K={K} does not split into {world} group-aligned shards")
                # Every rank draws the same full weight (seeded by layer and
                # projection) and keeps its shard, so TP=n reproduces TP=1.
                gen.manual_seed(seed * 1_000_003 + li * 16 + pi)
                full = random_weight(K, N, group_size, gen, self.device)
                w = shard_weight(full, style, rank, world)
                del full
                if K not in x_full:
                    gen.manual_seed(seed * 1_000_003 + 999_983 + K)
                    x_full[K] = torch.randn(batch, K, generator=gen, device=self.device).to(dtype)
                x = shard_input(x_full[K], style, rank, world)
                layer.append(Projection(name, style, w, x,
                                        torch.empty(batch, w.N, dtype=dtype, device=self.device)))
            self.proj.append(layer)
        # Row-parallel outputs are summed across ranks: by default with the
        # one-shot peer-memory all-reduce (ng_allreduce_sum), else NCCL.
        self._peer = None
        if world > 1 and reduce == "peer":
            from .comm import PeerAllReduce
            max_n = max(p.y.numel() for layer in self.proj for p in layer if p.style == "row")
            self._peer = PeerAllReduce(max_n, device=self.device)

    @property
    def weight_bytes(self) -> int:
        """INT4 codes + scales this rank streams per token."""
        return sum(p.weight.weight_bytes for layer in self.proj for p in layer)

    def step(self) -> None:
        """Launch one token's projections (and, under TP, the row-parallel all-reduces)."""
        ext = self.ext
        for layer in self.proj:
            for p in layer:
                if p.x.size(0) <= 16:
                    # The cluster GEMV (algo 1 fp16 / 2 bf16): measured fastest in
                    # this mixed chain of shapes, where the ring kernels' 219 KB
                    # CTAs keep the next projection from starting early.
                    ext.gemv_w4a16(p.x, p.weight.qweight, p.weight.scales, p.weight.group_size,
                                   algo=2 if p.x.dtype == torch.bfloat16 else 1, out=p.y)
                else:
                    ext.gemm_w4a16(p.x, p.weight.qweight, p.weight.scales, p.weight.group_size, out=p.y)
                if p.style == "row" and self.world > 1:
                    if self._peer is not None:
                        self._peer(p.y)
                    else:
                        torch.distributed.all_reduce(p.y)
