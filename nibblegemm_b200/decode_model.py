"""A full Llama-3-architecture decode step on this library's kernels.

BASELINE config 4/5 asks for tokens/s of a whole decode step: embedding,
per layer RMSNorm -> q/k/v -> RoPE + KV-cache append -> GQA attention over the
cache -> o -> residual + RMSNorm -> gate/up -> SwiGLU -> down -> residual, then
the final norm, the fp16 lm_head and an argmax, captured in one CUDA graph and
tensor-parallel over the ranks of one node.  The reference's own step is
projections only (arvindcr4/nibblegemm ``bench/bench_model.py:57-86``); the
projections here are exactly its W4A16 ops (``gemv_w4a16``), the rest are the
kernels of ``csrc/decode_ops.cu``.

Layout choices:
* q|k|v and gate|up are each ONE packed INT4 weight (column concatenation of
  the projections, per rank), so a layer is four GEMV launches;
* tensor parallelism is Megatron-style: q/k/v by heads and gate/up by
  intermediate columns (column-parallel), o and down by rows (row-parallel,
  followed by an all-reduce -- the peer-memory kernel or NCCL); each rank
  keeps its KV heads' cache; the lm_head is vocab-parallel and the argmax is
  combined with one all-gather of (value, index) pairs;
* weights are random-init (seeded N(0, 0.02)) and quantised round-to-nearest
  on the device with the reference's RTN rule; every rank draws the same full
  weights and keeps its shard, so TP = n computes the TP = 1 model.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib
from .ops import DECODE_MAX_M, extension
from .quant import QuantizedWeight, quantize_on_device

LLAMA3_8B_MODEL = dict(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128,
                       intermediate=14336, vocab=128256, rope_theta=500000.0, eps=1e-5)
LLAMA3_70B_MODEL = dict(layers=80, hidden=8192, heads=64, kv_heads=8, head_dim=128,
                        intermediate=28672, vocab=128256, rope_theta=500000.0, eps=1e-5)

_DT = {torch.float16: _lib.NG_DTYPE_F16, torch.bfloat16: _lib.NG_DTYPE_BF16}


def _cat_cols(ws):
    return QuantizedWeight(torch.cat([w.qweight for w in ws], 1).contiguous(),
                           torch.cat([w.scales for w in ws], 1).contiguous(), ws[0].group_size,
                           ws[0].K, sum(w.N for w in ws))


class Llama3Decoder:
    """Random-init INT4 Llama-3 decoder for batch ``batch`` decode steps.

    ``step()`` advances every sequence by one token (reads ``self.tokens``,
    writes the argmax token back into it) and is capturable into one CUDA graph;
    ``self.pos`` (device int32 [batch]) is the position being written.
    """

    def __init__(self, cfg=LLAMA3_8B_MODEL, batch: int = 1, max_ctx: int = 1024,
                 layers: Optional[int] = None, rank: int = 0, world: int = 1,
                 device: Optional[torch.device] = None, seed: int = 0,
                 dtype: torch.dtype = torch.float16, group_size: int = 128,
                 reduce: str = "peer", attn_splits: int = 32, fused_rope: bool = True,
                 fused_norm: bool = True, wide_split: bool = True, keep_logits: bool = True,
                 gemv_algo: Optional[int] = None, fold_act: bool = True,
                 fold_silu: Optional[bool] = None, fold_attn: Optional[bool] = None):
        self.cfg, self.batch, self.rank, self.world, self.dtype = cfg, batch, rank, world, dtype
        self.keep_logits = keep_logits  # write the (rounded) logits besides the fused argmax
        self.gemv_algo = gemv_algo      # None: per-shape choice below; else this ng_gemv_w4a16 algo everywhere
        # SwiGLU folded into the down GEMV and the attention combine into the o GEMV
        # (needs the fused RoPE + attention kernel, which can leave its partials)
        # Measured in the Llama-3-8B step: the SwiGLU fold is neutral at batch 1 and a
        # loss at batch 4; the combine fold is a loss (every column tile of o re-does
        # the combine of its heads), so it is off unless asked for.
        self.fold_silu = (fold_act and batch <= 2) if fold_silu is None else fold_silu
        self.fold_attn = (False if fold_attn is None else fold_attn) and fused_rope
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.layers = layers if layers is not None else cfg["layers"]
        self.max_ctx, self.attn_splits, self.fused_rope = max_ctx, attn_splits, fused_rope
        # The folded norm re-reduces each token's row in every CTA: worth it for a
        # few tokens only (measured: a loss at batch 16).
        self.fused_norm = fused_norm and batch <= 4
        # Projections with more 128-column tiles than SMs (gate|up) run faster on
        # the library's split ring than on the cluster kernel the batch <= 4
        # chain uses elsewhere, so they keep their norm separate.  Measured in
        # the full 8B step: 1029 -> 1220 tok/s at batch 4, but 464 -> 405 at
        # batch 1, where the cluster kernel's free SMs let the next kernel start.
        self.wide_split = wide_split and batch >= 2
        self._sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        H, D = cfg["hidden"], cfg["head_dim"]
        hq, hkv, inter = cfg["heads"] // world, cfg["kv_heads"] // world, cfg["intermediate"] // world
        if cfg["heads"] % world or cfg["kv_heads"] % world or cfg["intermediate"] % world:
            raise ValueError(f"{world} ranks do not divide the heads / intermediate size")
        self.hq, self.hkv, self.inter = hq, hkv, inter
        self.ext = extension()
        dev, g = self.device, torch.Generator(device=self.device)

        def dense(K, N, tag):
            g.manual_seed(seed * 1_000_003 + tag)
            return torch.randn(K, N, generator=g, device=dev) * 0.02

        def q4(W):
            return quantize_on_device(W, group_size)

        self.w = []
        for li in range(self.layers):
            base = 100 * li
            wq, wk, wv = q4(dense(H, cfg["heads"] * D, base + 1)), q4(dense(H, cfg["kv_heads"] * D, base + 2)), \
                q4(dense(H, cfg["kv_heads"] * D, base + 3))
            qkv = _cat_cols([wq.shard_columns(rank * hq * D, (rank + 1) * hq * D),
                             wk.shard_columns(rank * hkv * D, (rank + 1) * hkv * D),
                             wv.shard_columns(rank * hkv * D, (rank + 1) * hkv * D)])
            del wq, wk, wv
            wo = q4(dense(cfg["heads"] * D, H, base + 4)).shard_rows(rank * hq * D, (rank + 1) * hq * D)
            wg = q4(dense(H, cfg["intermediate"], base + 5))
            wu = q4(dense(H, cfg["intermediate"], base + 6))
            gu = _cat_cols([wg.shard_columns(rank * inter, (rank + 1) * inter),
                            wu.shard_columns(rank * inter, (rank + 1) * inter)])
            del wg, wu
            wd = q4(dense(cfg["intermediate"], H, base + 7)).shard_rows(rank * inter, (rank + 1) * inter)
            g.manual_seed(seed * 1_000_003 + base + 8)
            n1 = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dtype)
            n2 = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dtype)
            self.w.append(dict(qkv=qkv, o=wo, gu=gu, down=wd, attn_norm=n1, mlp_norm=n2))
        g.manual_seed(seed * 1_000_003 + 99_999)
        V = cfg["vocab"]
        self.embed = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(dtype)
        vl = (V + world - 1) // world
        self.v0, self.v1 = rank * vl, min(V, (rank + 1) * vl)
        g.manual_seed(seed * 1_000_003 + 99_998)
        self.lm_head = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(dtype)[self.v0:self.v1].contiguous()
        self.final_norm = torch.ones(H, device=dev, dtype=dtype)
        torch.cuda.synchronize(dev)

        B = batch
        # one cache per sequence: [batch, max_ctx, kv heads, head_dim] per layer
        self.k_cache = [torch.zeros(B, max_ctx, hkv, D, device=dev, dtype=dtype) for _ in range(self.layers)]
        self.v_cache = [torch.zeros(B, max_ctx, hkv, D, device=dev, dtype=dtype) for _ in range(self.layers)]
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.ctx = torch.ones(B, dtype=torch.int32, device=dev)
        self.res = torch.zeros(B, H, device=dev, dtype=dtype)
        self.res2 = torch.zeros(B, H, device=dev, dtype=dtype)  # ping-pong partner (folded norms)
        self.xn = torch.empty(B, H, device=dev, dtype=dtype)
        self.xemb = torch.empty(B, H, device=dev, dtype=dtype)
        self.qkv = torch.empty(B, (hq + 2 * hkv) * D, device=dev, dtype=dtype)
        self.q = torch.empty(B, hq * D, device=dev, dtype=dtype)
        self.attn = torch.empty(B, hq * D, device=dev, dtype=dtype)
        self.o = torch.empty(B, H, device=dev, dtype=dtype)
        self.gu = torch.empty(B, 2 * inter, device=dev, dtype=dtype)
        self.act = torch.empty(B, inter, device=dev, dtype=dtype)
        self.down = torch.empty(B, H, device=dev, dtype=dtype)
        self.logits = torch.empty(B, self.v1 - self.v0, device=dev, dtype=dtype)
        # Per-token argmax keys of the fused head (LLONG_MIN = empty; the token
        # decode at the end of the step re-arms them).
        self.keys = torch.full((B,), -(2 ** 63), dtype=torch.int64, device=dev)
        self.attn_ws = torch.empty(self.ext.lib.ng_attn_workspace_bytes(B, hq, attn_splits),
                                   dtype=torch.uint8, device=dev)
        self._peer = None
        self._fused = None  # (o buffers, down buffers) of the fused GEMV + all-reduce
        self.reduce = reduce if world > 1 else None
        if world > 1 and reduce in ("peer", "fused"):
            from .comm import PeerAllReduce
            self._peer = PeerAllReduce(B * H, device=dev)
        if world > 1 and reduce == "fused":
            # The row-parallel o / down projections reduce inside their GEMV (cluster
            # schedule, up to 4 tokens); larger batches keep the separate all-reduce.
            from .comm import PeerBuffers
            nbytes = self.ext.lib.ng_gemv_allreduce_buffer_bytes(world, H)
            self._fused = (PeerBuffers(nbytes, device=dev), PeerBuffers(nbytes, device=dev))
        self.weight_bytes = sum(w[k].weight_bytes for w in self.w for k in ("qkv", "o", "gu", "down"))

    # -- helpers ---------------------------------------------------------------
    def _stream(self):
        return torch.cuda.current_stream().cuda_stream

    def _wide(self, w):
        return self.wide_split and (w.N + 127) // 128 > self._sms

    def _gemv(self, x, w, out):
        # batch <= 4: the cluster GEMV (algo 1 / 2), fastest in this mixed chain of
        # shapes; larger batches and wide projections: the library's default
        # routing (tensor-pipe ring)
        algo = (2 if x.dtype == torch.bfloat16 else 1) if x.size(0) <= 4 and not self._wide(w) else 0
        if self.gemv_algo is not None:
            algo = self.gemv_algo
        self.ext.gemv_w4a16(x, w.qweight, w.scales, w.group_size, algo=algo, out=out)

    def _allreduce(self, t):
        if self.world == 1:
            return
        if self._peer is not None:
            self._peer(t)
        else:
            torch.distributed.all_reduce(t)

    def _norm_gemv(self, x, res_in, res_out, norm_w, wq, out):
        """RMSNorm folded into the projection's activation staging."""
        _lib.check(self.ext.lib.ng_gemv_w4a16_rmsnorm(
            x.data_ptr(), res_in.data_ptr(), res_out.data_ptr(), norm_w.data_ptr(), float(self.cfg["eps"]),
            _DT[self.dtype], wq.qweight.data_ptr(), wq.scales.data_ptr(), out.data_ptr(), x.size(0),
            wq.K, wq.N, wq.group_size, self._stream()), "gemv_w4a16_rmsnorm")

    def _norm(self, x, res, w, y):
        _lib.check(self.ext.lib.ng_rmsnorm(x.data_ptr(), res.data_ptr() if res is not None else None,
                                           w.data_ptr(), y.data_ptr(), _DT[self.dtype], x.size(0),
                                           x.size(1), float(self.cfg["eps"]), self._stream()),
                   "rmsnorm")

    def launches_per_step(self) -> int:
        """Kernels of this library one ``step()`` launches (torch's own ops and
        NCCL's are not counted)."""
        L = len(self.w)
        # 4 GEMVs; attention partials (+ combine unless folded into o; + RoPE kernel
        # unless fused); SwiGLU unless folded into down
        per_layer = 4 + 1 + (0 if self.fold_attn else 1) + (0 if self.fused_rope else 1) + \
            (0 if self.fold_silu else 1)
        norms = sum(1 for w in self.w for k in ("qkv", "gu") if not (self.fused_norm and not self._wide(w[k])))
        fused = self._fused is not None and self.batch <= 4 and not self.fold_attn
        peer = 2 * L if (self._peer is not None and not fused) else 0
        return L * per_layer + norms + peer + 1 + 1 + 1 + 1  # embed, final norm, head, token decode

    # -- prefill -----------------------------------------------------------------
    def _prefill_buffers(self, S: int) -> dict:
        """Activations of a prefill of S tokens per sequence (kept for reuse)."""
        bufs = getattr(self, "_pf", None)
        if bufs is not None and bufs["S"] == S:
            return bufs
        cfg, D, dev, dt = self.cfg, self.cfg["head_dim"], self.device, self.dtype
        M, H = self.batch * S, cfg["hidden"]
        e = lambda n: torch.empty(M, n, device=dev, dtype=dt)  # noqa: E731
        self._pf = dict(S=S, res=e(H), xemb=e(H), xn=e(H), qkv=e((self.hq + 2 * self.hkv) * D),
                        q=e(self.hq * D), attn=e(self.hq * D), o=e(H), gu=e(2 * self.inter),
                        act=e(self.inter), down=e(H))
        return self._pf

    def _proj(self, x, w, out):
        """A projection of a prefill: the tensor-core GEMM, or the GEMV for a few rows."""
        if x.size(0) <= DECODE_MAX_M:
            self.ext.gemv_w4a16(x, w.qweight, w.scales, w.group_size, out=out)
        else:
            self.ext.gemm_w4a16(x, w.qweight, w.scales, w.group_size, out=out)

    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """Run the prompt ``tokens`` (int64 [batch, S] on the device) through the
        model at positions ``self.pos + 0 .. S - 1`` of each sequence: every
        projection as one [batch * S]-row tensor-core GEMM, RoPE + KV append for
        the whole run, causal attention over the cache, and the head on each
        sequence's last position.  Fills the KV caches, writes the next token of
        each sequence into ``self.tokens`` (and the last position's logits into
        ``self.logits``), advances ``self.pos`` by S and returns ``self.tokens``,
        so ``step()`` continues the sequences."""
        cfg, D, B = self.cfg, self.cfg["head_dim"], self.batch
        if tokens.dim() != 2 or tokens.size(0) != B or tokens.dtype != torch.int64 or not tokens.is_cuda:
            raise ValueError(f"tokens must be an int64 CUDA tensor [{B}, S]")
        S = tokens.size(1)
        tokens = tokens.contiguous()
        lib, dt, st = self.ext.lib, _DT[self.dtype], self._stream()
        H, M, eps = cfg["hidden"], B * S, float(cfg["eps"])
        f = self._prefill_buffers(S)
        _lib.check(lib.ng_embed_tokens(tokens.data_ptr(), None, None, self.embed.data_ptr(), dt, M, H,
                                       cfg["vocab"], f["xemb"].data_ptr(), f["res"].data_ptr(), st),
                   "embed_tokens")
        delta, res = f["xemb"], f["res"]

        def norm(x, w, y, rows=M):
            _lib.check(lib.ng_rmsnorm(x.data_ptr(), res.data_ptr(), w.data_ptr(), y.data_ptr(), dt, rows,
                                      H, eps, st), "rmsnorm")

        for li, w in enumerate(self.w):
            norm(delta, w["attn_norm"], f["xn"])
            self._proj(f["xn"], w["qkv"], f["qkv"])
            _lib.check(lib.ng_rope_prefill(f["qkv"].data_ptr(), f["q"].data_ptr(), self.k_cache[li].data_ptr(),
                                           self.v_cache[li].data_ptr(), self.pos.data_ptr(), dt, B, S,
                                           self.hq, self.hkv, D, float(cfg["rope_theta"]), self.max_ctx, st),
                       "rope_prefill")
            _lib.check(lib.ng_attn_prefill(f["q"].data_ptr(), self.k_cache[li].data_ptr(),
                                           self.v_cache[li].data_ptr(), self.pos.data_ptr(), f["attn"].data_ptr(),
                                           dt, B, S, self.hq, self.hkv, D, self.max_ctx, 1.0 / math.sqrt(D), st),
                       "attn_prefill")
            self._proj(f["attn"], w["o"], f["o"])
            if self.world > 1:
                torch.distributed.all_reduce(f["o"])
            norm(f["o"], w["mlp_norm"], f["xn"])
            self._proj(f["xn"], w["gu"], f["gu"])
            _lib.check(lib.ng_silu_mul(f["gu"].data_ptr(), f["act"].data_ptr(), dt, M, self.inter, st), "silu_mul")
            self._proj(f["act"], w["down"], f["down"])
            if self.world > 1:
                torch.distributed.all_reduce(f["down"])
            delta = f["down"]
        # the head reads each sequence's last position only
        for b in range(B):
            r = b * S + S - 1
            _lib.check(lib.ng_rmsnorm(delta[r].data_ptr(), res[r].data_ptr(), self.final_norm.data_ptr(),
                                      self.xn[b].data_ptr(), dt, 1, H, eps, st), "rmsnorm")
        _lib.check(lib.ng_lm_head_argmax(self.xn.data_ptr(), self.lm_head.data_ptr(), dt, B, self.v1 - self.v0,
                                         H, self.v0, self.logits.data_ptr() if self.keep_logits else None,
                                         self.keys.data_ptr(), st), "lm_head_argmax")
        if self.world > 1:
            torch.distributed.all_reduce(self.keys, op=torch.distributed.ReduceOp.MAX)
        _lib.check(lib.ng_embed_tokens(None, self.keys.data_ptr(), self.tokens.data_ptr(), self.embed.data_ptr(),
                                       dt, B, H, cfg["vocab"], None, None, st), "embed_tokens")
        self.pos.add_(S)
        return self.tokens

    # -- the step ----------------------------------------------------------------
    def step(self, advance: bool = True) -> None:
        """One token per sequence at position ``self.pos``; ``advance=False``
        keeps the position (a benchmark holding the context length fixed)."""
        cfg, D, B = self.cfg, self.cfg["head_dim"], self.batch
        lib, dt = self.ext.lib, _DT[self.dtype]
        torch.add(self.pos, 1, out=self.ctx)
        # embedding gather; the residual stream of the step starts at zero
        _lib.check(lib.ng_embed_tokens(self.tokens.data_ptr(), None, None, self.embed.data_ptr(), dt, B,
                                       cfg["hidden"], cfg["vocab"], self.xemb.data_ptr(), self.res.data_ptr(),
                                       self._stream()), "embed_tokens")
        delta = self.xemb
        # The residual stream lives in `res`; a folded norm writes h to the other
        # buffer of the pair and the stream moves there (fixed per model, so a
        # captured graph replays the same buffers).
        res, spare = self.res, self.res2

        def norm_proj(x_in, norm_w, wq, out):
            nonlocal res, spare
            if self.fused_norm and not self._wide(wq):
                self._norm_gemv(x_in, res, spare, norm_w, wq, out)
                res, spare = spare, res
            else:
                self._norm(x_in, res, norm_w, self.xn)
                self._gemv(self.xn, wq, out)

        for li, w in enumerate(self.w):
            norm_proj(delta, w["attn_norm"], w["qkv"], self.qkv)
            if self.fused_rope:  # RoPE + KV append inside the attention kernel
                _lib.check(lib.ng_attn_decode_rope(
                    self.qkv.data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                    self.pos.data_ptr(), None if self.fold_attn else self.attn.data_ptr(), dt, B,
                    self.hq, self.hkv, D,
                    self.max_ctx, self.attn_splits, 1.0 / math.sqrt(D), float(cfg["rope_theta"]),
                    self.attn_ws.data_ptr(), self.attn_ws.numel(), self._stream()), "attn_decode_rope")
            else:
                _lib.check(lib.ng_rope_append(self.qkv.data_ptr(), self.q.data_ptr(),
                                              self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                                              self.pos.data_ptr(), dt, B, self.hq, self.hkv, D,
                                              float(cfg["rope_theta"]), self.max_ctx, self._stream()),
                           "rope_append")
                _lib.check(lib.ng_attn_decode(self.q.data_ptr(), self.k_cache[li].data_ptr(),
                                              self.v_cache[li].data_ptr(), self.ctx.data_ptr(),
                                              self.attn.data_ptr(), dt, B, self.hq, self.hkv, D,
                                              self.max_ctx, self.attn_splits, 1.0 / math.sqrt(D),
                                              self.attn_ws.data_ptr(), self.attn_ws.numel(),
                                              self._stream()), "attn_decode")
            fused_ar = self._fused is not None and B <= 4 and not self.fold_attn
            if fused_ar:  # o projection + its tensor-parallel reduction, one kernel
                wo = w["o"]
                _lib.check(lib.ng_gemv_w4a16_allreduce(
                    self.attn.data_ptr(), dt, wo.qweight.data_ptr(), wo.scales.data_ptr(), self.o.data_ptr(),
                    B, wo.K, wo.N, wo.group_size, 0, self._fused[0].ptrs, self.rank, self.world,
                    self._stream()), "gemv_w4a16_allreduce")
            elif self.fold_attn:  # o projection with the attention combine in its staging
                wo = w["o"]
                _lib.check(lib.ng_gemv_w4a16_attn(self.attn_ws.data_ptr(), self.attn_splits, dt,
                                                  wo.qweight.data_ptr(), wo.scales.data_ptr(),
                                                  self.o.data_ptr(), B, wo.K, wo.N, wo.group_size,
                                                  self._stream()), "gemv_w4a16_attn")
            else:
                self._gemv(self.attn, w["o"], self.o)
            if not fused_ar:
                self._allreduce(self.o)
            norm_proj(self.o, w["mlp_norm"], w["gu"], self.gu)
            if fused_ar:  # down projection (SwiGLU folded in or not) + its reduction
                wd = w["down"]
                src = self.gu if self.fold_silu else self.act
                if not self.fold_silu:
                    _lib.check(lib.ng_silu_mul(self.gu.data_ptr(), self.act.data_ptr(), dt, B, self.inter,
                                               self._stream()), "silu_mul")
                _lib.check(lib.ng_gemv_w4a16_allreduce(
                    src.data_ptr(), dt, wd.qweight.data_ptr(), wd.scales.data_ptr(), self.down.data_ptr(),
                    B, wd.K, wd.N, wd.group_size, 2 if self.fold_silu else 0, self._fused[1].ptrs, self.rank,
                    self.world, self._stream()), "gemv_w4a16_allreduce")
            elif self.fold_silu:  # down projection with SwiGLU in its staging
                wd = w["down"]
                _lib.check(lib.ng_gemv_w4a16_silu(self.gu.data_ptr(), dt, wd.qweight.data_ptr(),
                                                  wd.scales.data_ptr(), self.down.data_ptr(), B, wd.K,
                                                  wd.N, wd.group_size, self._stream()), "gemv_w4a16_silu")
            else:
                _lib.check(lib.ng_silu_mul(self.gu.data_ptr(), self.act.data_ptr(), dt, B, self.inter,
                                           self._stream()), "silu_mul")
                self._gemv(self.act, w["down"], self.down)
            if not fused_ar:
                self._allreduce(self.down)
            delta = self.down
        self._norm(delta, res, self.final_norm, self.xn)
        # fp16 lm_head with the argmax fused into its epilogue (vocab shard per rank)
        _lib.check(lib.ng_lm_head_argmax(self.xn.data_ptr(), self.lm_head.data_ptr(), dt, B, self.v1 - self.v0,
                                         cfg["hidden"], self.v0,
                                         self.logits.data_ptr() if self.keep_logits else None,
                                         self.keys.data_ptr(), self._stream()), "lm_head_argmax")
        if self.world > 1:  # one MAX all-reduce of B int64 keys combines the vocabulary shards
            torch.distributed.all_reduce(self.keys, op=torch.distributed.ReduceOp.MAX)
        # next token ids out of the keys (which are re-armed for the next step)
        _lib.check(lib.ng_embed_tokens(None, self.keys.data_ptr(), self.tokens.data_ptr(), self.embed.data_ptr(),
                                       dt, B, cfg["hidden"], cfg["vocab"], None, None, self._stream()),
                   "embed_tokens")
        if advance:
            self.pos.add_(1)
