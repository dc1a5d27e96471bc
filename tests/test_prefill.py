"""Prefill of a prompt through ``Llama3Decoder.prefill``: every projection as a
tensor-core GEMM over all prompt tokens, RoPE + KV append for the run
(``ng_rope_prefill``) and causal GQA attention over the cache
(``ng_attn_prefill``).

* The attention kernel against a torch fp32 causal restatement, including a
  sequence that continues after rows the cache already holds.
* A full prefill against the fp32 restatement of the model
  (``tests/test_decode_model.py``) fed the same tokens one position at a time;
  gate max|err| / max|ref| <= 2e-2 (fp16) / 4e-2 (bf16), as for decode.
* Prefill followed by decode steps against decode steps alone (teacher
  forced): the caches and the next token's logits agree.
"""
from __future__ import annotations

import math
import os

import pytest
import torch
import torch.multiprocessing as mp

import nibblegemm_b200 as ng
from nibblegemm_b200 import _lib
from nibblegemm_b200.decode_model import Llama3Decoder
from tests.test_decode_model import TINY, RefModel, _rel

pytestmark = pytest.mark.gpu

_DT = {torch.float16: _lib.NG_DTYPE_F16, torch.bfloat16: _lib.NG_DTYPE_BF16}


def _attn_ref(q, kc, vc, pos0, S):
    """fp32 causal GQA attention: q [B, S, Hq, D], caches [B, ctx, Hkv, D]."""
    B, _, Hq, D = q.shape
    Hkv = kc.size(2)
    out = torch.empty(B, S, Hq, D, device=q.device)
    for b in range(B):
        p0 = int(pos0[b])
        K, V = kc[b, :p0 + S].float(), vc[b, :p0 + S].float()
        for h in range(Hq):
            kh = h // (Hq // Hkv)
            s = (q[b, :, h].float() @ K[:, kh].t()) / math.sqrt(D)  # [S, T]
            mask = torch.arange(p0 + S, device=q.device)[None, :] > (p0 + torch.arange(S, device=q.device))[:, None]
            s = s.masked_fill(mask, float("-inf"))
            out[b, :, h] = torch.softmax(s, -1) @ V[:, kh]
    return out


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,S,Hq,Hkv,pos0", [(1, 64, 4, 1, [0]), (2, 130, 8, 2, [0, 5]), (1, 1, 8, 8, [3]),
                                             (1, 200, 16, 2, [64])])
def test_attn_prefill_matches_fp32_causal_attention(dtype, B, S, Hq, Hkv, pos0):
    D, ctx = 128, 320
    g = torch.Generator(device="cuda").manual_seed(S + Hq)
    q = (torch.randn(B, S, Hq, D, generator=g, device="cuda") * 2).to(dtype)
    kc = torch.randn(B, ctx, Hkv, D, generator=g, device="cuda").to(dtype)
    vc = torch.randn(B, ctx, Hkv, D, generator=g, device="cuda").to(dtype)
    pos = torch.tensor(pos0, dtype=torch.int32, device="cuda")
    out = torch.full((B, S, Hq, D), float("nan"), device="cuda", dtype=dtype)
    lib = ng.extension().lib
    st = lib.ng_attn_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), out.data_ptr(),
                             _DT[dtype], B, S, Hq, Hkv, D, ctx, 1.0 / math.sqrt(D),
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    ref = _attn_ref(q, kc, vc, pos, S)
    assert torch.isfinite(out.float()).all()
    tol = 1e-2 if dtype == torch.float16 else 3e-2
    assert _rel(out, ref) <= tol


def test_attn_prefill_rejects_bad_arguments():
    lib = ng.extension().lib
    F = 0x1000
    assert lib.ng_attn_prefill(None, F, F, F, F, 0, 1, 4, 4, 1, 128, 64, 1.0, None) == 1  # null pointer
    assert lib.ng_attn_prefill(F, F, F, F, F, 0, 1, 4, 4, 1, 64, 64, 1.0, None) == 3     # D != 128
    assert lib.ng_attn_prefill(F, F, F, F, F, 0, 1, 4, 6, 4, 128, 64, 1.0, None) == 3    # Hq % Hkv
    assert lib.ng_rope_prefill(F, F, F, F, F, 0, 2, 0, 4, 1, 128, 5e5, 64, None) == 3   # S < 1


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("batch,S", [(1, 37), (2, 70)])
def test_prefill_matches_fp32_restatement(dtype, batch, S):
    m = Llama3Decoder(TINY, batch=batch, max_ctx=96, dtype=dtype, attn_splits=4)
    ref = RefModel(m)
    g = torch.Generator().manual_seed(S)
    toks = torch.randint(0, TINY["vocab"], (batch, S), generator=g).cuda()
    m.prefill(toks)
    torch.cuda.synchronize()
    for s in range(S):  # the restatement, one position at a time
        xn_ref, logits_ref = ref.step(toks[:, s], torch.full((batch,), s, device="cuda"))
    tol = 2e-2 if dtype == torch.float16 else 4e-2
    assert _rel(m.xn, xn_ref) <= tol
    assert _rel(m.logits, logits_ref) <= tol
    lg = m.logits.float()
    assert torch.equal(lg.gather(1, m.tokens[:, None]).squeeze(1), lg.max(1).values)
    assert torch.equal(m.pos.cpu(), torch.full((batch,), S, dtype=torch.int32))
    # the caches hold the prompt's K / V rows (K rotated) as the restatement does
    for li in range(TINY["layers"]):
        assert _rel(m.k_cache[li][:, :S], ref.kc[li][:, :S]) <= tol
        assert _rel(m.v_cache[li][:, :S], ref.vc[li][:, :S]) <= tol
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("S", [5, 40])
def test_prefill_then_decode_matches_decode_only(S):
    """Prefill of S tokens then 3 decode steps == S + 3 teacher-forced decode steps."""
    batch = 2
    a = Llama3Decoder(TINY, batch=batch, max_ctx=64, attn_splits=4)
    b = Llama3Decoder(TINY, batch=batch, max_ctx=64, attn_splits=4)
    g = torch.Generator().manual_seed(7 + S)
    toks = torch.randint(0, TINY["vocab"], (batch, S + 3), generator=g).cuda()
    a.prefill(toks[:, :S])
    for s in range(S):
        b.tokens.copy_(toks[:, s])
        b.step()
    torch.cuda.synchronize()
    assert _rel(a.logits, b.logits.float()) <= 2e-2
    for t in range(3):
        a.tokens.copy_(toks[:, S + t])
        b.tokens.copy_(toks[:, S + t])
        a.step()
        b.step()
        torch.cuda.synchronize()
        assert _rel(a.logits, b.logits.float()) <= 2e-2, t
    for li in range(TINY["layers"]):
        assert _rel(a.k_cache[li][:, :S + 3], b.k_cache[li][:, :S + 3].float()) <= 2e-2
    assert torch.equal(a.pos, b.pos)
    assert ng.extension().device_status() == 0


def _tp_prefill_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        cfg = dict(TINY, kv_heads=max(TINY["kv_heads"], world))  # one key/value head per rank at least
        toks = torch.randint(0, cfg["vocab"], (2, 40), generator=torch.Generator().manual_seed(3)).cuda()
        m = Llama3Decoder(cfg, batch=2, max_ctx=48, rank=rank, world=world, attn_splits=2, reduce="nccl")
        out = [m.prefill(toks).cpu().tolist()]
        for _ in range(3):
            m.step()
            out.append(m.tokens.cpu().tolist())
        torch.cuda.synchronize()
        if rank == 0:
            r = Llama3Decoder(cfg, batch=2, max_ctx=48, attn_splits=2)
            ref = [r.prefill(toks).cpu().tolist()]
            for _ in range(3):
                r.step()
                ref.append(r.tokens.cpu().tolist())
            q.put({"tp": out, "tp1": ref})
    except Exception as e:  # report instead of leaving the parent waiting
        q.put({"worker error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_prefill_then_decode_generates_the_tp1_tokens(world):
    """Megatron-sharded prefill (column-parallel q|k|v, gate|up; row-parallel
    o, down with an NCCL all-reduce of the [batch x S, hidden] partials) and
    the decode steps after it give the TP = 1 tokens."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_prefill_worker, args=(r, world, 29811 + world, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=150)
    for p in procs:
        p.join(timeout=60)
    assert "worker error" not in res, res
    assert res["tp"] == res["tp1"]
