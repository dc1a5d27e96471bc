"""The full decode step (``Llama3Decoder``) against a plain torch fp32
restatement of the same model on the same (dequantised, bit-exact) weights:
embedding, RMSNorm, RoPE (rotate-half, theta 500000), GQA attention over the
KV cache, SwiGLU, residuals, final norm, lm_head.  Teacher-forced tokens so
errors do not compound through the argmax.  Gate: max|err| / max|ref| <= 2e-2
on the final hidden state and the logits (fp16 activations and residual stream
vs fp32 throughout, two layers)."""
from __future__ import annotations

import math
import os

import pytest
import torch
import torch.multiprocessing as mp

import nibblegemm_b200 as ng
from nibblegemm_b200.decode_model import Llama3Decoder

pytestmark = pytest.mark.gpu

TINY = dict(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, intermediate=1024, vocab=1000,
            rope_theta=500000.0, eps=1e-5)


def _deq(w):
    return ng.extension().dequant_w4(w.qweight, w.scales, w.group_size).float()


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _rope(x, pos, theta):  # x [B, heads, D]
    D = x.size(-1)
    i = torch.arange(D // 2, device=x.device, dtype=torch.float32)
    ang = pos.float()[:, None] * theta ** (-2 * i / D)  # [B, D/2]
    c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
    a, b = x[..., :D // 2], x[..., D // 2:]
    return torch.cat([a * c - b * s, b * c + a * s], -1)


class RefModel:
    def __init__(self, m: Llama3Decoder):
        self.m, c = m, m.cfg
        self.W = [{k: _deq(w[k]) for k in ("qkv", "o", "gu", "down")} | {"n1": w["attn_norm"], "n2": w["mlp_norm"]}
                  for w in m.w]
        self.kc = [torch.zeros(m.batch, m.max_ctx, c["kv_heads"], c["head_dim"], device=m.device) for _ in m.w]
        self.vc = [torch.zeros_like(k) for k in self.kc]

    def step(self, tokens, pos):
        m, c = self.m, self.m.cfg
        H, D, hq, hkv, eps = c["hidden"], c["head_dim"], c["heads"], c["kv_heads"], c["eps"]
        res = torch.zeros(tokens.numel(), H, device=m.device)
        delta = m.embed[tokens].float()
        for li, W in enumerate(self.W):
            res = res + delta
            xn = _rms(res, W["n1"], eps)
            qkv = xn @ W["qkv"]
            q = _rope(qkv[:, :hq * D].view(-1, hq, D), pos, c["rope_theta"])
            k = _rope(qkv[:, hq * D:(hq + hkv) * D].view(-1, hkv, D), pos, c["rope_theta"])
            v = qkv[:, (hq + hkv) * D:].view(-1, hkv, D)
            out = torch.empty(tokens.numel(), hq, D, device=m.device)
            for b in range(tokens.numel()):
                p = int(pos[b])
                self.kc[li][b, p], self.vc[li][b, p] = k[b], v[b]
                K, V = self.kc[li][b, :p + 1], self.vc[li][b, :p + 1]  # [T, hkv, D]
                for h in range(hq):
                    kh = h // (hq // hkv)
                    s = (K[:, kh] @ q[b, h]) / math.sqrt(D)
                    out[b, h] = torch.softmax(s, 0) @ V[:, kh]
            o = out.reshape(-1, hq * D) @ W["o"]
            res = res + o
            xn = _rms(res, W["n2"], eps)
            gu = xn @ W["gu"]
            I = gu.size(1) // 2
            act = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            delta = act @ W["down"]
        res = res + delta
        xn = _rms(res, m.final_norm, eps)
        return xn, xn @ m.lm_head.float().t()


def _rel(a, b):
    return float((a.float() - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("batch", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fused,sms,fold", [(True, None, True), (True, None, False), (False, None, True),
                                             (True, 14, True), (True, 1, True)])
def test_decoder_matches_fp32_restatement(batch, dtype, fused, sms, fold):
    m = Llama3Decoder(TINY, batch=batch, max_ctx=64, dtype=dtype, attn_splits=4, fused_rope=fused,
                      fused_norm=fused, fold_silu=fold, fold_attn=fold)
    if sms is not None:
        # pretend a smaller GPU: 14 SMs makes only gate|up (16 column tiles)
        # "wide" (separate norm + split ring, the residual stream changes buffer
        # once per layer), 1 SM makes every projection wide
        m._sms = sms
    ref = RefModel(m)
    g = torch.Generator().manual_seed(batch)
    for step in range(6):
        toks = torch.randint(0, TINY["vocab"], (batch,), generator=g).cuda()
        pos = m.pos.clone()
        m.tokens.copy_(toks)
        m.step()
        torch.cuda.synchronize()
        xn_ref, logits_ref = ref.step(toks, pos)
        tol = 2e-2 if dtype == torch.float16 else 4e-2
        assert _rel(m.xn, xn_ref) <= tol, (step, _rel(m.xn, xn_ref))
        assert _rel(m.logits, logits_ref) <= tol, (step, _rel(m.logits, logits_ref))
        # the fused argmax works on fp32 logits: the chosen token's rounded logit is the maximum
        lg = m.logits.float()
        assert torch.equal(lg.gather(1, m.tokens[:, None]).squeeze(1), lg.max(1).values)
    assert ng.extension().device_status() == 0


def test_decoder_graph_replay_matches_eager_and_never_writes_past_the_cache():
    m = Llama3Decoder(TINY, batch=2, max_ctx=8, attn_splits=2)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m.step()
        torch.cuda.synchronize()
        m.pos.zero_()
        m.tokens.zero_()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            m.step()
    torch.cuda.current_stream().wait_stream(s)
    m.pos.zero_()
    m.tokens.zero_()
    seen = []
    for _ in range(12):  # past max_ctx = 8: cache rows beyond it are never written
        g.replay()
        torch.cuda.synchronize()
        seen.append(m.tokens.clone())
    e = Llama3Decoder(TINY, batch=2, max_ctx=8, attn_splits=2)
    for i in range(8):  # eager run of the positions inside the cache
        e.step()
        torch.cuda.synchronize()
        assert torch.equal(e.tokens, seen[i]), i
    assert ng.extension().device_status() == 0


def _tp_worker(rank, world, port, q, reduce="peer"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        # Key/value heads are sharded, not replicated: at least one per rank.
        cfg = dict(TINY, kv_heads=max(TINY["kv_heads"], world))
        m = Llama3Decoder(cfg, batch=2, max_ctx=16, rank=rank, world=world, attn_splits=2, reduce=reduce)
        toks = []
        for _ in range(5):
            m.step()
            torch.cuda.synchronize()
            toks.append(m.tokens.cpu())
        if rank == 0:
            r = Llama3Decoder(cfg, batch=2, max_ctx=16, attn_splits=2)
            ref = []
            for _ in range(5):
                r.step()
                torch.cuda.synchronize()
                ref.append(r.tokens.cpu())
            q.put({"tp": [t.tolist() for t in toks], "tp1": [t.tolist() for t in ref]})
    except Exception as e:  # report instead of leaving the parent waiting
        q.put({"worker error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("reduce", ["peer", "fused", "nccl"])
def test_decoder_tp_generates_the_tp1_tokens(world, reduce):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29741 + world + 10 * ["peer", "fused", "nccl"].index(reduce)
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q, reduce)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=150)
    for p in procs:
        p.join(timeout=60)
    assert "worker error" not in res, res
    assert res["tp"] == res["tp1"]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,V", [(1, 128256), (3, 1000), (5, 7)])
def test_argmax_kernel_matches_torch_and_rearms(dtype, M, V):
    ext = ng.extension()
    scratch = torch.zeros(M, dtype=torch.int64, device="cuda")
    for trial in range(3):
        x = torch.randn(M, V, generator=torch.Generator().manual_seed(trial)).to(dtype).cuda()
        x[:, V // 2] = x.max() if trial == 2 else x[:, V // 2]  # a tie on the last trial
        val = torch.empty(M, dtype=torch.float32, device="cuda")
        idx = torch.empty(M, dtype=torch.int64, device="cuda")
        st = ext.lib.ng_argmax(x.data_ptr(), 1 if dtype == torch.bfloat16 else 0, M, V, 100,
                               scratch.data_ptr(), val.data_ptr(), idx.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        ref_v, ref_i = x.float().max(dim=1)  # torch returns the first maximal index
        assert torch.equal(idx - 100, ref_i) and torch.equal(val, ref_v)
        assert int(scratch.count_nonzero()) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (3, 512, 1028), (16, 1024, 256)])
def test_rmsnorm_folded_gemv_matches_separate_kernels(dtype, M, K, N):
    """ng_gemv_w4a16_rmsnorm == ng_rmsnorm then the cluster GEMV (same rounding
    of the normalised activations), and the new residual equals x + residual."""
    ext, lib = ng.extension(), ng.extension().lib
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    res = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    nw = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(dtype)
    qw = ng.quantize(torch.randn(K, N) * 0.02).to("cuda")
    code = 1 if dtype == torch.bfloat16 else 0
    st = torch.cuda.current_stream().cuda_stream
    y = torch.empty(M, N, dtype=dtype, device="cuda")
    res_out = torch.empty_like(res)
    assert lib.ng_gemv_w4a16_rmsnorm(x.data_ptr(), res.data_ptr(), res_out.data_ptr(), nw.data_ptr(), 1e-5,
                                     code, qw.qweight.data_ptr(), qw.scales.data_ptr(), y.data_ptr(),
                                     M, K, N, 128, st) == 0
    r2, xn = res.clone(), torch.empty_like(x)
    assert lib.ng_rmsnorm(x.data_ptr(), r2.data_ptr(), nw.data_ptr(), xn.data_ptr(), code, M, K, 1e-5, st) == 0
    ref = ext.gemv_w4a16(xn, qw.qweight, qw.scales, 128, algo=2 if code else 1)
    torch.cuda.synchronize()
    assert torch.equal(res_out, r2)
    d = (y.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert d < (1e-2 if code else 2e-3), d
    assert ext.device_status() == 0


def _keys_to_tokens(keys, M):
    ext = ng.extension()
    tok = torch.empty(M, dtype=torch.int64, device="cuda")
    table = torch.zeros(1, 8, dtype=torch.float16, device="cuda")
    st = ext.lib.ng_embed_tokens(None, keys.data_ptr(), tok.data_ptr(), table.data_ptr(), 0, M, 8,
                                 2 ** 31, None, None, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return tok


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,V,H", [(1, 128256 // 8, 4096), (3, 1000, 512), (8, 37, 256), (11, 4099, 1024)])
def test_lm_head_argmax_matches_fp32_and_rearms(dtype, M, V, H):
    """The fused head: logits (rounded to dtype) against an fp32 torch
    restatement, the argmax against the fp32 maximum (an index whose fp32
    logit is within the fp32 summation-order noise of the maximum), a planted
    clear winner exactly, and the keys re-armed by the token decode."""
    ext = ng.extension()
    g = torch.Generator().manual_seed(M * 7 + V)
    x = torch.randn(M, H, generator=g).to(dtype).cuda()
    w = (torch.randn(V, H, generator=g) * 0.02).to(dtype).cuda()
    win = [(m * 997 + 5) % V for m in range(M)]
    for m in range(M):
        w[win[m]] = (x[m].float() * 0.05).to(dtype)  # a clear winner per token
    keys = torch.full((M,), -(2 ** 63), dtype=torch.int64, device="cuda")
    logits = torch.empty(M, V, dtype=dtype, device="cuda")
    dt = 1 if dtype == torch.bfloat16 else 0
    st = ext.lib.ng_lm_head_argmax(x.data_ptr(), w.data_ptr(), dt, M, V, H, 123, logits.data_ptr(),
                                   keys.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    ref = x.float() @ w.float().t()
    assert _rel(logits, ref) <= (4e-3 if dtype == torch.float16 else 8e-3)
    tok = _keys_to_tokens(keys, M) - 123
    assert tok.tolist() == win
    assert int((keys != -(2 ** 63)).sum()) == 0  # re-armed
    # without a planted winner: the chosen logit is the fp32 maximum up to summation noise
    w2 = (torch.randn(V, H, generator=g) * 0.02).to(dtype).cuda()
    st = ext.lib.ng_lm_head_argmax(x.data_ptr(), w2.data_ptr(), dt, M, V, H, 0, None, keys.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 0
    tok = _keys_to_tokens(keys, M)
    ref2 = x.float() @ w2.float().t()
    chosen = ref2.gather(1, tok[:, None]).squeeze(1)
    assert torch.all(chosen >= ref2.max(1).values - 1e-4 * ref2.abs().max())
    assert ext.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_embed_tokens_gathers_zeroes_and_flags_bad_ids(dtype):
    ext = ng.extension()
    V, H, M = 1000, 4096, 5
    table = torch.randn(V, H).to(dtype).cuda()
    tokens = torch.tensor([0, 999, 17, 17, 500], dtype=torch.int64, device="cuda")
    out = torch.empty(M, H, dtype=dtype, device="cuda")
    res = torch.full((M, H), 3.0, dtype=dtype, device="cuda")
    dt = 1 if dtype == torch.bfloat16 else 0
    st = ext.lib.ng_embed_tokens(tokens.data_ptr(), None, None, table.data_ptr(), dt, M, H, V, out.data_ptr(),
                                 res.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    assert torch.equal(out, table[tokens]) and int(res.count_nonzero()) == 0
    assert ext.device_status() == 0
    bad = torch.tensor([3, 1000], dtype=torch.int64, device="cuda")  # 1000 is outside the table
    st = ext.lib.ng_embed_tokens(bad.data_ptr(), None, None, table.data_ptr(), dt, 2, H, V, out.data_ptr(),
                                 None, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    assert ext.device_status() == 10  # NG_ERR_BAD_INDEX, reported once and cleared
    assert ext.device_status() == 0
    assert torch.equal(out[0], table[3]) and int(out[1].count_nonzero()) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K,N", [(1, 14336, 4096), (3, 1792, 4096), (16, 512, 1028)])
def test_silu_folded_gemv_is_bit_identical_to_separate_kernels(dtype, M, K, N):
    ext = ng.extension()
    dt = 1 if dtype == torch.bfloat16 else 0
    g = torch.Generator().manual_seed(M + K)
    gu = torch.randn(M, 2 * K, generator=g).to(dtype).cuda()
    qw = ng.quantize(torch.randn(K, N, generator=g) * 0.02, 128).to("cuda")
    st = torch.cuda.current_stream().cuda_stream
    act = torch.empty(M, K, dtype=dtype, device="cuda")
    assert ext.lib.ng_silu_mul(gu.data_ptr(), act.data_ptr(), dt, M, K, st) == 0
    y_ref = ext.gemv_w4a16(act, qw.qweight, qw.scales, 128, algo=2 if dt else 1)
    y = torch.empty(M, N, dtype=dtype, device="cuda")
    assert ext.lib.ng_gemv_w4a16_silu(gu.data_ptr(), dt, qw.qweight.data_ptr(), qw.scales.data_ptr(),
                                      y.data_ptr(), M, K, N, 128, st) == 0
    assert torch.equal(y, y_ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,hq,hkv,ctx,splits,pos", [(1, 32, 8, 1024, 32, 1023), (2, 8, 2, 64, 4, 5),
                                                   (3, 4, 4, 40, 7, 39)])
def test_attn_folded_gemv_is_bit_identical_to_combine_then_gemv(dtype, M, hq, hkv, ctx, splits, pos):
    """The o projection with the split combine in its staging equals the
    attention kernel's own combine followed by the plain GEMV, bit for bit;
    pos < ctx - 1 leaves trailing splits empty."""
    ext = ng.extension()
    dt = 1 if dtype == torch.bfloat16 else 0
    D = 128
    g = torch.Generator().manual_seed(M * 13 + hq)
    qkv = torch.randn(M, (hq + 2 * hkv) * D, generator=g).to(dtype).cuda()
    kc = torch.randn(M, ctx, hkv, D, generator=g).to(dtype).cuda()
    vc = torch.randn(M, ctx, hkv, D, generator=g).to(dtype).cuda()
    posd = torch.full((M,), pos, dtype=torch.int32, device="cuda")
    ws = torch.empty(ext.lib.ng_attn_workspace_bytes(M, hq, splits), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    out = torch.empty(M, hq * D, dtype=dtype, device="cuda")
    args = lambda o, k, v: (qkv.data_ptr(), k.data_ptr(), v.data_ptr(), posd.data_ptr(), o, dt, M, hq, hkv, D,
                            ctx, splits, 1.0 / math.sqrt(D), 500000.0, ws.data_ptr(), ws.numel(), st)
    kc2, vc2 = kc.clone(), vc.clone()
    assert ext.lib.ng_attn_decode_rope(*args(out.data_ptr(), kc, vc)) == 0
    K, N = hq * D, 1024
    qw = ng.quantize(torch.randn(K, N, generator=g) * 0.02, 128).to("cuda")
    y_ref = ext.gemv_w4a16(out, qw.qweight, qw.scales, 128, algo=2 if dt else 1)
    assert ext.lib.ng_attn_decode_rope(*args(None, kc2, vc2)) == 0
    y = torch.empty(M, N, dtype=dtype, device="cuda")
    assert ext.lib.ng_gemv_w4a16_attn(ws.data_ptr(), splits, dt, qw.qweight.data_ptr(), qw.scales.data_ptr(),
                                      y.data_ptr(), M, K, N, 128, st) == 0
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(y, y_ref)


FULL_WIDTH = dict(layers=2, hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=14336,
                  vocab=128256, rope_theta=500000.0, eps=1e-5)


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 5e-3), (torch.bfloat16, 2e-2)])
def test_decoder_full_llama3_8b_widths_matches_fp32_restatement(dtype, tol):
    """Two layers at the Llama-3-8B widths (the shapes that route through the
    wide GEMV schedules and the 32-way context split), three teacher-forced
    steps against the fp32 restatement: final hidden state and logits within
    max|err|/max|ref| <= 5e-3 with fp16 activations (bf16 keeps 8 mantissa
    bits, so its residual stream alone differs by ~4e-3 per rounding; 2e-2)."""
    m = Llama3Decoder(FULL_WIDTH, batch=1, max_ctx=64, dtype=dtype)
    ref = RefModel(m)
    g = torch.Generator().manual_seed(7)
    for step in range(3):
        toks = torch.randint(0, FULL_WIDTH["vocab"], (1,), generator=g).cuda()
        pos = m.pos.clone()
        m.tokens.copy_(toks)
        m.step()
        torch.cuda.synchronize()
        xn_ref, logits_ref = ref.step(toks, pos)
        assert _rel(m.xn, xn_ref) <= tol, (step, _rel(m.xn, xn_ref))
        assert _rel(m.logits, logits_ref) <= tol, (step, _rel(m.logits, logits_ref))
    assert ng.extension().device_status() == 0


@pytest.mark.parametrize("G", [64, 128])
def test_quantize_on_device_matches_reference_golden(golden, G):
    """RTN quantisation run on the GPU (how every projection of the decode
    models is built) reproduces the reference's own quantize() bit for bit."""
    from nibblegemm_b200.quant import quantize_on_device
    W = torch.from_numpy(golden[f"quant_g{G}_W"]).cuda()
    qw = quantize_on_device(W, G)
    assert qw.qweight.is_cuda
    assert torch.equal(qw.qweight.cpu(), torch.from_numpy(golden[f"quant_g{G}_qweight"]))
    assert torch.equal(qw.scales.cpu(), torch.from_numpy(golden[f"quant_g{G}_scales"]))
