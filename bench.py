"""Benchmark of the W4A16 hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemv|gemm|step8b|decode8b|decode70b|prefill8b|prefill70b|
                                readfloor|sweep2|sweep3]
                    [--batch B] [--reduce peer|nccl] [--algo A] [--no-wide-split]

Workload (default ``gemv``): BASELINE config 1 -- the decode GEMV
Y[1, 14336] = X[1, 4096] @ W4(4096 x 14336), group 128, fp16 activations, the
shape the headline "decode GEMV us & HBM GB/s at M=1" is quoted on.  A step is
one fused dequant-GEMV over one batch.  ``--workload gemm`` times BASELINE
config 3's M=2048, K=4096, N=14336 prefill GEMM instead (TFLOP/s).  The
decode workloads (``step8b`` projection stack, ``decode8b`` / ``decode70b``
full Llama-3 steps, tokens/s) replay one CUDA graph per token, tensor-parallel
over torchrun ranks; the prefill workloads (``prefill8b`` / ``prefill70b``)
time ``Llama3Decoder.prefill`` of 2048 prompt tokens (prompt tokens/s); ``readfloor``, ``sweep2`` and ``sweep3`` print one line
per measured point (diagnostics, not the headline).

* ``value``: algorithmic bytes (``K*N/2 + K/G*N*2 + M*K*2 + M*N*2``, the
  reference's byte model, bench/harness.py:243-255) per step x steps x ranks,
  divided by the device time of the timed region (CUDA events on the launching
  stream, max over ranks).  Inputs are resident in HBM; the weight rotates
  over enough distinct copies to exceed L2 (so every step reads HBM).  The
  K steps are replayed from one CUDA graph so launch gaps are the device's.
* ``e2e``: the same metric through the public API (``nibblegemm_b200.gemv``)
  with the activation copied host->device from pinned memory and the result
  copied back every step, host-synchronised -- what a caller sees.
* ``roofline``: the GEMV kernel's achieved HBM GB/s against the measured copy
  bandwidth in MEASURED_PEAKS.json (burst figure: the kernel is timed alone).
* ``cpu_baseline``: the reference's CPU path (numpy unpack + fp32 dequantise +
  fp32 matmul, restated in ``oracle/quant_oracle.py``) on a bounded sample.
* ``--impl reference``: that CPU path alone, all host threads, as the
  reference arm (rank 0 only under torchrun).

Multi-GPU: the GEMV does not shard -- ranks run independent replicas (weak
scaling, no collective on the data path).  The default line also carries the
sharded paths measured over all ranks of the run (strong scaling):
``tp_decode8b`` (the Llama-3-8B decode step) and ``tp_prefill70b`` (config 5's
Llama-3-70B prefill of 2048 tokens).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode GEMV µs & HBM GB/s (% of 8 TB/s) at M=1; prefill TFLOP/s; 8B tok/s @1/2/4/8"
WORKLOADS = {
    "gemv": dict(M=1, K=4096, N=14336, G=128, name="W4A16 decode GEMV M=1 K=4096 N=14336 g128 fp16 (BASELINE config 1)"),
    "gemm": dict(M=2048, K=4096, N=14336, G=128, name="W4A16 prefill GEMM M=2048 K=4096 N=14336 g128 fp16 (BASELINE config 3)"),
    "step8b": dict(M=1, K=4096, N=14336, G=128, name="Llama-3-8B INT4 g128 projection stack (224 projections), batch 1, tensor-parallel over the ranks"),
    "decode8b": dict(M=1, K=4096, N=14336, G=128, name="Llama-3-8B INT4 g128 full decode step (BASELINE config 4): attention over a 1024-token KV cache, norms, RoPE, SwiGLU, fp16 lm_head + argmax, batch --batch (default 1), tensor-parallel over the ranks"),
    "decode70b": dict(M=1, K=8192, N=28672, G=128, name="Llama-3-70B INT4 g128 full decode step (BASELINE config 5): attention over a 2048-token KV cache, norms, RoPE, SwiGLU, fp16 lm_head + argmax, batch --batch, tensor-parallel over the ranks"),
    "prefill70b": dict(M=2048, K=8192, N=28672, G=128, name="Llama-3-70B INT4 g128 prefill of 2048 synthetic token ids uniform over the vocab (BASELINE config 5): every projection a [batch x 2048]-row tcgen05 GEMM, causal GQA attention, norms, RoPE, SwiGLU, head on the last position, batch --batch, tensor-parallel over the ranks"),
    "prefill8b": dict(M=2048, K=4096, N=14336, G=128, name="Llama-3-8B INT4 g128 prefill of 2048 synthetic token ids (config 4 model), as prefill70b"),
    "sweep2": dict(M=1, K=4096, N=14336, G=128, name="BASELINE config 2: decode GEMV sweep M x (K, N), eager and graph, vs cuBLAS fp16"),
    "readfloor": dict(M=1, K=4096, N=14336, G=128, name="transfer-size floor: config-1 GEMV at N x 1/2/4/8 beside a torch fp32 sum reading the same bytes"),
    "sweep3": dict(M=2048, K=4096, N=14336, G=128, name="BASELINE config 3: prefill GEMM sweep M x (K, N) x {fp16, bf16}"),
}

SWEEP2_M = (1, 2, 4, 8, 16)
SWEEP2_SHAPES = ((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096), (8192, 8192))
SWEEP3_M = (16, 128, 512, 2048, 8192)
SWEEP3_SHAPES = ((4096, 14336), (14336, 4096))


def _graph_us(fn, n, stream):
    """Device time per call of `fn(i)`, `n` calls captured in one CUDA graph."""
    with torch.cuda.stream(stream):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / n


def _eager_us(fn, n):
    """Wall-inclusive device time per call of `fn(i)` launched eagerly from Python."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / n


def run_readfloor(args, local):
    """How fast can one launch read B bytes?  For the config-1 byte count and
    2x/4x/8x it, our M=1 GEMV (K=4096, N scaled) and a torch ``sum`` (fp32
    accumulate) over a buffer of the same algorithmic bytes, both replayed from a
    CUDA graph with operands rotated over more than L2.  One JSON line per size."""
    import nibblegemm_b200 as ng
    from oracle import quant_oracle as qo  # seeded synthetic inputs (generator only)
    ext = ng.extension()
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    hbm, _, src = measured_peaks()
    stream = torch.cuda.Stream()
    K, G = 4096, 128
    for r in (1, 2, 4, 8):
        N = 14336 * r
        x, q, sc = qo.synthetic_case(1, K, N, group_size=G, seed=3)
        nb = algo_bytes(1, K, N, G)
        nrot = max(2, -(-3 * l2 // nb))
        Q = [torch.from_numpy(q).cuda() for _ in range(nrot)]
        S = [torch.from_numpy(sc).cuda() for _ in range(nrot)]
        X = torch.from_numpy(x).cuda()
        Y = torch.empty(1, N, dtype=torch.float16, device="cuda")
        ours = lambda i: ext.gemv_w4a16(X, Q[i % nrot], S[i % nrot], G, out=Y)
        B = [torch.randn(nb // 2, device="cuda").half() for _ in range(nrot)]
        out = torch.empty((), dtype=torch.float32, device="cuda")
        red = lambda i: out.copy_(torch.sum(B[i % nrot], dtype=torch.float32))
        ug, ur = _graph_us(ours, 100, stream), _graph_us(red, 100, stream)
        print(json.dumps({
            "readfloor": "config1", "bytes": nb, "N": N, "gemv_us": round(ug, 2),
            "gemv_GBs": round(nb / ug / 1e3, 1), "torch_sum_us": round(ur, 2),
            "torch_sum_GBs": round(nb / ur / 1e3, 1), "gemv_frac_hbm": round(nb / ug / 1e3 / hbm, 3),
            "torch_sum_frac_hbm": round(nb / ur / 1e3 / hbm, 3), "peak_source": src}), flush=True)
        del Q, S, B
        torch.cuda.empty_cache()


def run_sweep(args, local):
    """BASELINE configs 2 and 3 as one JSON line per point (seeded synthetic data;
    weights rotated over more than L2 between calls)."""
    import nibblegemm_b200 as ng
    from oracle import quant_oracle as qo  # seeded synthetic inputs (generator only)
    ext = ng.extension()
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    hbm, bf16_peak, src = measured_peaks()
    stream = torch.cuda.Stream()
    shapes = SWEEP2_SHAPES if args.workload == "sweep2" else SWEEP3_SHAPES
    for K, N in shapes:
        _, q, s = qo.synthetic_case(1, K, N, group_size=128, seed=7)
        wbytes = q.nbytes + s.nbytes
        nrot = max(2, -(-3 * l2 // (2 * wbytes)))
        Q = [torch.from_numpy(q).cuda() for _ in range(nrot)]
        S = torch.from_numpy(s).cuda()
        W16 = ext.dequant_w4(Q[0], S, 128)  # cuBLAS comparison operand (fp16 [K, N])
        n16 = max(2, -(-3 * l2 // (2 * W16.numel() * 2)))
        W16s = [W16] + [W16.clone() for _ in range(n16 - 1)]
        if args.workload == "sweep2":
            for M in SWEEP2_M:
                X = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().cuda()
                Y = torch.empty(M, N, dtype=torch.float16, device="cuda")
                ours = lambda i: ext.gemv_w4a16(X, Q[i % nrot], S, 128, out=Y)
                Y16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
                cub = lambda i: torch.mm(X, W16s[i % n16], out=Y16)
                n = 100
                ug, ue = _graph_us(ours, n, stream), _eager_us(ours, n)
                cg_, ce = _graph_us(cub, n, stream), _eager_us(cub, n)
                nb = algo_bytes(M, K, N, 128)
                b16 = K * N * 2 + M * K * 2 + M * N * 2
                print(json.dumps({
                    "sweep": "config2", "M": M, "K": K, "N": N, "us_graph": round(ug, 2),
                    "us_eager": round(ue, 2), "GBs_graph": round(nb / ug / 1e3, 1),
                    "frac_hbm_graph": round(nb / ug / 1e3 / hbm, 3),
                    "cublas_fp16_us_graph": round(cg_, 2), "cublas_fp16_us_eager": round(ce, 2),
                    "speedup_vs_cublas_graph": round(cg_ / ug, 2),
                    "speedup_vs_cublas_eager": round(ce / ue, 2),
                    "byte_ratio_ceiling": round(b16 / nb, 3), "peak_source": src}), flush=True)
        else:
            for M in SWEEP3_M:
                for dt in (torch.float16, torch.bfloat16):
                    X = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).to(dt).cuda()
                    Y = torch.empty(M, N, dtype=dt, device="cuda")
                    ours = lambda i: ext.gemm_w4a16(X, Q[i % nrot], S, 128, out=Y)
                    Wd = W16s if dt == torch.float16 else [w.to(dt) for w in W16s]
                    Yc = torch.empty(M, N, dtype=dt, device="cuda")
                    cub = lambda i: torch.mm(X, Wd[i % len(Wd)], out=Yc)
                    flops = 2.0 * M * K * N
                    n = max(5, min(100, int(2e12 / flops)))
                    ug, cg_ = _graph_us(ours, n, stream), _graph_us(cub, n, stream)
                    print(json.dumps({
                        "sweep": "config3", "M": M, "K": K, "N": N, "dtype": str(dt).split(".")[-1],
                        "us_graph": round(ug, 2), "TFLOPs": round(flops / ug / 1e6, 1),
                        "frac_dense_peak": round(flops / ug / 1e6 / bf16_peak, 3),
                        "GBs": round(algo_bytes(M, K, N, 128) / ug / 1e3, 1),
                        "cublas_dense_us_graph": round(cg_, 2),
                        "cublas_dense_TFLOPs": round(flops / cg_ / 1e6, 1),
                        "peak_source": src}), flush=True)
                    del Wd
        del Q, W16s, W16
        torch.cuda.empty_cache()
    assert ext.device_status() == 0, "a kernel reported a bounded-wait timeout"


def algo_bytes(M, K, N, G):
    return K * N // 2 + (K // G) * N * 2 + M * K * 2 + M * N * 2


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi SM clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [int(r[0]) for r in self.rows if r[0].isdigit()]
        mx = [int(r[1]) for r in self.rows if r[1].isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 2 + i and r[2 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


def cpu_model() -> str:
    """The host CPU's model string (from /proc/cpuinfo), for the baseline record."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_sample(wl, seconds: float = 12.0, threads: int = 0):
    """Time the reference's CPU path (the oracle port of quant.py's
    reference_matmul: dequantise, then an fp32 matmul) on the workload shape:
    the median of >= 5 full calls, and the steady state (weights dequantised
    once, the fp32 matmul alone), bounded to about `seconds` in total.
    Returns (GB/s of the full path, seconds per full call, sample text,
    threads, extras dict)."""
    from oracle import quant_oracle as qo
    M, K, N, G = wl["M"], wl["K"], wl["N"], wl["G"]
    if threads > 0:
        torch.set_num_threads(threads)
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=1)
    xt = torch.from_numpy(x.astype(np.float32))
    full, t_start = [], time.perf_counter()
    while len(full) < 5 or (time.perf_counter() - t_start < seconds * 0.7 and len(full) < 50):
        t0 = time.perf_counter()
        W = torch.from_numpy(qo.dequantize_np(q, s, G, K).astype(np.float32))
        _ = (xt @ W).to(torch.float16)
        full.append(time.perf_counter() - t0)
    steady = []
    for _ in range(max(5, min(50, int(seconds * 0.3 / max(1e-4, min(full) / 4))))):
        t0 = time.perf_counter()
        _ = (xt @ W).to(torch.float16)
        steady.append(time.perf_counter() - t0)
    per = float(np.median(full))
    per_mm = float(np.median(steady))
    nbytes = algo_bytes(M, K, N, G)
    extras = {"median_of": len(full), "steady_state_value": round(nbytes / per_mm / 1e9, 4),
              "steady_state_ms_per_call": round(per_mm * 1e3, 3),
              "steady_state_sample": f"median of {len(steady)} fp32 matmuls on pre-dequantised weights",
              "cpu_model": cpu_model(), "os_cpu_count": os.cpu_count()}
    return (nbytes / per / 1e9, per,
            f"median of {len(full)} full reference_matmul calls (numpy dequantise + torch fp32 matmul) "
            f"at M={M} K={K} N={N}", torch.get_num_threads(), extras)


def run_reference_decode(args):
    """Reference arm of the decode workloads: the reference's CPU path for one
    token's projections (its model benchmark is the 7 projections of every
    layer, bench/bench_model.py:43-125), each shape timed once per step with
    ``reference_matmul`` (numpy dequantise + torch fp32 matmul) and scaled by the
    layer count.  Attention, norms and the lm_head are not counted, which
    favours the reference."""
    from nibblegemm_b200.decode_step import LLAMA3_70B, LLAMA3_8B, layer_projections
    from oracle import quant_oracle as qo
    wl = WORKLOADS[args.workload]
    cfg = LLAMA3_70B if args.workload == "decode70b" else LLAMA3_8B
    batch = args.batch if args.workload != "step8b" else 1
    cases = []
    for i, (_, K, N, _) in enumerate(layer_projections(cfg)):
        x, q, s = qo.synthetic_case(batch, K, N, group_size=128, seed=i)
        cases.append((torch.from_numpy(x.astype(np.float32)), q, s, K))

    def step():
        t = 0.0
        for xt, q, s, K in cases:
            t0 = time.perf_counter()
            W = qo.dequantize_np(q, s, 128, K).astype(np.float32)
            (xt @ torch.from_numpy(W)).to(torch.float16)
            t += time.perf_counter() - t0
        return t * cfg["layers"]

    for _ in range(3):  # warm-up passes (each pass is seconds)
        step()
    t0, times = time.perf_counter(), []
    while len(times) < args.steps:
        times.append(step())
        if time.perf_counter() - t0 > 90.0:
            break
    per = sum(times) / len(times)
    value = batch / per
    sample = (f"{len(times)} passes over the 7 projection shapes of one {args.workload} layer at "
              f"M={batch} (reference_matmul each), x {cfg['layers']} layers; projections only")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": 3, "ms_per_step": round(per * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (BASELINE distributions, seeded)",
        "config": {"workload": wl["name"], "batch": batch, "group_size": 128},
        "cpu_baseline": {"value": round(value, 6), "unit": "tok/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference(args, rank):
    if rank != 0:
        return
    if args.workload in ("step8b", "decode8b", "decode70b"):
        return run_reference_decode(args)
    if args.workload in ("prefill8b", "prefill70b"):
        return run_reference_prefill(args)
    wl = WORKLOADS[args.workload]
    M, K, N, G = wl["M"], wl["K"], wl["N"], wl["G"]
    from oracle import quant_oracle as qo
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=1)
    xt = torch.from_numpy(x.astype(np.float32))

    def step():
        W = qo.dequantize_np(q, s, G, K).astype(np.float32)
        return (xt @ torch.from_numpy(W)).to(torch.float16)

    # Each step is one full reference call (seconds on a CPU): warm-up and the
    # timed steps are capped so the arm ends within a few minutes; the line
    # reports the steps actually timed.
    for _ in range(min(args.warmup, 3)):
        step()
    t0, times = time.perf_counter(), []
    while len(times) < args.steps:
        t1 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t1)
        if time.perf_counter() - t0 > 90.0 and len(times) >= 5:
            break
    done = len(times)
    per = float(np.median(times))
    args.steps, args.warmup = done, min(args.warmup, 3)
    if args.workload == "gemv":
        value, unit = algo_bytes(M, K, N, G) / per / 1e9, "GB/s"
    else:
        value, unit = 2.0 * M * K * N / per / 1e12, "TFLOP/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (BASELINE distributions, seeded)",
        "config": {"workload": wl["name"], "M": M, "K": K, "N": N, "group_size": G,
                   "l2": "n/a (host)"},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": torch.get_num_threads(),
                         "kind": "port", "cpu_model": cpu_model(), "os_cpu_count": os.cpu_count(),
                         "sample": f"median of {args.steps} timed reference_matmul calls (numpy unpack + fp32 dequantise + torch fp32 matmul)"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure_decode(cfg, ctx, batch, steps, warmup, world, rank, dist, reduce="peer", wide_split=True,
                   local=0, sample_clocks=True, **model_kw):
    """Device-timed tokens/s of one Llama-3 decode step (every rank runs its
    tensor-parallel shard), plus the end-to-end figure with the token ids
    crossing PCIe.  Returns a dict of raw figures (identical on every rank)."""
    from nibblegemm_b200.decode_model import Llama3Decoder
    m = Llama3Decoder(cfg, batch=batch, max_ctx=ctx, rank=rank, world=world, reduce=reduce,
                      wide_split=wide_split, **model_kw)
    m.pos.fill_(ctx - 1)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            m.step(advance=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        m.step(advance=False)
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if sample_clocks else contextlib.nullcontext()
    with sampler as clocks:
        for _ in range(50):  # fixed count on every rank: the graph holds collectives
            graph.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    per_ms = ms / steps
    # e2e: the token ids in from pinned host memory, the step (graph), the next ids back
    tok_host = torch.zeros(batch, dtype=torch.int64).pin_memory()
    out_host = torch.zeros(batch, dtype=torch.int64).pin_memory()
    e2e_steps = max(3, min(steps, 50))
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            m.tokens.copy_(tok_host, non_blocking=True)
            graph.replay()
            out_host.copy_(m.tokens, non_blocking=True)
            stream.synchronize()
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    status = m.ext.device_status()
    kv = 2 * cfg["layers"] * ctx * m.hkv * cfg["head_dim"] * 2 * batch
    nbytes = m.weight_bytes + m.lm_head.numel() * 2 + kv + cfg["hidden"] * 2 * batch
    out = dict(per_ms=per_ms, e2e_ms=e2e_ms, nbytes=nbytes, launches=m.launches_per_step(),
               clocks=clocks.summary() if sample_clocks else None, status=status)
    del graph, m
    torch.cuda.empty_cache()
    return out


def run_decode(args, wl, world, rank, local, dist):
    """Tokens/s of the full Llama-3-8B decode step (with
    ``--workload decode70b`` the Llama-3-70B step of config 5: context 2048,
    ``--batch`` sequences).

    One step = one token through embedding, 32 layers (RMSNorm, fused q|k|v
    GEMV, GQA attention with RoPE + KV append over 1024 cached positions, o GEMV,
    all-reduce, RMSNorm, fused gate|up GEMV, SwiGLU, down GEMV, all-reduce),
    final norm, fp16 lm_head with the argmax fused in; captured once in a CUDA
    graph and replayed with the position held at ctx - 1.  Strong scaling.
    """
    from nibblegemm_b200.decode_model import LLAMA3_8B_MODEL, LLAMA3_70B_MODEL
    big = args.workload == "decode70b"
    cfg = LLAMA3_70B_MODEL if big else LLAMA3_8B_MODEL
    ctx = 2048 if big else 1024
    batch = args.batch
    kw = {}
    if args.gemv_algo is not None:
        kw["gemv_algo"] = args.gemv_algo
    if args.attn_splits:
        kw["attn_splits"] = args.attn_splits
    if args.no_fused_norm:
        kw["fused_norm"] = False
    if args.fold is not None:
        kw["fold_silu"] = "silu" in args.fold
        kw["fold_attn"] = "attn" in args.fold
    r = measure_decode(cfg, ctx, batch, args.steps, args.warmup, world, rank, dist, args.reduce,
                       not args.no_wide_split, local, **kw)
    assert r["status"] == 0, "a kernel reported a bounded-wait timeout"
    if rank == 0:
        hbm, _, src = measured_peaks()
        per_ms, e2e_ms, nbytes = r["per_ms"], r["e2e_ms"], r["nbytes"]
        achieved = nbytes / (per_ms * 1e-3) / 1e9
        L = cfg["layers"]
        line = {
            "metric": METRIC, "value": round(1000.0 * batch / per_ms, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": f"synthetic random-init {'Llama-3-70B' if big else 'Llama-3-8B'} (seeded N(0,0.02) weights, RTN INT4 g128), batch {batch}",
            "config": {"workload": wl["name"], "layers": L, "hidden": cfg["hidden"], "heads": cfg["heads"],
                       "kv_heads": cfg["kv_heads"], "intermediate": cfg["intermediate"], "vocab": cfg["vocab"],
                       "context": ctx, "group_size": 128, "batch": batch, "parallelism": f"tp{world}",
                       "tp_reduce": (args.reduce if world > 1 else None),
                       "l2": f"{nbytes / 1e9:.1f} GB read per step per rank (>> L2)",
                       "timing": "one CUDA graph per step (every sequence advances one token), replayed `steps` times"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None,
                         "peak_source": f"{src} copy bandwidth", "algorithmic_bytes_per_step_per_rank": nbytes},
            "e2e": {"value": round(1000.0 * batch / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * batch,
                    "d2h_bytes_per_step": 8 * batch, "path": "token ids in -> Llama3Decoder.step() graph -> next ids out"},
            "gpu_launches": r["launches"],
            "clocks": r["clocks"],
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


PREFILL_TOKENS = 2048


def prefill_flops(cfg, m, batch, S):
    """FLOPs of one prefill on one rank: 2 per weight per token in the
    projections, 4 * S^2 / 2 * D per (sequence, query head) in causal attention
    (QK^T and PV), and the head on one position per sequence."""
    proj = sum(w[k].K * w[k].N for w in m.w for k in ("qkv", "o", "gu", "down"))
    attn = 2 * S * (S + 1) * cfg["head_dim"] * m.hq * cfg["layers"]
    head = (m.v1 - m.v0) * cfg["hidden"]
    return 2.0 * proj * batch * S + attn * batch + 2.0 * head * batch


def measure_prefill(cfg, batch, steps, warmup, world, rank, dist, local=0, sample_clocks=True):
    """Device-timed prefill of PREFILL_TOKENS prompt tokens per sequence
    (every rank runs its tensor-parallel shard), plus the end-to-end figure
    with the prompt ids crossing PCIe.  Returns raw figures (same on every rank)."""
    from nibblegemm_b200.decode_model import Llama3Decoder
    S = PREFILL_TOKENS
    m = Llama3Decoder(cfg, batch=batch, max_ctx=S + 64, rank=rank, world=world, reduce="nccl")
    g = torch.Generator().manual_seed(1234)
    tok_host = torch.randint(0, cfg["vocab"], (batch, S), generator=g).pin_memory()
    toks = tok_host.cuda()
    out_host = torch.zeros(batch, dtype=torch.int64).pin_memory()

    def one():
        m.pos.zero_()
        m.prefill(toks)

    for _ in range(max(1, warmup)):
        one()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if sample_clocks else contextlib.nullcontext()
    with sampler as clocks:
        a.record()
        for _ in range(steps):
            one()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    per_ms = ms / steps
    # e2e: the prompt's ids from pinned host memory, the prefill, the next ids back
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    e_steps = max(1, min(steps, 5))
    e0.record()
    for _ in range(e_steps):
        toks.copy_(tok_host, non_blocking=True)
        one()
        out_host.copy_(m.tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    out = dict(per_ms=per_ms, e2e_ms=e2e_ms, flops=prefill_flops(cfg, m, batch, S),
               launches=1 + 9 * cfg["layers"] + batch + 2, status=m.ext.device_status(),
               clocks=clocks.summary() if sample_clocks else None)
    del m
    torch.cuda.empty_cache()
    return out


def sustained_tflops():
    _, tf_burst, src = measured_peaks()
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if src == "measured" else {}
    return peaks.get("bf16_tflops_sustained", tf_burst), src


def run_prefill(args, wl, world, rank, local, dist):
    """Prompt tokens/s of ``Llama3Decoder.prefill`` (the
    Llama-3-70B prefill of 2048 synthetic token ids; ``prefill8b``: the 8B model).

    One step = one prefill of 2048 tokens per sequence from position 0: the
    embedding, then per layer RMSNorm, the q|k|v GEMM, RoPE + KV append for all
    positions, causal GQA attention over the cache, the o GEMM (+ all-reduce),
    RMSNorm, the gate|up GEMM, SwiGLU, the down GEMM (+ all-reduce), and the head
    with its argmax on the last position.  Eager launches (each GEMM is
    milliseconds long), CUDA events on the stream, max over ranks.  Strong
    scaling: the same prompt, the model sharded over the ranks.
    """
    from nibblegemm_b200.decode_model import LLAMA3_8B_MODEL, LLAMA3_70B_MODEL
    big = args.workload == "prefill70b"
    cfg = LLAMA3_70B_MODEL if big else LLAMA3_8B_MODEL
    S, batch = PREFILL_TOKENS, args.batch
    r = measure_prefill(cfg, batch, args.steps, args.warmup, world, rank, dist, local)
    assert r["status"] == 0, "a kernel reported a bounded-wait timeout"
    if rank == 0:
        tf, src = sustained_tflops()
        per_ms, flops = r["per_ms"], r["flops"]
        achieved = flops / (per_ms * 1e-3) / 1e12
        L = cfg["layers"]
        line = {
            "metric": METRIC, "value": round(1000.0 * batch * S / per_ms, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": f"synthetic random-init {'Llama-3-70B' if big else 'Llama-3-8B'} (seeded N(0,0.02) weights, RTN INT4 g128); prompt ids uniform over the vocab",
            "config": {"workload": wl["name"], "layers": L, "hidden": cfg["hidden"], "heads": cfg["heads"],
                       "kv_heads": cfg["kv_heads"], "intermediate": cfg["intermediate"], "vocab": cfg["vocab"],
                       "prompt_tokens": S, "group_size": 128, "batch": batch, "parallelism": f"tp{world}",
                       "tp_reduce": "nccl" if world > 1 else None,
                       "l2": "every step streams all projection weights (>> L2)",
                       "timing": "eager launches, CUDA events around `steps` prefills"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf, "unit": "TFLOP/s",
                         "frac": round(achieved / tf, 4), "traffic": None,
                         "peak_source": f"{src} cuBLAS bf16 (sustained: a step of {per_ms:.0f} ms)",
                         "algorithmic_flops_per_step_per_rank": flops},
            "e2e": {"value": round(1000.0 * batch * S / r["e2e_ms"], 1), "unit": "tok/s",
                    "h2d_bytes_per_step": 8 * batch * S, "d2h_bytes_per_step": 8 * batch,
                    "path": "prompt ids in -> Llama3Decoder.prefill -> next ids out"},
            "gpu_launches": r["launches"] * args.steps,
            "clocks": r["clocks"],
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def run_reference_prefill(args):
    """Reference arm of the prefill workloads: the reference's CPU path
    (``reference_matmul``: numpy dequantise + torch fp32 matmul) for the 7
    projection shapes of one layer on a bounded sample of 64 prompt rows,
    scaled to the 2048-token prompt and the layer count.  Attention, norms and
    the head are not counted, which favours the reference."""
    from nibblegemm_b200.decode_step import LLAMA3_70B, LLAMA3_8B, layer_projections
    from oracle import quant_oracle as qo
    wl = WORKLOADS[args.workload]
    cfg = LLAMA3_70B if args.workload == "prefill70b" else LLAMA3_8B
    rows, batch = 64, args.batch
    cases = []
    for i, (_, K, N, _) in enumerate(layer_projections(cfg)):
        x, q, s = qo.synthetic_case(rows, K, N, group_size=128, seed=i)
        cases.append((torch.from_numpy(x.astype(np.float32)), q, s, K))

    def step():
        t = 0.0
        for xt, q, s, K in cases:
            t0 = time.perf_counter()
            W = qo.dequantize_np(q, s, 128, K).astype(np.float32)
            (xt @ torch.from_numpy(W)).to(torch.float16)
            t += time.perf_counter() - t0
        # one layer at `rows` prompt rows -> every layer at batch x 2048 rows
        return t * (batch * PREFILL_TOKENS / rows) * cfg["layers"]

    step()  # warm-up
    t0, times = time.perf_counter(), []
    while len(times) < max(1, min(args.steps, 5)):
        times.append(step())
        if time.perf_counter() - t0 > 90.0:
            break
    per = float(np.median(times))
    value = batch * PREFILL_TOKENS / per
    sample = (f"median of {len(times)} passes over the 7 projection shapes of one {args.workload} layer at "
              f"{rows} prompt rows (reference_matmul each), scaled to {batch} x {PREFILL_TOKENS} tokens x "
              f"{cfg['layers']} layers; projections only")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": 1, "ms_per_step": round(per * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (BASELINE distributions, seeded)",
        "config": {"workload": wl["name"], "batch": batch, "prompt_tokens": PREFILL_TOKENS, "group_size": 128},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_step(args, wl, world, rank, local, dist):
    """Tokens/s of the Llama-3-8B INT4 projection stack.

    One step = one batch-1 token through all 224 decoder projections; under
    torchrun the projections are Megatron-sharded over the ranks with an NCCL
    all-reduce after o and down (strong scaling: the token is the same).  The
    step is captured once into a CUDA graph and replayed `steps` times.
    """
    import nibblegemm_b200 as ng
    from nibblegemm_b200.decode_step import LLAMA3_8B, ProjectionStackStep
    step = ProjectionStackStep(LLAMA3_8B, batch=1, rank=rank, world=world, reduce=("peer" if args.reduce == "fused" else args.reduce))
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step.step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step.step()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        # A fixed replay count on every rank: each replay holds NCCL all-reduces,
        # so all ranks must run the same number (a wall-clock loop would not).
        for _ in range(300):
            graph.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        dist.barrier()
    per_ms = ms / args.steps
    # e2e: eager public-API step, activation in from pinned host memory, last output back
    x_host = torch.randn(1, LLAMA3_8B["hidden"]).half().pin_memory()
    y_host = torch.empty(1, LLAMA3_8B["hidden"]).half().pin_memory()
    first, last = step.proj[0][0], step.proj[-1][-1]
    e2e_steps = max(3, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        first.x.copy_(x_host, non_blocking=True)
        step.step()
        y_host.copy_(last.y, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    if rank == 0:
        hbm, _, src = measured_peaks()
        wbytes = step.weight_bytes
        achieved = wbytes / (per_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(1000.0 / per_ms, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic random-init INT4 weights (BASELINE distributions), batch-1 activations",
            "config": {"workload": wl["name"], "layers": 32, "hidden": 4096, "kv": 1024,
                       "intermediate": 14336, "group_size": 128, "batch": 1,
                       "parallelism": f"tp{world}",
                       "tp_reduce": (args.reduce if world > 1 else None), "l2": "3.6 GB of distinct weights per token (>> L2)",
                       "timing": "one CUDA graph per token, replayed `steps` times"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None,
                         "peak_source": f"{src} copy bandwidth", "algorithmic_bytes_per_step_per_rank": wbytes},
            "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 8192,
                    "d2h_bytes_per_step": 8192, "path": "ProjectionStackStep.step() eager"},
            "gpu_launches": 224 + (64 if (world > 1 and args.reduce == "peer") else 0),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="gemv")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true",
                    help="gemv workload: skip the config-3 prefill GEMM point")
    ap.add_argument("--no-tp-prefill", action="store_true",
                    help="default workload: skip the tensor-parallel Llama-3-70B prefill object")
    ap.add_argument("--no-tp-decode", action="store_true",
                    help="gemv workload: skip the tensor-parallel Llama-3-8B decode-step measurement")
    ap.add_argument("--reduce", choices=["peer", "nccl", "fused"], default="peer",
                    help="tensor-parallel reduction: fused into the row-parallel GEMV (decode steps; the "
                    "projection stack uses peer), the peer-memory all-reduce kernel, or NCCL")
    ap.add_argument("--batch", type=int, default=1, help="sequences per step (decode8b, decode70b)")
    ap.add_argument("--gemv-algo", type=int, default=None,
                    help="decode workloads: one ng_gemv_w4a16 algo for every projection")
    ap.add_argument("--attn-splits", type=int, default=0, help="decode workloads: context splits")
    ap.add_argument("--no-fused-norm", action="store_true", help="decode workloads: separate RMSNorm kernels")
    ap.add_argument("--fold", default=None, help="decode workloads: kernels folded into GEMV staging "
                    "('silu', 'attn', 'silu,attn' or 'none'; default: the model's choice)")
    ap.add_argument("--no-wide-split", action="store_true",
                    help="decode workloads: keep wide projections on the cluster GEMV")
    ap.add_argument("--algo", type=int, default=0, help="GEMV schedule (see ng_gemv_w4a16)")
    ap.add_argument("--profile", action="store_true",
                    help="profiling target: run the op warmup+1 times eagerly on one GPU and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import nibblegemm_b200 as ng
    from nibblegemm_b200 import _lib

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    wl = WORKLOADS[args.workload]
    if args.workload == "step8b":
        return run_step(args, wl, world, rank, local, dist)
    if args.workload in ("decode8b", "decode70b"):
        return run_decode(args, wl, world, rank, local, dist)
    if args.workload in ("prefill8b", "prefill70b"):
        return run_prefill(args, wl, world, rank, local, dist)
    if args.workload == "readfloor":
        if rank == 0:
            run_readfloor(args, local)
        return
    if args.workload in ("sweep2", "sweep3"):
        if rank == 0:
            run_sweep(args, local)
        return
    M, K, N, G = wl["M"], wl["K"], wl["N"], wl["G"]
    from oracle import quant_oracle as qo  # seeded synthetic inputs (generator only)
    x, q, s = qo.synthetic_case(M, K, N, group_size=G, seed=1 + rank)
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    wbytes = q.nbytes + s.nbytes
    nrot = max(2, -(-3 * l2 // wbytes))
    qw_dev = [ng.QuantizedWeight(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), G, K, N)
              for _ in range(nrot)]
    X = torch.from_numpy(x).cuda()
    Y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ext = ng.extension()
    if args.workload == "gemv":
        op = lambda i: ext.gemv_w4a16(X, qw_dev[i % nrot].qweight, qw_dev[i % nrot].scales, G,
                                      algo=args.algo, out=Y)
    else:
        op = lambda i: ext.gemm_w4a16(X, qw_dev[i % nrot].qweight, qw_dev[i % nrot].scales, G, out=Y)

    if args.profile:  # a short, eager launch sequence for ncu -k ... -s <warmup> -c 1
        for i in range(args.warmup + 1):
            op(i)
        torch.cuda.synchronize()
        print(json.dumps({"profile_target": args.workload, "launches": args.warmup + 1}))
        return

    # ---- device-timed region: K steps replayed from one CUDA graph ----------------
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            op(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            op(i)
    graph.replay()  # warm the graph itself
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        # Keep the GPU busy with the same graph for ~0.5 s first so the
        # sampler (100 ms period) sees clocks under this load; the timed
        # region below is one replay of exactly `steps` launches.
        t_end = time.perf_counter() + 0.5
        while time.perf_counter() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end)
    assert ext.device_status() == 0, "a kernel reported a bounded-wait timeout"
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    per_ms = ms / args.steps
    nbytes = algo_bytes(M, K, N, G)
    flops = 2.0 * M * K * N
    if args.workload == "gemv":
        value, unit = nbytes * args.steps * world / (ms * 1e-3) / 1e9, "GB/s"
    else:
        value, unit = flops * args.steps * world / (ms * 1e-3) / 1e12, "TFLOP/s"

    # ---- end-to-end through the public API with host buffers ----------------------
    x_host = torch.from_numpy(x).pin_memory()
    y_host = torch.empty(M, N, dtype=torch.float16).pin_memory()
    e2e_steps = max(20, min(args.steps, 200))
    fn = ng.gemv if args.workload == "gemv" else ng.gemm
    for i in range(3):
        y_host.copy_(fn(x_host.cuda(non_blocking=True), qw_dev[i % nrot]), non_blocking=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        xd = x_host.cuda(non_blocking=True)
        y_host.copy_(fn(xd, qw_dev[i % nrot]), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    if args.workload == "gemv":
        e2e_val = nbytes * e2e_steps * world / (e2e_ms * 1e-3) / 1e9
    else:
        e2e_val = flops * e2e_steps * world / (e2e_ms * 1e-3) / 1e12

    # ---- the sharded path at this N: the Llama-3-8B decode step, tensor-parallel ----
    tp = None
    if args.workload == "gemv" and not args.no_tp_decode:
        from nibblegemm_b200.decode_model import LLAMA3_8B_MODEL
        tp = measure_decode(LLAMA3_8B_MODEL, 1024, 1, max(10, min(args.steps, 100)), 3, world, rank, dist,
                            reduce=args.reduce, local=local, sample_clocks=(rank == 0))
        assert tp["status"] == 0, "a decode-step kernel reported an error"

    # ---- config 5's prefill at this N: Llama-3-70B, 2048 prompt tokens, tensor-parallel ----
    tpp = None
    if args.workload == "gemv" and not args.no_tp_prefill:
        from nibblegemm_b200.decode_model import LLAMA3_70B_MODEL
        tpp = measure_prefill(LLAMA3_70B_MODEL, 1, 3, 2, world, rank, dist, local, sample_clocks=(rank == 0))
        assert tpp["status"] == 0, "a prefill kernel reported an error"

    # ---- BASELINE config 3's headline point on this GPU: the prefill GEMM ----------
    gemm_obj = None
    if args.workload == "gemv" and not args.no_gemm:
        gm = WORKLOADS["gemm"]
        Mg, Kg, Ng, Gg = gm["M"], gm["K"], gm["N"], gm["G"]
        xg, qg, sg = qo.synthetic_case(Mg, Kg, Ng, group_size=Gg, seed=5 + rank)
        gw = [(torch.from_numpy(qg).cuda(), torch.from_numpy(sg).cuda()) for _ in range(8)]  # 8 x 30 MB
        Xg = torch.from_numpy(xg).cuda()
        Yg = torch.empty(Mg, Ng, dtype=torch.float16, device="cuda")
        gsteps = max(10, min(args.steps, 50))
        gop = lambda i: ext.gemm_w4a16(Xg, gw[i % 8][0], gw[i % 8][1], Gg, out=Yg)
        gus = _graph_us(gop, gsteps, torch.cuda.Stream())
        if dist:
            t = torch.tensor([gus], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            gus = t.item()
        gemm_obj = {"workload": gm["name"], "us_per_launch": round(gus, 2),
                    "tflops": round(2.0 * Mg * Kg * Ng / (gus * 1e-6) / 1e12, 1),
                    "timing": f"one CUDA graph of {gsteps} launches, weights rotated over 8 copies (240 MB > L2), "
                              "device time, max over ranks"}
        del gw, Xg, Yg

    if rank == 0:
        hbm, tf, src = measured_peaks()
        if gemm_obj is not None:
            gemm_obj["roofline"] = {"bound": "tensor", "achieved": gemm_obj["tflops"], "peak": tf,
                                    "unit": "TFLOP/s", "frac": round(gemm_obj["tflops"] / tf, 4),
                                    "peak_source": f"{src} cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops)"}
        if args.workload == "gemv":
            achieved = nbytes / (per_ms * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(achieved / hbm, 4), "traffic": None,
                    "peak_source": f"{src} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                    "algorithmic_bytes_per_launch": nbytes}
        else:
            achieved = flops / (per_ms * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf, "unit": "TFLOP/s",
                    "frac": round(achieved / tf, 4), "traffic": None,
                    "peak_source": f"{src} cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops)",
                    "algorithmic_flops_per_launch": flops}
        traffic_file = os.path.join(ROOT, "profiles", f"traffic_{args.workload}.json")
        if os.path.exists(traffic_file):
            roof["traffic"] = json.load(open(traffic_file)).get("dram_bytes_per_launch")
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (BASELINE distributions: codes U[0,15], scales |N(0,1)|*0.02+1e-3, X~N(0,1); seeded)",
            "config": {"workload": wl["name"], "M": M, "K": K, "N": N, "group_size": G,
                       "l2": f"weights rotated over {nrot} copies ({nrot * wbytes / 1e6:.0f} MB > L2 {l2 / 1e6:.0f} MB)",
                       "parallelism": f"replicas x{world}", "timing": "one CUDA graph of `steps` launches"},
            "roofline": roof,
            "e2e": {"value": round(e2e_val, 2), "unit": unit, "h2d_bytes_per_step": M * K * 2,
                    "d2h_bytes_per_step": M * N * 2, "steps": e2e_steps,
                    "path": "nibblegemm_b200.gemv/gemm with pinned host X in, Y out, host sync per step"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "us_per_step": round(per_ms * 1e3, 3),
        }
        if gemm_obj is not None:
            line["prefill_gemm"] = gemm_obj
        if tp is not None:
            line["tp_decode8b"] = {
                "metric": "Llama-3-8B INT4 g128 decode tokens/s (BASELINE config 4), batch 1, context 1024",
                "value": round(1000.0 / tp["per_ms"], 2), "unit": "tok/s", "world": world,
                "parallelism": f"tp{world}", "reduce": args.reduce if world > 1 else None,
                "ms_per_token": round(tp["per_ms"], 4),
                "e2e_tok_s": round(1000.0 / tp["e2e_ms"], 2),
                "roofline_per_rank": {"bound": "hbm", "algorithmic_bytes": tp["nbytes"],
                                      "achieved_gbs": round(tp["nbytes"] / (tp["per_ms"] * 1e-3) / 1e9, 1),
                                      "frac": round(tp["nbytes"] / (tp["per_ms"] * 1e-3) / 1e9 / hbm, 4)},
                "gpu_launches_per_token": tp["launches"], "clocks": tp["clocks"],
                "timing": "device time of one CUDA-graph step, max over ranks; strong scaling (fixed model)",
            }
        if tpp is not None:
            tf, src = sustained_tflops()
            ach = tpp["flops"] / (tpp["per_ms"] * 1e-3) / 1e12
            line["tp_prefill70b"] = {
                "metric": "Llama-3-70B INT4 g128 prefill of 2048 prompt tokens (BASELINE config 5), batch 1",
                "value": round(1000.0 * PREFILL_TOKENS / tpp["per_ms"], 1), "unit": "tok/s", "world": world,
                "parallelism": f"tp{world}", "reduce": "nccl" if world > 1 else None,
                "ms_per_prefill": round(tpp["per_ms"], 3),
                "e2e_tok_s": round(1000.0 * PREFILL_TOKENS / tpp["e2e_ms"], 1),
                "roofline_per_rank": {"bound": "tensor", "algorithmic_flops": tpp["flops"],
                                      "achieved_tflops": round(ach, 1), "peak": tf, "frac": round(ach / tf, 4),
                                      "peak_source": f"{src} cuBLAS bf16 sustained"},
                "gpu_launches_per_prefill": tpp["launches"], "clocks": tpp["clocks"],
                "timing": "device time of 3 eager prefills after 2 warm-up, max over ranks; strong scaling (fixed model)",
            }
        if not args.no_cpu_baseline:
            v, per, sample, cores, extras = cpu_reference_sample(wl)
            if args.workload == "gemm":
                v = flops / per / 1e12
                extras["steady_state_value"] = round(flops / (extras["steady_state_ms_per_call"] * 1e-3) / 1e12, 6)
            line["cpu_baseline"] = {"value": round(v, 6), "unit": unit,
                                    "cores": cores, "kind": "port", "sample": sample,
                                    "ms_per_call": round(per * 1e3, 1), **extras}
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
