"""Torch-facing ops over the C ABI -- the reference's Python surface, B200 kernels.

Mirrors arvindcr4/nibblegemm ``python/nibblegemm/ops.py`` (names, arguments,
errors) and the pybind module ``csrc/bindings.cpp`` it builds:

* ``extension()`` returns an object with ``gemv_w4a16``, ``gemm_w4a16`` and
  ``dequant_w4`` taking tensors, like the reference's JIT-built module.  Here
  the kernels are a prebuilt sm_100a shared library reached through ctypes;
  the call is enqueued on the current torch stream of the input's device.
* ``dequant``, ``gemv``, ``gemm``, ``matmul``, ``DECODE_MAX_M``, ``QuantLinear``.

Validation failures raise ``RuntimeError`` (the reference's TORCH_CHECK
behaviour); ``matmul`` raises ``ValueError`` for rank / K mismatches, as the
reference does.  There is no CPU path: tensors must be on a CUDA device.
"""
from __future__ import annotations

import contextlib
from typing import Optional

import torch

from . import _lib
from .quant import QuantizedWeight, quantize  # noqa: F401  (re-exported)

#: Batch sizes at or below this go to the bandwidth-bound decode GEMV.
DECODE_MAX_M = 8

_DTYPE_CODE = {torch.float16: _lib.NG_DTYPE_F16, torch.bfloat16: _lib.NG_DTYPE_BF16}


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _on_device(dev: torch.device):
    """Make ``dev`` current for the C call (a no-op when it already is)."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def _check_weight(Wq: torch.Tensor, S: torch.Tensor, dev: torch.device) -> None:
    _require(Wq.is_cuda and S.is_cuda, "all tensors must live on CUDA")
    _require(Wq.device == dev and S.device == dev, "all tensors must be on the same device")
    _require(Wq.dtype == torch.int32, "packed weights must be int32")
    _require(S.dtype == torch.float16, "scales must be fp16")
    _require(Wq.is_contiguous() and S.is_contiguous(), "inputs must be contiguous")
    _require(Wq.dim() == 2 and S.dim() == 2, "expected 2-D inputs")


def _check_act(X: torch.Tensor, Wq: torch.Tensor, S: torch.Tensor, group_size: int):
    _require(X.is_cuda, "all tensors must live on CUDA")
    _check_weight(Wq, S, X.device)
    _require(X.dtype in _DTYPE_CODE, "activations must be fp16 or bf16")
    _require(X.is_contiguous(), "inputs must be contiguous")
    _require(X.dim() == 2, "expected 2-D inputs")
    M, K = X.shape
    N = Wq.size(1)
    _require(Wq.size(0) * 8 == K, "packed weight rows disagree with K")
    _require(group_size > 0 and S.size(0) * group_size == K, "scale rows disagree with K/group_size")
    _require(S.size(1) == N, "scale columns disagree with N")
    return M, K, N


def _out(out, M, N, X):
    if out is None:
        return torch.empty((M, N), dtype=X.dtype, device=X.device)
    _require(out.shape == (M, N) and out.dtype == X.dtype and out.device == X.device
             and out.is_contiguous(), "out must be a contiguous [M, N] tensor like X")
    return out


class _Extension:
    """Tensor-level ops with the reference extension's signatures."""

    def __init__(self):
        self.lib = _lib.load()
        self._ws = {}  # (device index, stream handle) -> zero-initialised GEMV workspace
        self._gws = {}  # (device index, stream handle) -> zero-initialised GEMM split-K workspace

    def gemm_workspace(self, M: int, N: int, device: torch.device, stream: int) -> torch.Tensor:
        """The prefill-GEMM split-K workspace for (device, stream), grown on demand
        (zero-filled once; every call leaves its per-tile counters at zero)."""
        need = self.lib.ng_gemm_workspace_bytes(M, N)
        key = (device.index, stream)
        ws = self._gws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
            self._gws[key] = ws
        return ws

    def workspace(self, N: int, device: torch.device, stream: int) -> torch.Tensor:
        """The decode-GEMV workspace for (device, stream), grown on demand.

        Allocated zero-filled once; every call leaves its arrival counters at
        zero, so it is reused as is (also across CUDA-graph replays).  One per
        stream, because calls sharing a workspace must not overlap on the GPU.
        """
        need = self.lib.ng_gemv_workspace_bytes(1, N)
        key = (device.index, stream)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 4 << 20), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def dequant_w4(self, Wq: torch.Tensor, S: torch.Tensor, group_size: int, fast: bool = True,
                   out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        _check_weight(Wq, S, Wq.device)
        K, N = Wq.size(0) * 8, Wq.size(1)
        _require(S.size(1) == N, "scale columns disagree with N")
        _require(group_size > 0 and S.size(0) * group_size == K, "scale rows disagree with K/group_size")
        _require(out_dtype in _DTYPE_CODE, "out_dtype must be fp16 or bf16")
        out = torch.empty((K, N), dtype=out_dtype, device=Wq.device)
        with _on_device(Wq.device):
            st = self.lib.ng_dequant_w4(Wq.data_ptr(), S.data_ptr(), out.data_ptr(),
                                        _DTYPE_CODE[out_dtype], K, N, int(group_size), int(bool(fast)),
                                        torch.cuda.current_stream().cuda_stream)
        _lib.check(st, "dequant_w4")
        return out

    def gemv_w4a16(self, X: torch.Tensor, Wq: torch.Tensor, S: torch.Tensor, group_size: int,
                   version: int = 4, splits_override: int = 0, threads_override: int = 0,
                   algo: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M, K, N = _check_act(X, Wq, S, group_size)
        _require(N % 4 == 0, "N must be a multiple of 4 for 128-bit weight loads")
        _require(group_size in (64, 128, 256), "group_size must be 64, 128 or 256")
        _require(1 <= M <= 16, "gemv path supports 1 <= M <= 16; use gemm_w4a16 for larger M")
        _require(version in (0, 1, 2, 3, 4), "version must be one of 0..4")
        # Version 3 of the reference ladder is version 4 pinned to one K split.
        splits = 1 if version == 3 else int(splits_override)
        y = _out(out, M, N, X)
        with _on_device(X.device):
            stream = torch.cuda.current_stream().cuda_stream
            ws = self.workspace(N, X.device, stream)
            st = self.lib.ng_gemv_w4a16(X.data_ptr(), _DTYPE_CODE[X.dtype], Wq.data_ptr(),
                                        S.data_ptr(), y.data_ptr(), M, K, N, int(group_size), splits,
                                        int(threads_override), int(algo), ws.data_ptr(), ws.numel(),
                                        stream)
        _lib.check(st, "gemv_w4a16")
        return y

    def gemm_w4a16(self, X: torch.Tensor, Wq: torch.Tensor, S: torch.Tensor, group_size: int,
                   version: int = 6, tile_tokens: int = 0,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M, K, N = _check_act(X, Wq, S, group_size)
        _require(version in (6, 7), "version must be 6 or 7")
        y = _out(out, M, N, X)
        with _on_device(X.device):
            stream = torch.cuda.current_stream().cuda_stream
            ws = self.gemm_workspace(M, N, X.device, stream)
            st = self.lib.ng_gemm_w4a16(X.data_ptr(), _DTYPE_CODE[X.dtype], Wq.data_ptr(),
                                        S.data_ptr(), y.data_ptr(), M, K, N, int(group_size),
                                        int(tile_tokens), ws.data_ptr(), ws.numel(), stream)
        _lib.check(st, "gemm_w4a16")
        return y

    def device_status(self) -> int:
        """Synchronise the current stream and return (and clear) the device error word."""
        return self.lib.ng_device_status(torch.cuda.current_stream().cuda_stream)


_ext: Optional[_Extension] = None


def extension() -> _Extension:
    """Load (once) and return the kernel library's tensor-level ops."""
    global _ext
    if _ext is None:
        _ext = _Extension()
    return _ext


def dequant(qw: QuantizedWeight, fast: bool = True, dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """Expand packed INT4 to a dense ``[K, N]`` matrix on the weight's device."""
    return extension().dequant_w4(qw.qweight, qw.scales, qw.group_size, fast, out_dtype=dtype)


def gemv(X: torch.Tensor, qw: QuantizedWeight, version: int = 4, splits: int = 0,
         block_threads: int = 0, algo: int = 0) -> torch.Tensor:
    """Decode-regime ``X @ dequant(qw)`` for 1 <= M <= 16.

    ``splits`` (K slices = cluster size, 1..16) and ``block_threads`` (128/256)
    override the launch heuristic; 0 lets it decide.  ``version`` is accepted
    for compatibility with the reference's ladder (3 = a single K split).
    """
    return extension().gemv_w4a16(X, qw.qweight, qw.scales, qw.group_size, version, splits,
                                  block_threads, algo)


def gemm(X: torch.Tensor, qw: QuantizedWeight, version: int = 6) -> torch.Tensor:
    """Prefill-regime tensor-core ``X @ dequant(qw)`` (tcgen05, TMEM accumulators)."""
    return extension().gemm_w4a16(X, qw.qweight, qw.scales, qw.group_size, version)


def matmul(X: torch.Tensor, qw: QuantizedWeight, splits: int = 0,
           block_threads: int = 0) -> torch.Tensor:
    """``X @ dequant(qw)``, dispatching on batch size at ``DECODE_MAX_M``."""
    if X.dim() != 2:
        raise ValueError(f"expected a 2-D activation matrix, got {tuple(X.shape)}")
    if X.size(1) != qw.K:
        raise ValueError(f"K mismatch: activations have {X.size(1)}, weights have {qw.K}")
    if X.size(0) <= DECODE_MAX_M:
        return gemv(X, qw, version=4, splits=splits, block_threads=block_threads)
    return gemm(X, qw)


class QuantLinear(torch.nn.Module):
    """Drop-in ``nn.Linear`` with packed INT4 weights (reference ops.py:107-135).

    Buffers ``qweight``, ``scales`` and ``bias`` keep the reference's names, so
    state dicts move between the two libraries unchanged.
    """

    def __init__(self, qw: QuantizedWeight, bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.register_buffer("qweight", qw.qweight)
        self.register_buffer("scales", qw.scales)
        self.register_buffer("bias", bias if bias is not None else None)
        self.group_size, self.K, self.N = qw.group_size, qw.K, qw.N

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, group_size: int = 128) -> "QuantLinear":
        # nn.Linear stores [out, in]; the kernels consume [in, out].
        qw = quantize(linear.weight.data.t().contiguous(), group_size)
        bias = linear.bias.data.clone() if linear.bias is not None else None
        return cls(qw.to(linear.weight.device), bias)

    def _qw(self) -> QuantizedWeight:
        return QuantizedWeight(self.qweight, self.scales, self.group_size, self.K, self.N)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        y = matmul(x.reshape(-1, shape[-1]).contiguous(), self._qw())
        y = y.reshape(*shape[:-1], self.N)
        return y + self.bias if self.bias is not None else y
