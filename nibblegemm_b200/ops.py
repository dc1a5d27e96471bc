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
import os
from typing import Optional

import torch

from . import _lib
from .quant import QuantizedWeight, quantize  # noqa: F401  (re-exported)

#: Batch sizes at or below this go to the bandwidth-bound decode GEMV.  The
#: reference's crossover is 8 (ops.py:29-30); on B200 the GEMV stays ahead of the
#: tcgen05 GEMM through M = 16 (4096 x 14336: 34.8 vs 38.9 us; 14336 x 4096:
#: 26.4 vs 43.5 us, CUDA graph), and 16 is the largest M the GEMV takes.
DECODE_MAX_M = 16

_DTYPE_CODE = {torch.float16: _lib.NG_DTYPE_F16, torch.bfloat16: _lib.NG_DTYPE_BF16}


#: When true, every op synchronises its stream after the launch and raises if a
#: kernel reported a bounded-wait timeout or a bad index (see ``check_device``).
#: Off by default: it costs a host synchronisation per call and cannot be used
#: inside CUDA-graph capture.  Also enabled by ``NIBBLEGEMM_DEBUG=1``.
DEBUG_CHECKS = os.environ.get("NIBBLEGEMM_DEBUG", "") not in ("", "0")


def set_debug_checks(enabled: bool) -> None:
    """Turn the per-op device-status check on or off."""
    global DEBUG_CHECKS
    DEBUG_CHECKS = bool(enabled)


def check_device() -> None:
    """Synchronise the current stream and raise ``NibbleError`` if a kernel of
    this library gave up on a bounded wait (its output is then undefined) or met
    an out-of-range index since the last check; clears the flag."""
    _lib.check(extension().device_status(), "device status")


def _after(op: str) -> None:
    if DEBUG_CHECKS and not torch.cuda.is_current_stream_capturing():
        _lib.check(extension().device_status(), op)


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


def _load_binding():
    """The compiled tensor-level binding (``csrc/torch_binding.cpp``), or None if
    it has not been built (the ops then marshal through ctypes: same kernels,
    more host time per call)."""
    import importlib.machinery
    import importlib.util
    from .build import TORCH_EXT_NAME, torch_binding_path
    path = torch_binding_path()
    if not os.path.exists(path):
        return None
    loader = importlib.machinery.ExtensionFileLoader(TORCH_EXT_NAME, path)
    spec = importlib.util.spec_from_loader(TORCH_EXT_NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


class _Extension:
    """Tensor-level ops with the reference extension's signatures."""

    def __init__(self):
        self.lib = _lib.load()
        self.binding = _load_binding()
        self._ws = {}  # (device index, stream handle) -> zero-initialised GEMV workspace
        self._gws = {}  # (device index, stream handle) -> zero-initialised GEMM split-K workspace

    def gemm_workspace(self, M: int, N: int, device: torch.device, stream: int) -> torch.Tensor:
        """The prefill-GEMM split-K workspace for (device, stream), grown on demand
        (zero-filled once; every call leaves its per-tile counters at zero)."""
        need = self.lib.ng_gemm_workspace_bytes(M, N)
        if self.binding is not None:
            return self.binding.workspace(device.index, stream, 1, need)
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
        if self.binding is not None:
            return self.binding.workspace(device.index, stream, 0, need)
        key = (device.index, stream)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 4 << 20), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def dequant_w4(self, Wq: torch.Tensor, S: torch.Tensor, group_size: int, fast: bool = True,
                   out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if self.binding is not None:
            out, st = self.binding.dequant_w4(Wq, S, int(group_size), bool(fast), out_dtype)
            _lib.check(st, "dequant_w4")
            _after("dequant_w4")
            return out
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
        _after("dequant_w4")
        return out

    def gemv_w4a16(self, X: torch.Tensor, Wq: torch.Tensor, S: torch.Tensor, group_size: int,
                   version: int = 4, splits_override: int = 0, threads_override: int = 0,
                   algo: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.binding is not None:
            y, st = self.binding.gemv_w4a16(X, Wq, S, int(group_size), int(version), int(splits_override),
                                            int(threads_override), int(algo), out)
            _lib.check(st, "gemv_w4a16")
            _after("gemv_w4a16")
            return y
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
        _after("gemv_w4a16")
        return y

    def gemm_w4a16(self, X: torch.Tensor, Wq: torch.Tensor, S: torch.Tensor, group_size: int,
                   version: int = 6, tile_tokens: int = 0,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.binding is not None:
            y, st = self.binding.gemm_w4a16(X, Wq, S, int(group_size), int(version), int(tile_tokens), out)
            _lib.check(st, "gemm_w4a16")
            _after("gemm_w4a16")
            return y
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
        _after("gemm_w4a16")
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


def dequantize(qw: QuantizedWeight) -> torch.Tensor:
    """The reference's ``dequantize``: dense fp16 ``[K, N]`` = (u - 8) * scale with
    one rounding, on ``qw``'s device.  A CPU weight is expanded by the GPU kernel
    on the current CUDA device and the result returned to the CPU (there is no
    CPU implementation in this library)."""
    if qw.qweight.is_cuda:
        return dequant(qw)
    return dequant(qw.to(torch.device("cuda", torch.cuda.current_device()))).cpu()


def reference_matmul(X: torch.Tensor, qw: QuantizedWeight) -> torch.Tensor:
    """The reference's accuracy yardstick: fp16(X.float() @ dequantize(qw).float()),
    on X's device (dense fp32 product; slow, for checking, not serving)."""
    W = dequantize(qw).to(X.device)
    return (X.float() @ W.float()).to(torch.float16)


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
    """``X @ dequant(qw)`` routed by the number of rows of ``X``.

    Up to ``DECODE_MAX_M`` rows the product is a bandwidth-bound GEMV (one pass
    over the packed weight); beyond that it is a tensor-core GEMM.  ``splits`` and
    ``block_threads`` reach the GEMV only.  Shape errors raise ``ValueError``.
    """
    if X.dim() != 2:
        raise ValueError(f"matmul takes a 2-D [M, K] activation, not shape {tuple(X.shape)}")
    rows, depth = X.shape
    if depth != qw.K:
        raise ValueError(f"activation depth {depth} does not match the weight's K = {qw.K}")
    use_gemv = rows <= DECODE_MAX_M
    return (gemv(X, qw, version=4, splits=splits, block_threads=block_threads) if use_gemv
            else gemm(X, qw))


class QuantLinear(torch.nn.Module):
    """``nn.Linear`` replacement holding a packed INT4 weight.

    The state-dict entries are ``qweight`` ([K/8, N] int32), ``scales`` ([K/G, N]
    fp16) and ``bias`` (optional), the names the reference library uses, so a
    checkpoint of one loads into the other.  ``forward`` accepts any leading
    shape ``[..., K]`` and returns ``[..., N]``.
    """

    def __init__(self, qw: QuantizedWeight, bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.K, self.N, self.group_size = qw.K, qw.N, qw.group_size
        for name, t in (("qweight", qw.qweight), ("scales", qw.scales), ("bias", bias)):
            self.register_buffer(name, t)

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, group_size: int = 128) -> "QuantLinear":
        """Quantise an existing layer (round-to-nearest, per-group scales)."""
        weight_kn = linear.weight.detach().transpose(0, 1).contiguous()  # Linear keeps [N, K]
        packed = quantize(weight_kn, group_size).to(linear.weight.device)
        bias = None if linear.bias is None else linear.bias.detach().clone()
        return cls(packed, bias)

    def packed(self) -> QuantizedWeight:
        """The layer's weight as a :class:`QuantizedWeight` view of its buffers."""
        return QuantizedWeight(self.qweight, self.scales, self.group_size, self.K, self.N)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        out = matmul(x.reshape(-1, x.shape[-1]).contiguous(), self.packed()).view(*lead, self.N)
        if self.bias is None:
            return out
        return out + self.bias
