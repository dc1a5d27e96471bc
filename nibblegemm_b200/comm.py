"""Tensor-parallel reduction over NVLink peer memory (the ``ng_allreduce_sum`` kernel).

``PeerAllReduce`` sets up the one-shot all-reduce of ``include/nibblegemm_b200.h``
for a ``torch.distributed`` group of ranks on one node: each rank allocates its
exchange buffer, exports it with CUDA IPC, and maps every peer's buffer; the
handles travel through the process group.  ``__call__`` reduces a contiguous
fp16/bf16 tensor in place on the current stream (CUDA-graph capturable: the
call counters live on the device).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_DT = {torch.float16: _lib.NG_DTYPE_F16, torch.bfloat16: _lib.NG_DTYPE_BF16}


class PeerBuffers:
    """One zero-filled exchange buffer per rank of a ``torch.distributed`` group on
    one node, allocated by the library (``ng_ipc_alloc``), exported as a CUDA IPC
    handle and mapped by every peer; ``ptrs`` is the ctypes array of every rank's
    buffer as mapped in this process (this rank's own at index ``rank``)."""

    def __init__(self, nbytes: int, group=None, device=None):
        self.lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            base, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            _lib.check(self.lib.ng_ipc_alloc(int(nbytes), ctypes.byref(base), handle), "ng_ipc_alloc")
        self._base = base.value
        infos = [None] * self.world
        dist.all_gather_object(infos, handle.raw, group=group)
        self._opened, ptrs = [], []
        for p, h in enumerate(infos):
            if p == self.rank:
                ptrs.append(self._base)
                continue
            out = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(self.lib.ng_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(out)),
                           "ng_ipc_open")
            self._opened.append(out.value)
            ptrs.append(out.value)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def close(self):
        """Unmap the peers' buffers, then free this rank's (call on every rank,
        after a barrier, when nothing is in flight)."""
        for p in self._opened:
            self.lib.ng_ipc_close(p)
        self._opened = []
        if self._base:
            self.lib.ng_ipc_free(self._base)
            self._base = None


class PeerAllReduce:
    def __init__(self, max_elems: int, group=None, device=None):
        self.lib = _lib.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_elems = int(max_elems)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        nbytes = self.lib.ng_allreduce_buffer_bytes(self.world, self.max_elems)
        if nbytes == 0:
            raise RuntimeError(f"unsupported world size {self.world}")
        self.epochs = torch.zeros(16, dtype=torch.int32, device=self.device)
        # The exchange buffer is the library's own cudaMalloc (not the torch
        # caching allocator), so its IPC handle covers exactly this buffer.
        with torch.cuda.device(self.device):
            base, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            _lib.check(self.lib.ng_ipc_alloc(nbytes, ctypes.byref(base), handle), "ng_ipc_alloc")
        self._base = base.value
        infos = [None] * self.world
        dist.all_gather_object(infos, handle.raw, group=group)
        self._opened = []
        ptrs = []
        for p, h in enumerate(infos):
            if p == self.rank:
                ptrs.append(self._base)
                continue
            out = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(self.lib.ng_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(out)),
                           "ng_ipc_open")
            self._opened.append(out.value)
            ptrs.append(out.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        if not (t.is_cuda and t.is_contiguous() and t.dtype in _DT):
            raise RuntimeError("PeerAllReduce needs a contiguous fp16/bf16 CUDA tensor")
        st = self.lib.ng_allreduce_sum(t.data_ptr(), _DT[t.dtype], t.numel(), self._ptrs, self.rank,
                                       self.world, self.max_elems, self.epochs.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
        _lib.check(st, "ng_allreduce_sum")
        return t

    def close(self):
        """Unmap the peers' buffers, then free this rank's (call on every rank,
        after a barrier, when no reduction is in flight)."""
        for p in self._opened:
            self.lib.ng_ipc_close(p)
        self._opened = []
        if self._base:
            self.lib.ng_ipc_free(self._base)
            self._base = None
