"""Build ``nibblegemm_b200/libnibblegemm_b200.so`` from ``csrc/*.cu`` with nvcc.

    python -m nibblegemm_b200.build          # incremental
    python -m nibblegemm_b200.build --force  # rebuild everything
    python -m nibblegemm_b200.build -v       # also print ptxas resource usage

Every translation unit is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), without fast-math so the
kernels' rounding is the IEEE rounding the parity tests reason about.  The
library links the CUDA runtime statically; the driver API entry point it needs
(tensor-map encoding) is fetched with ``cudaGetDriverEntryPoint`` -- no torch,
no Python, no libcuda link.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libnibblegemm_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills", "-I", CSRC, "-I", INCLUDE,
]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if force or verbose or not os.path.exists(obj) or os.path.getmtime(obj) < newest_dep:
        cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, file=sys.stderr)
    return obj


TORCH_EXT_NAME = "nibblegemm_b200_torch"
TORCH_EXT_DIR = os.path.join(OBJ, "torchext")


def build_torch_binding(verbose: bool = False) -> str:
    """Compile ``csrc/torch_binding.cpp`` (the tensor-level ops over the C ABI)
    into ``_build/torchext/nibblegemm_b200_torch*.so``, linked against the
    library with an rpath to the package directory.  Host C++ only (no nvcc)."""
    import torch.utils.cpp_extension as ext
    os.makedirs(TORCH_EXT_DIR, exist_ok=True)
    ext.load(name=TORCH_EXT_NAME, sources=[os.path.join(CSRC, "torch_binding.cpp")],
             extra_include_paths=[INCLUDE], extra_cflags=["-O3", "-std=c++17"],
             extra_ldflags=[f"-L{PKG}", "-lnibblegemm_b200", f"-Wl,-rpath,{PKG}"],
             build_directory=TORCH_EXT_DIR, with_cuda=True, verbose=verbose, is_python_module=True)
    return torch_binding_path()


def torch_binding_path() -> str:
    """Path of the built binding module (may not exist)."""
    cands = sorted(glob.glob(os.path.join(TORCH_EXT_DIR, TORCH_EXT_NAME + "*.so")))
    return cands[0] if cands else os.path.join(TORCH_EXT_DIR, TORCH_EXT_NAME + ".so")


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    print(build_torch_binding(a.verbose))
