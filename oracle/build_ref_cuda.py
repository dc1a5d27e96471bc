"""Build the reference's own CUDA extension for the B200 (test infrastructure).

The reference (arvindcr4/nibblegemm) JIT-builds ``csrc/bindings.cpp``,
``gemv_w4a16.cu``, ``gemm_w4a16.cu`` and ``dequant_kernel.cu`` with
``torch.utils.cpp_extension.load`` for sm_80 (``python/nibblegemm/ops.py:37-56``).
This recipe compiles those same files, where they lie in the reference
checkout, unmodified, with the reference's own flags but for sm_100a, and
writes the module only into ``oracle/_ref/cuda/``.  That directory is
git-ignored and travels to the GPU box with the other built files.  The
product never loads it.  It is the comparison that ``tests/test_reference_gpu.py``
runs: the reference's Ampere-era kernels (``mma.sync`` / ``wmma``) recompiled
for the B200, side by side with this library's kernels on the same inputs.

    python -m oracle.build_ref_cuda [/path/to/reference]
"""
from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "cuda")
NAME = "nibblegemm_ref_cuda"
SOURCES = ["bindings.cpp", "gemv_w4a16.cu", "gemm_w4a16.cu", "dequant_kernel.cu"]
DEFAULT_REF = os.environ.get("NIBBLEGEMM_REFERENCE", os.path.join(os.sep, "root", "reference"))


def module_path() -> str:
    """The built module, or '' if it has not been built."""
    c = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return c[0] if c else ""


def build(ref_root: str = DEFAULT_REF, verbose: bool = False) -> str:
    csrc = os.path.join(ref_root, "csrc")
    if not all(os.path.exists(os.path.join(csrc, s)) for s in SOURCES):
        return ""
    from torch.utils.cpp_extension import load
    os.makedirs(OUT, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    load(name=NAME, sources=[os.path.join(csrc, s) for s in SOURCES],
         extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=["-O3", "-std=c++17", "--expt-relaxed-constexpr", "-lineinfo"],
         extra_include_paths=[csrc], build_directory=OUT, verbose=verbose, is_python_module=False)
    return module_path()


def load_module():
    """Import the built module (raises if absent)."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (the module links against torch)
    path = module_path()
    if not path:
        raise FileNotFoundError("reference CUDA module not built")
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF, verbose=True) or "reference not found")
