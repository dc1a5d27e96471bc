"""nibblegemm_b200 -- W4A16 (packed INT4 weight, fp16/bf16 activation) kernels for B200.

A drop-in for the hot path of arvindcr4/nibblegemm: the same packed format, the
same ops (``gemv_w4a16`` / ``gemm_w4a16`` / ``dequant_w4`` via ``extension()``),
the same Python names, the same ``QuantLinear`` -- with hand-written sm_100a
kernels behind a C ABI (``include/nibblegemm_b200.h``).
"""
from .ops import (DECODE_MAX_M, QuantLinear, check_device, dequant, dequantize, extension, gemm, gemv,
                  matmul, reference_matmul, set_debug_checks)
from .decode_model import LLAMA3_8B_MODEL, LLAMA3_70B_MODEL, Llama3Decoder
from .importers import from_autogptq, to_autogptq
from .quant import QuantizedWeight, pack_nibbles, quantize, unpack_nibbles

__all__ = [
    "LLAMA3_8B_MODEL",
    "LLAMA3_70B_MODEL",
    "Llama3Decoder",
    "from_autogptq",
    "to_autogptq",
    "DECODE_MAX_M",
    "QuantLinear",
    "QuantizedWeight",
    "check_device",
    "dequant",
    "dequantize",
    "reference_matmul",
    "set_debug_checks",
    "extension",
    "gemm",
    "gemv",
    "matmul",
    "pack_nibbles",
    "quantize",
    "unpack_nibbles",
]
__version__ = "0.1.0"
