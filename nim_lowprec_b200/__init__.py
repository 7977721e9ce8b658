"""nim_lowprec_b200 -- B200 (sm_100a) implementation of nim-lowprec's fused
dequant-GEMV/GEMM hot path behind the reference's own kernel API.

The kernels live in liblowprec_cuda.so (built from csrc/ by
``python nim_lowprec_b200/build.py``); this package binds its C ABI and
mirrors the reference's Nim procs.  There is no CPU fallback: importing the
API without the built library raises.
"""
from . import _native
from .dequant import (  # noqa: F401
    batch, calibrateMX, calibrateSymmetric, dequantGemmF4, dequantGemmI4Q8, dequantGemmQ8, dequantGemv,
    dequantGemvF4, dequantGemvI4, dequantGemvI4Q8, dequantGemvQ4_0, dequantGemvQ4_0Q8,
    dequantGemvQ8, dequantGemvQ8_0, dequantGemvQ8_0Q8, dequantGemvQ4_K, dequantGemvQ6_K,
    dequantizeBatch, dequantizeQ4_0Batch,
    dequantizeQ4_K, dequantizeQ6_K, dequantizeQ8_0Batch, dequantizeNVFP4, quantizeBatch,
    quantizeNVFP4, quantizeF4Packed, quantizeI4Packed, quantizeQ4_0, quantizeDequantGemvI4Q8,
    quantizeDequantGemvQ8,
    quantizeQ4_0Batch, quantizeQ8_0, quantizeQ8_0Batch, quantizeQ8_0Split, fp32_mode,
    fp32Mode, gemmNVFP4, setFp32Mode)
from .ggml import QK, QK_K, BlockQ4_0, BlockQ4_K, BlockQ6_K, BlockQ8_0  # noqa: F401
from . import parallel  # noqa: F401  (LpPool's row-sharded forms)

_native.lib()  # fail loudly at import if the CUDA library is missing

__version__ = "0.1.0"
