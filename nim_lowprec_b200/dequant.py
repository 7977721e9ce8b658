"""The reference's kernel API, proc for proc, over the CUDA library.

Names, argument order and meaning follow nim-lowprec's ``simd/dequant`` and
``ggml``/``quant`` procs (cited per function).  As in the reference, shapes
come from array lengths and the output ``y`` (``var openArray[float32]``) is
written in place.  A failed shape precondition raises ``AssertionError`` (the
reference's ``assert``).

Arrays may be
  * torch CUDA tensors: the device path (``lp_*``), stream-ordered on
    ``torch.cuda.current_stream()``;
  * numpy arrays: the host drop-in path (``lph_*``), blocking, with every
    input copied to the device and ``y`` copied back.
Mixing the two in one call is an error.  Everything must be C-contiguous.
ggml block arrays are numpy structured arrays of ``BlockQ8_0``/``BlockQ4_0``
or uint8 arrays/tensors whose total size is a multiple of the block size.
"""
from __future__ import annotations

import contextlib

import numpy as np

from . import _native as N
from .ggml import Q4_0_BYTES, Q4_K_BYTES, Q6_K_BYTES, Q8_0_BYTES

try:  # torch is optional for the host path
    import torch
except Exception:  # pragma: no cover
    torch = None


def _is_tensor(a) -> bool:
    return torch is not None and isinstance(a, torch.Tensor)


def _mode(*arrs) -> str:
    dev = [a for a in arrs if a is not None]
    kinds = {("dev" if _is_tensor(a) else "host") for a in dev}
    if len(kinds) != 1:
        raise TypeError("pass all-torch-CUDA or all-numpy arrays, not a mix")
    kind = kinds.pop()
    if kind == "dev":
        for a in dev:
            if not a.is_cuda:
                raise TypeError("torch tensors must live on a CUDA device")
            if not a.is_contiguous():
                raise ValueError("tensors must be contiguous")
    else:
        for a in dev:
            if not isinstance(a, np.ndarray):
                raise TypeError(f"expected numpy array, got {type(a).__name__}")
            if not a.flags["C_CONTIGUOUS"]:
                raise ValueError("arrays must be C-contiguous")
    return kind


_TORCH_DT = {}
if torch is not None:
    _TORCH_DT = {torch.int8: np.int8, torch.uint8: np.uint8, torch.float32: np.float32}


def _check_dtype(a, want, name):
    if a is None:
        return
    got = _TORCH_DT.get(a.dtype) if _is_tensor(a) else a.dtype
    if got is None or np.dtype(got) != np.dtype(want):
        raise TypeError(f"{name}: expected {np.dtype(want)}, got {a.dtype}")


def _numel(a) -> int:
    return 0 if a is None else (a.numel() if _is_tensor(a) else a.size)


def _ptr(a):
    if a is None:
        return None
    return a.data_ptr() if _is_tensor(a) else a.ctypes.data


def _blocks(a, bb: int) -> int:
    """Block count of a ggml block array (structured or raw bytes)."""
    if isinstance(a, np.ndarray) and a.dtype.fields is not None:
        if a.dtype.itemsize != bb:
            raise TypeError(f"block dtype itemsize {a.dtype.itemsize} != {bb}")
        return a.size
    _check_dtype(a, np.uint8, "blocks")
    n = _numel(a)
    if n % bb:
        raise AssertionError(f"block array of {n} bytes is not a multiple of {bb}")
    return n // bb


def _stream():
    return torch.cuda.current_stream().cuda_stream


@contextlib.contextmanager
def batch():
    """Run the int8-activation GEMVs made inside as persistent launches
    (lp_batch_begin / lp_batch_end on the current stream; no counterpart in
    the reference).  Calls of dequantGemvQ8/I4Q8, quantizeDequantGemvQ8/I4Q8,
    dequantGemvQ8_0Q8/Q4_0Q8 and their pooled forms are queued and launched
    together -- up to 64 consecutive same-format calls per launch -- with the
    results of the calls made one by one, bit for bit.  Any other call of the
    library launches the queue first.  Device tensors only, and every tensor
    a queued call reads or writes must stay alive until the block ends (a
    temporary freed earlier may be reused by the allocator before the launch)."""
    st = _stream()
    N.check(N.lib().lp_batch_begin(st), "batch_begin")
    ok = False
    try:
        yield
        ok = True
    finally:
        r = N.lib().lp_batch_end(st)
        if ok:
            N.check(r, "batch_end")


def _call(mode, name, *args):
    L = N.lib()
    if mode == "dev":
        st = getattr(L, "lp_" + name)(*args, _stream())
    else:
        st = getattr(L, "lph_" + name)(*args)
    N.check(st, name)


# ====================================== fp32-activation fused GEMVs ======

def _gemv_group(name, w, scales, groupSize, x, y, wdt):
    mode = _mode(w, scales, x, y)
    _check_dtype(w, wdt, "w"); _check_dtype(scales, np.float32, "scales")
    _check_dtype(x, np.float32, "x"); _check_dtype(y, np.float32, "y")
    _call(mode, name, _ptr(w), _numel(w), _ptr(scales), _numel(scales), int(groupSize),
          _ptr(x), _numel(x), _ptr(y), _numel(y))


def dequantGemv(wq, scales, groupSize, x, y):
    """simd/dequant.nim:210-257: int8 weights, fp32 activations."""
    _gemv_group("dequant_gemv", wq, scales, groupSize, x, y, np.int8)


def dequantGemvI4(wpacked, scales, groupSize, x, y):
    """simd/dequant.nim:259-339: packed int4 weights (low nibble = even column)."""
    _gemv_group("dequant_gemv_i4", wpacked, scales, groupSize, x, y, np.uint8)


def dequantGemvF4(wpacked, scales, groupSize, x, y):
    """simd/dequant.nim:341-420: packed MXFP4 (e2m1) weights, fp32 E8M0 scales."""
    _gemv_group("dequant_gemv_f4", wpacked, scales, groupSize, x, y, np.uint8)


def _gemv_blocks(name, w, bb, blocksPerRow, x, y, xq_blocks=False):
    mode = _mode(w, x, y)
    nw = _blocks(w, bb)
    if xq_blocks:
        nx = _blocks(x, Q8_0_BYTES)
    else:
        _check_dtype(x, np.float32, "x")
        nx = _numel(x)
    _check_dtype(y, np.float32, "y")
    _call(mode, name, _ptr(w), nw, int(blocksPerRow), _ptr(x), nx, _ptr(y), _numel(y))


def dequantGemvQ8_0(w, blocksPerRow, x, y):
    """simd/dequant.nim:530-568: ggml Q8_0 weights, fp32 activations."""
    _gemv_blocks("dequant_gemv_q8_0", w, Q8_0_BYTES, blocksPerRow, x, y)


def dequantGemvQ4_0(w, blocksPerRow, x, y):
    """simd/dequant.nim:570-622: ggml Q4_0 weights, fp32 activations."""
    _gemv_blocks("dequant_gemv_q4_0", w, Q4_0_BYTES, blocksPerRow, x, y)


# ------------------------------------------------ fp32 arithmetic mode

_MODES = {"fast": N.LP_FP32_FAST, "exact": N.LP_FP32_EXACT}


def setFp32Mode(mode: str) -> None:
    """Arithmetic of the fp32-activation GEMVs, process-wide.

    ``"fast"`` (default): block-float activations with exact integer group
    dots, within the reference's fp32 tolerance (1e-5 relative).
    ``"exact"``: the reference scalar path's operation order, bit-identical.
    """
    if mode not in _MODES:
        raise ValueError(f"fp32 mode must be one of {sorted(_MODES)}, not {mode!r}")
    N.check(N.lib().lp_set_fp32_mode(_MODES[mode]), "lp_set_fp32_mode")


def fp32Mode() -> str:
    v = int(N.lib().lp_get_fp32_mode())
    return {b: a for a, b in _MODES.items()}[v]


class fp32_mode:
    """Context manager: ``with fp32_mode("exact"): ...``."""

    def __init__(self, mode: str):
        self.mode = mode
        self.prev = None

    def __enter__(self):
        self.prev = fp32Mode()
        setFp32Mode(self.mode)
        return self

    def __exit__(self, *exc):
        setFp32Mode(self.prev)
        return False


# ====================================== int8-activation GEMVs ===========

def _gemv_q8(name, w, wScales, groupSize, xq, xScales, y, wdt):
    mode = _mode(w, wScales, xq, xScales, y)
    _check_dtype(w, wdt, "w"); _check_dtype(wScales, np.float32, "wScales")
    _check_dtype(xq, np.int8, "xq"); _check_dtype(xScales, np.float32, "xScales")
    _check_dtype(y, np.float32, "y")
    _call(mode, name, _ptr(w), _numel(w), _ptr(wScales), _numel(wScales), int(groupSize),
          _ptr(xq), _numel(xq), _ptr(xScales), _numel(xScales), _ptr(y), _numel(y))


def dequantGemvQ8(wq, wScales, groupSize, xq, xScales, y):
    """simd/dequant.nim:753-878: int8 x int8, exact int32 group sums."""
    _gemv_q8("dequant_gemv_q8", wq, wScales, groupSize, xq, xScales, y, np.int8)


def dequantGemvI4Q8(wpacked, wScales, groupSize, xq, xScales, y):
    """simd/dequant.nim:968-1145: packed int4 x int8."""
    _gemv_q8("dequant_gemv_i4q8", wpacked, wScales, groupSize, xq, xScales, y, np.uint8)


def _quantize_gemv_q8(name, w, wScales, groupSize, x, y, wdt):
    _dev_only(name, w, wScales, x, y)
    _check_dtype(w, wdt, "w"); _check_dtype(wScales, np.float32, "wScales")
    _check_dtype(x, np.float32, "x"); _check_dtype(y, np.float32, "y")
    N.check(getattr(N.lib(), "lp_" + name)(_ptr(w), _numel(w), _ptr(wScales), _numel(wScales),
                                          int(groupSize), _ptr(x), _numel(x), _ptr(y), _numel(y),
                                          _stream()), name)


def quantizeDequantGemvQ8(wq, wScales, groupSize, x, y):
    """quantizeQ8_0 of fp32 x (ggml.nim:60-75) then dequantGemvQ8
    (simd/dequant.nim:753-878) in one launch; the two calls' bits.
    groupSize must be 32."""
    _quantize_gemv_q8("quantize_dequant_gemv_q8", wq, wScales, groupSize, x, y, np.int8)


def quantizeDequantGemvI4Q8(wpacked, wScales, groupSize, x, y):
    """quantizeQ8_0 of fp32 x then dequantGemvI4Q8 (simd/dequant.nim:968-1145)
    in one launch; the two calls' bits.  groupSize must be 32."""
    _quantize_gemv_q8("quantize_dequant_gemv_i4q8", wpacked, wScales, groupSize, x, y, np.uint8)


def dequantGemvQ8_0Q8(w, blocksPerRow, xq, y):
    """simd/dequant.nim:1187-1286: Q8_0 weights x Q8_0 activation blocks."""
    _gemv_blocks("dequant_gemv_q8_0q8", w, Q8_0_BYTES, blocksPerRow, xq, y, xq_blocks=True)


def dequantGemvQ4_0Q8(w, blocksPerRow, xq, y):
    """simd/dequant.nim:1288-1365: Q4_0 weights x Q8_0 activation blocks."""
    _gemv_blocks("dequant_gemv_q4_0q8", w, Q4_0_BYTES, blocksPerRow, xq, y, xq_blocks=True)


# ====================================== multi-column GEMM ===============

def _gemm(name, w, wScales, groupSize, xq, xScales, n, y, wdt):
    mode = _mode(w, wScales, xq, xScales, y)
    _check_dtype(w, wdt, "w"); _check_dtype(wScales, np.float32, "wScales")
    _check_dtype(xq, np.int8, "xq"); _check_dtype(xScales, np.float32, "xScales")
    _check_dtype(y, np.float32, "y")
    _call(mode, name, _ptr(w), _numel(w), _ptr(wScales), _numel(wScales), int(groupSize),
          _ptr(xq), _numel(xq), _ptr(xScales), _numel(xScales), int(n), _ptr(y), _numel(y))


def dequantGemmQ8(wq, wScales, groupSize, xq, xScales, n, y):
    """simd/dequant.nim:1382-1458: xq K x n column-major, y M x n row-major."""
    _gemm("dequant_gemm_q8", wq, wScales, groupSize, xq, xScales, n, y, np.int8)


def dequantGemmI4Q8(wpacked, wScales, groupSize, xq, xScales, n, y):
    """simd/dequant.nim:1460-1583."""
    _gemm("dequant_gemm_i4q8", wpacked, wScales, groupSize, xq, xScales, n, y, np.uint8)


# ====================================== encoders ========================

def quantizeQ8_0Batch(src, blocks):
    """simd/dequant.nim:1624-1641 (= quantizeQ8_0, ggml.nim:60-75)."""
    mode = _mode(src, blocks)
    _check_dtype(src, np.float32, "src")
    _call(mode, "quantize_q8_0_batch", _ptr(src), _numel(src), _ptr(blocks),
          _blocks(blocks, Q8_0_BYTES))


def quantizeQ4_0Batch(src, blocks):
    """simd/dequant.nim:1643-1715 (= quantizeQ4_0, ggml.nim:77-97)."""
    mode = _mode(src, blocks)
    _check_dtype(src, np.float32, "src")
    _call(mode, "quantize_q4_0_batch", _ptr(src), _numel(src), _ptr(blocks),
          _blocks(blocks, Q4_0_BYTES))


quantizeQ8_0 = quantizeQ8_0Batch
quantizeQ4_0 = quantizeQ4_0Batch


def quantizeBatch(x, scales, groupSize, dst, zeroPoint=None):
    """simd/dequant.nim:1717-1750 (and its scalar fall-through quant.nim:48-60):
    dst = toI8(x / scale[g] + zeroPoint[g]); ``zeroPoint`` None (or empty) is
    the symmetric case (+ 0.0), groupSize <= 0 per tensor (QParams.scheme =
    qPerTensor)."""
    mode = _mode(x, scales, dst, zeroPoint)
    _check_dtype(x, np.float32, "x"); _check_dtype(scales, np.float32, "scales")
    _check_dtype(dst, np.int8, "dst")
    if zeroPoint is not None:
        _check_dtype(zeroPoint, np.float32, "zeroPoint")
    _call(mode, "quantize_batch", _ptr(x), _numel(x), _ptr(scales), _numel(scales),
          _ptr(zeroPoint), _numel(zeroPoint), int(groupSize), _ptr(dst), _numel(dst))


def dequantizeBatch(q, scales, groupSize, dst, zeroPoint=None):
    """simd/dequant.nim:159-206 (and its scalar fall-through quant.nim:62-74):
    dst = (f32(q) - zeroPoint[g]) * scale[g] for I8 or I4 values held one per
    int8; ``zeroPoint`` None (or empty) is the symmetric case, groupSize <= 0
    per tensor."""
    mode = _mode(q, scales, dst, zeroPoint)
    _check_dtype(q, np.int8, "q"); _check_dtype(scales, np.float32, "scales")
    _check_dtype(dst, np.float32, "dst")
    if zeroPoint is not None:
        _check_dtype(zeroPoint, np.float32, "zeroPoint")
    _call(mode, "dequantize_batch", _ptr(q), _numel(q), _ptr(scales), _numel(scales),
          _ptr(zeroPoint), _numel(zeroPoint), int(groupSize), _ptr(dst), _numel(dst))


def _dev_only(name, *arrs):
    if _mode(*arrs) != "dev":
        raise TypeError(f"{name} takes torch CUDA tensors")


def quantizeQ8_0Split(src, qs, d):
    """quantizeQ8_0 (ggml.nim:60-75) with the block fields split into the
    (xq, xScales) arrays of dequantGemvQ8: d = f32(f16(amax/127))."""
    _dev_only("quantizeQ8_0Split", src, qs, d)
    N.check(N.lib().lp_quantize_q8_0_split(_ptr(src), _numel(src), _ptr(qs), _numel(qs),
                                           _ptr(d), _numel(d), _stream()), "quantize_q8_0_split")


def calibrateSymmetric(x, groupSize, qmax, scales):
    """quant.nim:95-110, writing the scales into `scales` (device)."""
    _dev_only("calibrateSymmetric", x, scales)
    N.check(N.lib().lp_calibrate_symmetric(_ptr(x), _numel(x), int(groupSize), float(qmax),
                                           _ptr(scales), _numel(scales), _stream()),
            "calibrate_symmetric")


def calibrateMX(x, blockSize, elemEmax, scales):
    """quant.nim:125-137, writing the E8M0-valued fp32 scales (device)."""
    _dev_only("calibrateMX", x, scales)
    N.check(N.lib().lp_calibrate_mx(_ptr(x), _numel(x), int(blockSize), int(elemEmax),
                                    _ptr(scales), _numel(scales), _stream()), "calibrate_mx")


def quantizeI4Packed(x, scales, groupSize, packed):
    """quantize[I4] (quant.nim:48-60) + packInt4 (intx.nim:83-94), device."""
    _dev_only("quantizeI4Packed", x, scales, packed)
    N.check(N.lib().lp_quantize_i4_packed(_ptr(x), _numel(x), _ptr(scales), _numel(scales),
                                          int(groupSize), _ptr(packed), _numel(packed),
                                          _stream()), "quantize_i4_packed")


def quantizeF4Packed(x, scales, blockSize, packed):
    """quantize[F4E2M1] (quant.nim:48-60) + packF4 (mxfloat.nim:138-149), device."""
    _dev_only("quantizeF4Packed", x, scales, packed)
    N.check(N.lib().lp_quantize_f4_packed(_ptr(x), _numel(x), _ptr(scales), _numel(scales),
                                          int(blockSize), _ptr(packed), _numel(packed),
                                          _stream()), "quantize_f4_packed")


def dequantizeQ8_0Batch(blocks, dst):
    """simd/dequant.nim:446-485 (= dequantizeQ8_0, ggml.nim:36-45), device."""
    _dev_only("dequantizeQ8_0Batch", blocks, dst)
    N.check(N.lib().lp_dequantize_q8_0_batch(_ptr(blocks), _blocks(blocks, Q8_0_BYTES),
                                             _ptr(dst), _numel(dst), _stream()),
            "dequantize_q8_0_batch")


def dequantizeQ4_0Batch(blocks, dst):
    """simd/dequant.nim:487-526 (= dequantizeQ4_0, ggml.nim:46-56), device."""
    _dev_only("dequantizeQ4_0Batch", blocks, dst)
    N.check(N.lib().lp_dequantize_q4_0_batch(_ptr(blocks), _blocks(blocks, Q4_0_BYTES),
                                             _ptr(dst), _numel(dst), _stream()),
            "dequantize_q4_0_batch")


def dequantizeQ4_K(blocks, dst):
    """dequantizeQ4_K (ggml.nim:136-161): 256-element super-blocks, device."""
    _dev_only("dequantizeQ4_K", blocks, dst)
    N.check(N.lib().lp_dequantize_q4_k(_ptr(blocks), _blocks(blocks, Q4_K_BYTES), _ptr(dst),
                                       _numel(dst), _stream()), "dequantize_q4_k")


def dequantizeQ6_K(blocks, dst):
    """dequantizeQ6_K (ggml.nim:163-213): 256-element super-blocks, device."""
    _dev_only("dequantizeQ6_K", blocks, dst)
    N.check(N.lib().lp_dequantize_q6_k(_ptr(blocks), _blocks(blocks, Q6_K_BYTES), _ptr(dst),
                                       _numel(dst), _stream()), "dequantize_q6_k")



def quantizeNVFP4(x, codes, blockScales, globalDecodeScale):
    """quantizeNVFP4 (nvfp4.nim:39-78), device: e2m1 codes (uint8 per element),
    e4m3 block scales (uint8 per 16 elements); the global decode scale the
    reference returns is written to the 1-element device tensor
    `globalDecodeScale`."""
    _dev_only("quantizeNVFP4", x, codes, blockScales, globalDecodeScale)
    N.check(N.lib().lp_quantize_nvfp4(_ptr(x), _numel(x), _ptr(codes), _numel(codes),
                                      _ptr(blockScales), _numel(blockScales),
                                      _ptr(globalDecodeScale), _stream()), "quantize_nvfp4")


def dequantizeNVFP4(codes, blockScales, globalDecodeScale, dst):
    """dequantizeNVFP4 (nvfp4.nim:80-92), device; globalDecodeScale is a float."""
    _dev_only("dequantizeNVFP4", codes, blockScales, dst)
    N.check(N.lib().lp_dequantize_nvfp4(_ptr(codes), _numel(codes), _ptr(blockScales),
                                        _numel(blockScales), float(globalDecodeScale),
                                        _ptr(dst), _numel(dst), _stream()), "dequantize_nvfp4")


def dequantGemmF4(wpacked, wScales, groupSize, xpacked, xScales, n, y):
    """MXFP4 x MXFP4 GEMM on the block-scaled tensor cores (tcgen05 kind::mxf4):
    the GEMM form of dequantGemvF4 (simd/dequant.nim:341-420) with MXFP4
    activations (K x n column-major packed codes, n x K/32 power-of-two fp32
    scales).  y is m x n row-major.  Torch CUDA tensors."""
    _dev_only("dequantGemmF4", wpacked, wScales, xpacked, xScales, y)
    N.check(N.lib().lp_dequant_gemm_f4(_ptr(wpacked), _numel(wpacked), _ptr(wScales),
                                       _numel(wScales), int(groupSize), _ptr(xpacked),
                                       _numel(xpacked), _ptr(xScales), _numel(xScales), int(n),
                                       _ptr(y), _numel(y), _stream()), "dequant_gemm_f4")


def gemmNVFP4(wpacked, wBlockScales, wGlobalDecodeScale, xpacked, xBlockScales,
              xGlobalDecodeScale, n, y):
    """NVFP4 x NVFP4 GEMM on the block-scaled tensor cores (tcgen05
    kind::mxf4nvf4): packed e2m1 codes, e4m3 block scales per 16 elements and
    the two global decode scales (one-element CUDA tensors, as quantizeNVFP4
    writes them); the decode of nvfp4.nim:80-92 on both operands."""
    _dev_only("gemmNVFP4", wpacked, wBlockScales, wGlobalDecodeScale, xpacked, xBlockScales,
              xGlobalDecodeScale, y)
    N.check(N.lib().lp_gemm_nvfp4(_ptr(wpacked), _numel(wpacked), _ptr(wBlockScales),
                                  _numel(wBlockScales), _ptr(wGlobalDecodeScale), _ptr(xpacked),
                                  _numel(xpacked), _ptr(xBlockScales), _numel(xBlockScales),
                                  _ptr(xGlobalDecodeScale), int(n), _ptr(y), _numel(y),
                                  _stream()), "gemm_nvfp4")


def dequantGemvQ4_K(w, superBlocksPerRow, x, y):
    """Fused GEMV over GGUF Q4_K super-blocks (144 bytes, ggml.nim:136-161
    values) with fp32 activations; block-float arithmetic.  Torch CUDA tensors."""
    _dev_only("dequantGemvQ4_K", w, x, y)
    N.check(N.lib().lp_dequant_gemv_q4_k(_ptr(w), _blocks(w, Q4_K_BYTES), int(superBlocksPerRow),
                                         _ptr(x), _numel(x), _ptr(y), _numel(y), _stream()),
            "dequant_gemv_q4_k")


def dequantGemvQ6_K(w, superBlocksPerRow, x, y):
    """Fused GEMV over GGUF Q6_K super-blocks (210 bytes, ggml.nim:163-213
    values) with fp32 activations; block-float arithmetic.  Torch CUDA tensors."""
    _dev_only("dequantGemvQ6_K", w, x, y)
    N.check(N.lib().lp_dequant_gemv_q6_k(_ptr(w), _blocks(w, Q6_K_BYTES), int(superBlocksPerRow),
                                         _ptr(x), _numel(x), _ptr(y), _numel(y), _stream()),
            "dequant_gemv_q6_k")
