"""CPU oracle for nim-lowprec's dequant-GEMV/GEMM hot path -- TEST INFRASTRUCTURE.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product library (``nim_lowprec_b200``) never loads it and has no
CPU fallback.

It wraps ``lowprec_oracle.c`` (a C restatement of the reference's scalar
branches; every function there cites the reference file:line it follows) with
numpy-facing helpers whose argument order follows the reference's Nim procs.

Parity status: pinned.  The encoders are checked bit-for-bit against gguf-py
and ml_dtypes goldens produced by the reference's own ``tests/gen_reference.py``
(fixtures under ``tests/golden/``), and the kernels against the reference
tests' own exact references (``tests/test_sdot.nim`` intRef/refQ8/refQ4,
restated in numpy in ``tests/test_oracle_kernels.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "lowprec_oracle.c")
LIB = os.path.join(HERE, "liblporacle.so")

QK = 32
Q8_0_BYTES = 34
Q4_0_BYTES = 18

CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread"]


def build(force: bool = False) -> str:
    """Compile the C restatement into ``oracle/liblporacle.so`` (gcc)."""
    stale = (not os.path.exists(LIB)) or os.path.getmtime(LIB) < os.path.getmtime(SRC)
    if force or stale:
        cmd = ["gcc", *CFLAGS, "-o", LIB, SRC, "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        i64, vp, f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
        L.lpo_f32_to_f16.restype = ctypes.c_uint16
        L.lpo_f32_to_f16.argtypes = [f32]
        L.lpo_f16_to_f32.restype = f32
        L.lpo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.lpo_to_f4e2m1.restype = ctypes.c_uint8
        L.lpo_to_f4e2m1.argtypes = [f32]
        L.lpo_f4e2m1_to_f32.restype = f32
        L.lpo_f4e2m1_to_f32.argtypes = [ctypes.c_uint8]
        L.lpo_to_e8m0.restype = ctypes.c_uint8
        L.lpo_to_e8m0.argtypes = [f32]
        L.lpo_e8m0_to_f32.restype = f32
        L.lpo_e8m0_to_f32.argtypes = [ctypes.c_uint8]
        L.lpo_calibrate_symmetric.restype = i64
        L.lpo_calibrate_symmetric.argtypes = [vp, i64, i64, f32, vp]
        L.lpo_calibrate_mx.restype = i64
        L.lpo_calibrate_mx.argtypes = [vp, i64, i64, ctypes.c_int, vp]
        L.lpo_quantize.argtypes = [vp, i64, vp, i64, ctypes.c_int, vp]
        L.lpo_quantize_batch.argtypes = [vp, i64, vp, vp, i64, vp]
        L.lpo_dequantize_batch.argtypes = [vp, i64, vp, vp, i64, vp]
        L.lpo_pack_int4.argtypes = [vp, i64, vp]
        L.lpo_pack_f4.argtypes = [vp, i64, vp]
        for nm in ("lpo_quantize_q8_0", "lpo_quantize_q4_0"):
            getattr(L, nm).argtypes = [vp, i64, vp]
        L.lpo_quantize_q8_0_split.argtypes = [vp, i64, vp, vp]
        for nm in ("lpo_dequantize_q8_0", "lpo_dequantize_q4_0", "lpo_dequantize_q4_k",
                   "lpo_dequantize_q6_k"):
            getattr(L, nm).argtypes = [vp, i64, vp]
        L.lpo_to_f8e4m3.restype = ctypes.c_uint8
        L.lpo_to_f8e4m3.argtypes = [f32]
        L.lpo_f8e4m3_to_f32.restype = f32
        L.lpo_f8e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.lpo_quantize_nvfp4.restype = f32
        L.lpo_quantize_nvfp4.argtypes = [vp, i64, vp, vp]
        L.lpo_dequantize_nvfp4.argtypes = [vp, vp, f32, i64, vp]
        L.lpo_pool_init.restype = vp
        L.lpo_pool_init.argtypes = [ctypes.c_int]
        L.lpo_pool_shutdown.argtypes = [vp]
        L.lpo_pool_thread_count.restype = ctypes.c_int
        L.lpo_pool_thread_count.argtypes = [vp]
        L.lpo_shard_count.restype = ctypes.c_int
        L.lpo_shard_count.argtypes = [i64, ctypes.c_int]
        L.lpo_shard.restype = None
        L.lpo_shard.argtypes = [i64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        L.lpo_run.argtypes = [vp, ctypes.c_int, vp, vp, i64, vp, vp, i64, i64, vp, i64]
        L.lpo_gemm_fp4.argtypes = [vp, vp, vp, vp, ctypes.c_int, i64, i64, i64, ctypes.c_double, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------ codecs --

def f32_to_f16(x: float) -> int:
    return int(lib().lpo_f32_to_f16(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().lpo_f16_to_f32(int(h)))


def to_f4e2m1(x: float) -> int:
    return int(lib().lpo_to_f4e2m1(float(x)))


def to_e8m0(x: float) -> int:
    return int(lib().lpo_to_e8m0(float(x)))


def e8m0_to_f32(c: int) -> float:
    return float(lib().lpo_e8m0_to_f32(int(c)))


# ---------------------------------------------------------- encoders --

def calibrateSymmetric(x, groupSize: int, qmax: float) -> np.ndarray:
    x = _c(x, np.float32)
    n = x.size
    gs = groupSize if groupSize > 0 else max(n, 1)
    out = np.empty((n + gs - 1) // gs, np.float32)
    lib().lpo_calibrate_symmetric(_p(x), n, groupSize, float(qmax), _p(out))
    return out


def calibrateMX(x, blockSize: int, elemEmax: int) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty((x.size + blockSize - 1) // blockSize, np.float32)
    lib().lpo_calibrate_mx(_p(x), x.size, blockSize, int(elemEmax), _p(out))
    return out


def quantize(x, scales, groupSize: int, kind: str) -> np.ndarray:
    """quantize[T] for symmetric QParams; kind in {'i8', 'i4', 'f4'}.
    'i4' returns one signed value per int8, 'f4' one e2m1 code per uint8."""
    x = _c(x, np.float32)
    scales = _c(scales, np.float32)
    out = np.empty(x.size, np.int8)
    lib().lpo_quantize(_p(x), x.size, _p(scales), groupSize, {"i8": 0, "i4": 1, "f4": 2}[kind], _p(out))
    return out.view(np.uint8) if kind == "f4" else out


def quantizeBatch(x, scales, groupSize: int, zeroPoint=None) -> np.ndarray:
    """toI8(x / scale[g] + zeroPoint[g]) (simd/dequant.nim:1717-1750 =
    quant.nim:48-60); ``zeroPoint`` None is symmetric (+ 0.0)."""
    x = _c(x, np.float32)
    scales = _c(scales, np.float32)
    zp = None if zeroPoint is None or np.size(zeroPoint) == 0 else _c(zeroPoint, np.float32)
    out = np.empty(x.size, np.int8)
    lib().lpo_quantize_batch(_p(x), x.size, _p(scales), _p(zp) if zp is not None else None,
                             groupSize, _p(out))
    return out


def dequantizeBatch(q, scales, groupSize: int, zeroPoint=None) -> np.ndarray:
    """(f32(q) - zeroPoint[g]) * scale[g] for int8-backed I8 / I4 values
    (simd/dequant.nim:159-206 = quant.nim:62-74); ``groupSize <= 0`` is per
    tensor, ``zeroPoint`` None is symmetric."""
    q = _c(q, np.int8)
    scales = _c(scales, np.float32)
    zp = None if zeroPoint is None else _c(zeroPoint, np.float32)
    out = np.empty(q.size, np.float32)
    lib().lpo_dequantize_batch(_p(q), q.size, _p(scales), None if zp is None else _p(zp),
                               groupSize, _p(out))
    return out


def packInt4(vals) -> np.ndarray:
    vals = _c(vals, np.int8)
    out = np.zeros((vals.size + 1) // 2, np.uint8)
    lib().lpo_pack_int4(_p(vals), vals.size, _p(out))
    return out


def packF4(codes) -> np.ndarray:
    codes = _c(codes, np.uint8)
    out = np.zeros((codes.size + 1) // 2, np.uint8)
    lib().lpo_pack_f4(_p(codes), codes.size, _p(out))
    return out


def quantizeQ8_0(src) -> np.ndarray:
    """Returns raw blocks, shape (n/32, 34) uint8."""
    src = _c(src, np.float32)
    assert src.size % QK == 0
    out = np.empty((src.size // QK, Q8_0_BYTES), np.uint8)
    lib().lpo_quantize_q8_0(_p(src), src.size, _p(out))
    return out


def quantizeQ8_0Split(src):
    """quantizeQ8_0 split into (qs int8[n], d float32[n/32]) with d = f32(f16 d)."""
    src = _c(src, np.float32)
    assert src.size % QK == 0
    qs = np.empty(src.size, np.int8)
    d = np.empty(src.size // QK, np.float32)
    lib().lpo_quantize_q8_0_split(_p(src), src.size, _p(qs), _p(d))
    return qs, d


def quantizeQ4_0(src) -> np.ndarray:
    src = _c(src, np.float32)
    assert src.size % QK == 0
    out = np.empty((src.size // QK, Q4_0_BYTES), np.uint8)
    lib().lpo_quantize_q4_0(_p(src), src.size, _p(out))
    return out


def dequantizeQ8_0(blocks) -> np.ndarray:
    blocks = _c(blocks, np.uint8).reshape(-1, Q8_0_BYTES)
    out = np.empty(blocks.shape[0] * QK, np.float32)
    lib().lpo_dequantize_q8_0(_p(blocks), blocks.shape[0], _p(out))
    return out


def dequantizeQ4_0(blocks) -> np.ndarray:
    blocks = _c(blocks, np.uint8).reshape(-1, Q4_0_BYTES)
    out = np.empty(blocks.shape[0] * QK, np.float32)
    lib().lpo_dequantize_q4_0(_p(blocks), blocks.shape[0], _p(out))
    return out


QK_K = 256
Q4_K_BYTES, Q6_K_BYTES = 144, 210


def dequantizeQ4_K(blocks) -> np.ndarray:
    """dequantizeQ4_K (ggml.nim:136-161)."""
    blocks = _c(blocks, np.uint8).reshape(-1, Q4_K_BYTES)
    out = np.empty(blocks.shape[0] * QK_K, np.float32)
    lib().lpo_dequantize_q4_k(_p(blocks), blocks.shape[0], _p(out))
    return out


def dequantizeQ6_K(blocks) -> np.ndarray:
    """dequantizeQ6_K (ggml.nim:163-213)."""
    blocks = _c(blocks, np.uint8).reshape(-1, Q6_K_BYTES)
    out = np.empty(blocks.shape[0] * QK_K, np.float32)
    lib().lpo_dequantize_q6_k(_p(blocks), blocks.shape[0], _p(out))
    return out


NVFP4_BLOCK = 16


def quantizeNVFP4(x):
    """quantizeNVFP4 (nvfp4.nim:39-78): (codes u8 per element, e4m3 block
    scales u8 per 16 elements, global decode scale)."""
    x = _c(x, np.float32).reshape(-1)
    assert x.size % NVFP4_BLOCK == 0
    codes = np.empty(x.size, np.uint8)
    scales = np.empty(x.size // NVFP4_BLOCK, np.uint8)
    gds = lib().lpo_quantize_nvfp4(_p(x), x.size, _p(codes), _p(scales))
    return codes, scales, np.float32(gds)


def dequantizeNVFP4(codes, scales, gds) -> np.ndarray:
    """dequantizeNVFP4 (nvfp4.nim:80-92)."""
    codes = _c(codes, np.uint8).reshape(-1)
    scales = _c(scales, np.uint8).reshape(-1)
    out = np.empty(codes.size, np.float32)
    lib().lpo_dequantize_nvfp4(_p(codes), _p(scales), float(gds), codes.size, _p(out))
    return out


# ----------------------------------------------------------- kernels --

KIND = {"i8": 0, "i4": 1, "f4": 2, "q8_0": 3, "q4_0": 4, "q8": 5, "i4q8": 6,
        "q8_0q8": 7, "q4_0q8": 8, "gemm_q8": 9, "gemm_i4q8": 10}


class Pool:
    """LpPool restatement (pthreads): initPool / threadCount / shutdown."""

    def __init__(self, threads: int = 0):
        self._h = lib().lpo_pool_init(int(threads))

    @property
    def handle(self):
        return self._h

    def threadCount(self) -> int:
        return int(lib().lpo_pool_thread_count(self._h)) if self._h else 0

    def shutdown(self) -> None:
        if self._h:
            lib().lpo_pool_shutdown(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.shutdown()
        except Exception:
            pass


def _run(kind, w, ws, gs, x, xs, k, n, rows, pool=None) -> np.ndarray:
    y = np.empty(rows * max(n, 1), np.float32)
    keep = [w, ws, x, xs]
    ptr = [(_p(a) if a is not None else None) for a in keep]
    lib().lpo_run(pool.handle if pool is not None else None, KIND[kind], ptr[0], ptr[1], int(gs),
                  ptr[2], ptr[3], int(k), int(n), _p(y), int(rows))
    return y


def dequantGemv(wq, scales, groupSize, x, pool=None):
    x = _c(x, np.float32); wq = _c(wq, np.int8); scales = _c(scales, np.float32)
    return _run("i8", wq, scales, groupSize, x, None, x.size, 1, wq.size // x.size, pool)


def dequantGemvI4(wpacked, scales, groupSize, x, pool=None):
    x = _c(x, np.float32); wp = _c(wpacked, np.uint8); scales = _c(scales, np.float32)
    return _run("i4", wp, scales, groupSize, x, None, x.size, 1, wp.size // (x.size // 2), pool)


def dequantGemvF4(wpacked, scales, groupSize, x, pool=None):
    x = _c(x, np.float32); wp = _c(wpacked, np.uint8); scales = _c(scales, np.float32)
    return _run("f4", wp, scales, groupSize, x, None, x.size, 1, wp.size // (x.size // 2), pool)


def dequantGemvQ8_0(w, blocksPerRow, x, pool=None):
    x = _c(x, np.float32); w = _c(w, np.uint8).reshape(-1)
    rows = w.size // (blocksPerRow * Q8_0_BYTES)
    return _run("q8_0", w, None, blocksPerRow, x, None, x.size, 1, rows, pool)


def dequantGemvQ4_0(w, blocksPerRow, x, pool=None):
    x = _c(x, np.float32); w = _c(w, np.uint8).reshape(-1)
    rows = w.size // (blocksPerRow * Q4_0_BYTES)
    return _run("q4_0", w, None, blocksPerRow, x, None, x.size, 1, rows, pool)


def dequantGemvQ8(wq, wScales, groupSize, xq, xScales, pool=None):
    wq = _c(wq, np.int8); ws = _c(wScales, np.float32); xq = _c(xq, np.int8); xs = _c(xScales, np.float32)
    return _run("q8", wq, ws, groupSize, xq, xs, xq.size, 1, wq.size // xq.size, pool)


def dequantGemvI4Q8(wpacked, wScales, groupSize, xq, xScales, pool=None):
    wp = _c(wpacked, np.uint8); ws = _c(wScales, np.float32); xq = _c(xq, np.int8); xs = _c(xScales, np.float32)
    return _run("i4q8", wp, ws, groupSize, xq, xs, xq.size, 1, wp.size // (xq.size // 2), pool)


def dequantGemvQ8_0Q8(w, blocksPerRow, xq, pool=None):
    w = _c(w, np.uint8).reshape(-1); xq = _c(xq, np.uint8).reshape(-1)
    rows = w.size // (blocksPerRow * Q8_0_BYTES)
    return _run("q8_0q8", w, None, blocksPerRow, xq, None, blocksPerRow * QK, 1, rows, pool)


def dequantGemvQ4_0Q8(w, blocksPerRow, xq, pool=None):
    w = _c(w, np.uint8).reshape(-1); xq = _c(xq, np.uint8).reshape(-1)
    rows = w.size // (blocksPerRow * Q4_0_BYTES)
    return _run("q4_0q8", w, None, blocksPerRow, xq, None, blocksPerRow * QK, 1, rows, pool)


def dequantGemmQ8(wq, wScales, groupSize, xq, xScales, n, pool=None):
    wq = _c(wq, np.int8); ws = _c(wScales, np.float32); xq = _c(xq, np.int8); xs = _c(xScales, np.float32)
    k = xq.size // n
    return _run("gemm_q8", wq, ws, groupSize, xq, xs, k, n, wq.size // k, pool)


def dequantGemmI4Q8(wpacked, wScales, groupSize, xq, xScales, n, pool=None):
    wp = _c(wpacked, np.uint8); ws = _c(wScales, np.float32); xq = _c(xq, np.int8); xs = _c(xScales, np.float32)
    k = xq.size // n
    return _run("gemm_i4q8", wp, ws, groupSize, xq, xs, k, n, wp.size // (k // 2), pool)


def shard(rows: int, workers: int, worker: int):
    """(first row, row count) of a worker's slice (parallel.nim:118-124)."""
    r0, cnt = ctypes.c_int64(), ctypes.c_int64()
    lib().lpo_shard(int(rows), int(workers), int(worker), ctypes.addressof(r0), ctypes.addressof(cnt))
    return r0.value, cnt.value


def shardCount(rows: int, threads: int) -> int:
    return int(lib().lpo_shard_count(int(rows), int(threads)))


def gemmFp4(wpacked, wScales, xpacked, xScales, n: int, nvfp4: bool = False,
            globalScale: float = 1.0) -> np.ndarray:
    """FP4 x FP4 GEMM in fp64 (lpo_gemm_fp4): MXFP4 (fp32 power-of-two scales
    per 32 elements) or NVFP4 (e4m3 byte scales per 16 elements times the
    product of the global decode scales).  Returns y (m x n row-major, fp64)."""
    wpacked = _c(wpacked, np.uint8)
    xpacked = _c(xpacked, np.uint8)
    dt = np.uint8 if nvfp4 else np.float32
    ws = _c(wScales, dt)
    xs = _c(xScales, dt)
    k = xpacked.size * 2 // n
    m = wpacked.size * 2 // k
    y = np.empty(m * n, np.float64)
    lib().lpo_gemm_fp4(_p(wpacked), _p(ws), _p(xpacked), _p(xs), 1 if nvfp4 else 0, m, k, n,
                       float(globalScale), _p(y))
    return y
