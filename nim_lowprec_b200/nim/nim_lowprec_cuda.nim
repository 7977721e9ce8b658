## nim_lowprec_cuda -- drop-in replacements for nim-lowprec's fused
## dequant-GEMV/GEMM procs, running on a B200 through liblowprec_cuda.so.
##
## Same proc names, argument order and meaning as the reference's
## `simd/dequant` and `ggml` modules (src/nim_lowprec/simd/dequant.nim,
## ggml.nim); an `openArray[T]` crosses the C ABI as (pointer, length), which is
## exactly how the C ABI in include/lowprec_cuda.h takes it.  These forms take
## HOST arrays and block (the `lph_*` entry points): inputs are copied to the
## device, the kernel runs, `y` is copied back.  A failed shape precondition
## raises AssertionDefect, like the reference's `assert`.
##
## Status: written against the C ABI, not compiled here (no Nim toolchain in
## this build environment).  Usage mirrors the reference:
##
##   import nim_lowprec/[intx, ggml]
##   import nim_lowprec_cuda
##   dequantGemvQ8(wq, wScales, 32, xq, xScales, y)
##
## Types come from the reference modules (I8, BlockQ8_0, BlockQ4_0), which
## are layout-compatible with the C ABI (34 / 18-byte blocks).

import nim_lowprec/[intx, ggml, quant]

const lpLib* {.strdefine.} = "liblowprec_cuda.so"

type LowprecCudaError* = object of CatchableError

proc lph_dequant_gemv(wq: pointer, wqLen: int64, scales: pointer, scalesLen: int64,
    groupSize: int64, x: pointer, xLen: int64, y: pointer, yLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequant_gemv_i4(w: pointer, wLen: int64, scales: pointer, scalesLen: int64,
    groupSize: int64, x: pointer, xLen: int64, y: pointer, yLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequant_gemv_f4(w: pointer, wLen: int64, scales: pointer, scalesLen: int64,
    groupSize: int64, x: pointer, xLen: int64, y: pointer, yLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequant_gemv_q8_0(w: pointer, wLen: int64, bpr: int64, x: pointer, xLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_dequant_gemv_q4_0(w: pointer, wLen: int64, bpr: int64, x: pointer, xLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_dequant_gemv_q8(wq: pointer, wqLen: int64, ws: pointer, wsLen: int64, gs: int64,
    xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, y: pointer, yLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequant_gemv_i4q8(w: pointer, wLen: int64, ws: pointer, wsLen: int64, gs: int64,
    xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, y: pointer, yLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequant_gemv_q8_0q8(w: pointer, wLen: int64, bpr: int64, xq: pointer, xqLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_dequant_gemv_q4_0q8(w: pointer, wLen: int64, bpr: int64, xq: pointer, xqLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_dequant_gemm_q8(wq: pointer, wqLen: int64, ws: pointer, wsLen: int64, gs: int64,
    xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, n: int64, y: pointer,
    yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_dequant_gemm_i4q8(w: pointer, wLen: int64, ws: pointer, wsLen: int64, gs: int64,
    xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, n: int64, y: pointer,
    yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_quantize_q8_0_batch(src: pointer, srcLen: int64, blocks: pointer,
    blocksLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_quantize_q4_0_batch(src: pointer, srcLen: int64, blocks: pointer,
    blocksLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_quantize_batch(x: pointer, xLen: int64, scales: pointer, scalesLen: int64,
    zp: pointer, zpLen: int64, gs: int64, dst: pointer, dstLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lph_dequantize_batch(q: pointer, qLen: int64, scales: pointer, scalesLen: int64,
    zp: pointer, zpLen: int64, gs: int64, dst: pointer, dstLen: int64): cint {.
    importc, dynlib: lpLib.}
proc lp_status_string(status: cint): cstring {.importc, dynlib: lpLib.}

template base[T](a: openArray[T]): pointer =
  (if a.len > 0: cast[pointer](unsafeAddr a[0]) else: nil)

proc check(status: cint, where: string) =
  if status == 0: return
  if status == 1:  # LP_ERR_SHAPE: the reference's entry asserts
    raise newException(AssertionDefect, where & ": " & $lp_status_string(status))
  raise newException(LowprecCudaError, where & ": " & $lp_status_string(status))

# ---- fp32-activation fused GEMVs (simd/dequant.nim:210-622) ----

proc dequantGemv*(wq: openArray[I8], scales: openArray[float32], groupSize: int,
    x: openArray[float32], y: var openArray[float32]) =
  check(lph_dequant_gemv(base(wq), wq.len, base(scales), scales.len, groupSize,
      base(x), x.len, base(y), y.len), "dequantGemv")

proc dequantGemvI4*(wpacked: openArray[byte], scales: openArray[float32], groupSize: int,
    x: openArray[float32], y: var openArray[float32]) =
  check(lph_dequant_gemv_i4(base(wpacked), wpacked.len, base(scales), scales.len,
      groupSize, base(x), x.len, base(y), y.len), "dequantGemvI4")

proc dequantGemvF4*(wpacked: openArray[byte], scales: openArray[float32], groupSize: int,
    x: openArray[float32], y: var openArray[float32]) =
  check(lph_dequant_gemv_f4(base(wpacked), wpacked.len, base(scales), scales.len,
      groupSize, base(x), x.len, base(y), y.len), "dequantGemvF4")

proc dequantGemvQ8_0*(w: openArray[BlockQ8_0], blocksPerRow: int, x: openArray[float32],
    y: var openArray[float32]) =
  check(lph_dequant_gemv_q8_0(base(w), w.len, blocksPerRow, base(x), x.len, base(y),
      y.len), "dequantGemvQ8_0")

proc dequantGemvQ4_0*(w: openArray[BlockQ4_0], blocksPerRow: int, x: openArray[float32],
    y: var openArray[float32]) =
  check(lph_dequant_gemv_q4_0(base(w), w.len, blocksPerRow, base(x), x.len, base(y),
      y.len), "dequantGemvQ4_0")

# ---- int8-activation GEMVs (simd/dequant.nim:753-1365) ----

proc dequantGemvQ8*(wq: openArray[I8], wScales: openArray[float32], groupSize: int,
    xq: openArray[I8], xScales: openArray[float32], y: var openArray[float32]) =
  check(lph_dequant_gemv_q8(base(wq), wq.len, base(wScales), wScales.len, groupSize,
      base(xq), xq.len, base(xScales), xScales.len, base(y), y.len), "dequantGemvQ8")

proc dequantGemvI4Q8*(wpacked: openArray[byte], wScales: openArray[float32],
    groupSize: int, xq: openArray[I8], xScales: openArray[float32],
    y: var openArray[float32]) =
  check(lph_dequant_gemv_i4q8(base(wpacked), wpacked.len, base(wScales), wScales.len,
      groupSize, base(xq), xq.len, base(xScales), xScales.len, base(y), y.len),
      "dequantGemvI4Q8")

proc dequantGemvQ8_0Q8*(w: openArray[BlockQ8_0], blocksPerRow: int,
    xq: openArray[BlockQ8_0], y: var openArray[float32]) =
  check(lph_dequant_gemv_q8_0q8(base(w), w.len, blocksPerRow, base(xq), xq.len, base(y),
      y.len), "dequantGemvQ8_0Q8")

proc dequantGemvQ4_0Q8*(w: openArray[BlockQ4_0], blocksPerRow: int,
    xq: openArray[BlockQ8_0], y: var openArray[float32]) =
  check(lph_dequant_gemv_q4_0q8(base(w), w.len, blocksPerRow, base(xq), xq.len, base(y),
      y.len), "dequantGemvQ4_0Q8")

# ---- multi-column GEMM (simd/dequant.nim:1382-1583) ----

proc dequantGemmQ8*(wq: openArray[I8], wScales: openArray[float32], groupSize: int,
    xq: openArray[I8], xScales: openArray[float32], n: int, y: var openArray[float32]) =
  check(lph_dequant_gemm_q8(base(wq), wq.len, base(wScales), wScales.len, groupSize,
      base(xq), xq.len, base(xScales), xScales.len, n, base(y), y.len), "dequantGemmQ8")

proc dequantGemmI4Q8*(wpacked: openArray[byte], wScales: openArray[float32],
    groupSize: int, xq: openArray[I8], xScales: openArray[float32], n: int,
    y: var openArray[float32]) =
  check(lph_dequant_gemm_i4q8(base(wpacked), wpacked.len, base(wScales), wScales.len,
      groupSize, base(xq), xq.len, base(xScales), xScales.len, n, base(y), y.len),
      "dequantGemmI4Q8")

# ---- encoders (simd/dequant.nim:1624-1715) ----

proc quantizeQ8_0Batch*(src: openArray[float32], blocks: var openArray[BlockQ8_0]) =
  check(lph_quantize_q8_0_batch(base(src), src.len, base(blocks), blocks.len),
      "quantizeQ8_0Batch")

proc quantizeQ4_0Batch*(src: openArray[float32], blocks: var openArray[BlockQ4_0]) =
  check(lph_quantize_q4_0_batch(base(src), src.len, base(blocks), blocks.len),
      "quantizeQ4_0Batch")

# ---- elementwise codecs over QParams (simd/dequant.nim:159-206, 1717-1750) ----

proc groupOf(p: QParams): int64 =
  ## QParams' group size as the C ABI takes it: 0 for a per-tensor scale.
  if p.scheme == qPerTensor: 0'i64 else: p.groupSize.int64

proc quantizeBatch*(x: openArray[float32], p: QParams, dst: var openArray[I8]) =
  ## toI8(x / scale + zeroPoint) per group: the reference's vector form for
  ## symmetric QParams and its scalar `quantize` fall-through for QParams with
  ## zero points, both in one kernel.
  check(lph_quantize_batch(base(x), x.len, base(p.scale), p.scale.len,
      base(p.zeroPoint), p.zeroPoint.len, groupOf(p), base(dst), dst.len),
      "quantizeBatch")

template defDequantizeBatch(T: untyped) =
  proc dequantizeBatch*(q: openArray[T], p: QParams, dst: var openArray[float32]) =
    ## (f32(q) - zeroPoint) * scale per group; symmetric and affine QParams.
    check(lph_dequantize_batch(base(q), q.len, base(p.scale), p.scale.len,
        base(p.zeroPoint), p.zeroPoint.len, groupOf(p), base(dst), dst.len),
        "dequantizeBatch")

defDequantizeBatch(I8)
defDequantizeBatch(I4)

# ---- LpPool over this box's GPUs (parallel.nim:82-474) ----
#
# The reference's pool is one process with a worker per core; this one has a
# worker per GPU.  Same procs and meaning: initPool(threads) (threads <= 0:
# every GPU), shutdown (idempotent), threadCount (0 after shutdown), the
# pooled int8-activation GEMV / GEMM forms, and the per-call par* forms with
# a `threads` count.  Results equal the serial calls bit for bit.

type LpPool* = object
  h: pointer

proc lph_pool_init(pool: ptr pointer, threads: cint): cint {.importc, dynlib: lpLib.}
proc lph_pool_shutdown(pool: ptr pointer): cint {.importc, dynlib: lpLib.}
proc lph_pool_thread_count(pool: pointer): cint {.importc, dynlib: lpLib.}
proc lph_pool_dequant_gemv_q8(pool: pointer, wq: pointer, wqLen: int64, ws: pointer,
    wsLen: int64, gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_pool_dequant_gemv_i4q8(pool: pointer, w: pointer, wLen: int64, ws: pointer,
    wsLen: int64, gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_pool_dequant_gemm_q8(pool: pointer, wq: pointer, wqLen: int64, ws: pointer,
    wsLen: int64, gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, n: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_pool_dequant_gemm_i4q8(pool: pointer, w: pointer, wLen: int64, ws: pointer,
    wsLen: int64, gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, n: int64,
    y: pointer, yLen: int64): cint {.importc, dynlib: lpLib.}
proc lph_par_dequant_gemv(wq: pointer, wqLen: int64, scales: pointer, scalesLen: int64,
    gs: int64, x: pointer, xLen: int64, y: pointer, yLen: int64, threads: cint): cint {.
    importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_i4(w: pointer, wLen: int64, scales: pointer, scalesLen: int64,
    gs: int64, x: pointer, xLen: int64, y: pointer, yLen: int64, threads: cint): cint {.
    importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_f4(w: pointer, wLen: int64, scales: pointer, scalesLen: int64,
    gs: int64, x: pointer, xLen: int64, y: pointer, yLen: int64, threads: cint): cint {.
    importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_q8_0(w: pointer, wLen: int64, bpr: int64, x: pointer,
    xLen: int64, y: pointer, yLen: int64, threads: cint): cint {.importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_q4_0(w: pointer, wLen: int64, bpr: int64, x: pointer,
    xLen: int64, y: pointer, yLen: int64, threads: cint): cint {.importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_q8(wq: pointer, wqLen: int64, ws: pointer, wsLen: int64,
    gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, y: pointer,
    yLen: int64, threads: cint): cint {.importc, dynlib: lpLib.}
proc lph_par_dequant_gemv_i4q8(w: pointer, wLen: int64, ws: pointer, wsLen: int64,
    gs: int64, xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, y: pointer,
    yLen: int64, threads: cint): cint {.importc, dynlib: lpLib.}

proc initPool*(threads = 0): LpPool =
  ## Workers = `threads` GPUs (default: every visible GPU).  Call `shutdown`.
  check(lph_pool_init(addr result.h, threads.cint), "initPool")

proc shutdown*(p: var LpPool) =
  ## Stop the workers and free the pool.  Idempotent.
  check(lph_pool_shutdown(addr p.h), "shutdown")

proc threadCount*(p: LpPool): int =
  ## Workers in this pool, 0 if it was never initialized or is shut down.
  lph_pool_thread_count(p.h).int

proc parDequantGemvQ8*(pool: var LpPool, wq: openArray[I8], wScales: openArray[float32],
    groupSize: int, xq: openArray[I8], xScales: openArray[float32],
    y: var openArray[float32]) =
  check(lph_pool_dequant_gemv_q8(pool.h, base(wq), wq.len, base(wScales), wScales.len,
      groupSize, base(xq), xq.len, base(xScales), xScales.len, base(y), y.len),
      "parDequantGemvQ8")

proc parDequantGemvI4Q8*(pool: var LpPool, wpacked: openArray[byte],
    wScales: openArray[float32], groupSize: int, xq: openArray[I8],
    xScales: openArray[float32], y: var openArray[float32]) =
  check(lph_pool_dequant_gemv_i4q8(pool.h, base(wpacked), wpacked.len, base(wScales),
      wScales.len, groupSize, base(xq), xq.len, base(xScales), xScales.len, base(y), y.len),
      "parDequantGemvI4Q8")

proc parDequantGemmQ8*(pool: var LpPool, wq: openArray[I8], wScales: openArray[float32],
    groupSize: int, xq: openArray[I8], xScales: openArray[float32], n: int,
    y: var openArray[float32]) =
  check(lph_pool_dequant_gemm_q8(pool.h, base(wq), wq.len, base(wScales), wScales.len,
      groupSize, base(xq), xq.len, base(xScales), xScales.len, n, base(y), y.len),
      "parDequantGemmQ8")

proc parDequantGemmI4Q8*(pool: var LpPool, wpacked: openArray[byte],
    wScales: openArray[float32], groupSize: int, xq: openArray[I8],
    xScales: openArray[float32], n: int, y: var openArray[float32]) =
  check(lph_pool_dequant_gemm_i4q8(pool.h, base(wpacked), wpacked.len, base(wScales),
      wScales.len, groupSize, base(xq), xq.len, base(xScales), xScales.len, n, base(y),
      y.len), "parDequantGemmI4Q8")

proc parDequantGemv*(wq: openArray[I8], scales: openArray[float32], groupSize: int,
    x: openArray[float32], y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv(base(wq), wq.len, base(scales), scales.len, groupSize,
      base(x), x.len, base(y), y.len, threads.cint), "parDequantGemv")

proc parDequantGemvI4*(wpacked: openArray[byte], scales: openArray[float32],
    groupSize: int, x: openArray[float32], y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv_i4(base(wpacked), wpacked.len, base(scales), scales.len,
      groupSize, base(x), x.len, base(y), y.len, threads.cint), "parDequantGemvI4")

proc parDequantGemvF4*(wpacked: openArray[byte], scales: openArray[float32],
    groupSize: int, x: openArray[float32], y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv_f4(base(wpacked), wpacked.len, base(scales), scales.len,
      groupSize, base(x), x.len, base(y), y.len, threads.cint), "parDequantGemvF4")

proc parDequantGemvQ8_0*(w: openArray[BlockQ8_0], blocksPerRow: int,
    x: openArray[float32], y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv_q8_0(base(w), w.len, blocksPerRow, base(x), x.len, base(y),
      y.len, threads.cint), "parDequantGemvQ8_0")

proc parDequantGemvQ4_0*(w: openArray[BlockQ4_0], blocksPerRow: int,
    x: openArray[float32], y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv_q4_0(base(w), w.len, blocksPerRow, base(x), x.len, base(y),
      y.len, threads.cint), "parDequantGemvQ4_0")

proc parDequantGemvQ8*(wq: openArray[I8], wScales: openArray[float32], groupSize: int,
    xq: openArray[I8], xScales: openArray[float32], y: var openArray[float32],
    threads = 0) =
  check(lph_par_dequant_gemv_q8(base(wq), wq.len, base(wScales), wScales.len, groupSize,
      base(xq), xq.len, base(xScales), xScales.len, base(y), y.len, threads.cint),
      "parDequantGemvQ8")

proc parDequantGemvI4Q8*(wpacked: openArray[byte], wScales: openArray[float32],
    groupSize: int, xq: openArray[I8], xScales: openArray[float32],
    y: var openArray[float32], threads = 0) =
  check(lph_par_dequant_gemv_i4q8(base(wpacked), wpacked.len, base(wScales), wScales.len,
      groupSize, base(xq), xq.len, base(xScales), xScales.len, base(y), y.len,
      threads.cint), "parDequantGemvI4Q8")

# ---------------------------------------------------- device forms, batched
# A decode loop whose weights stay on the GPU calls the device forms (device
# pointers, a CUDA stream) and may bracket a step's GEMVs in one batch: the
# queued calls run as one persistent launch, each with its own bits
# (lp_batch_begin / lp_batch_end; no counterpart in the reference).

proc lp_batch_begin(stream: pointer): cint {.importc, dynlib: lpLib.}
proc lp_batch_end(stream: pointer): cint {.importc, dynlib: lpLib.}
proc lp_quantize_dequant_gemv_i4q8(w: pointer, wLen: int64, ws: pointer, wsLen: int64,
    gs: int64, x: pointer, xLen: int64, y: pointer, yLen: int64,
    stream: pointer): cint {.importc, dynlib: lpLib.}
proc lp_dequant_gemv_i4q8(w: pointer, wLen: int64, ws: pointer, wsLen: int64, gs: int64,
    xq: pointer, xqLen: int64, xs: pointer, xsLen: int64, y: pointer, yLen: int64,
    stream: pointer): cint {.importc, dynlib: lpLib.}

template withBatch*(stream: pointer, body: untyped) =
  ## The GEMVs `body` issues on `stream` run as batched launches.
  check(lp_batch_begin(stream), "batchBegin")
  body
  check(lp_batch_end(stream), "batchEnd")

proc quantizeDequantGemvI4Q8Dev*(w: pointer, wLen: int, ws: pointer, wsLen: int,
    x: pointer, xLen: int, y: pointer, yLen: int, stream: pointer) =
  ## quantizeQ8_0 of device fp32 x, then dequantGemvI4Q8 (group 32), on `stream`.
  check(lp_quantize_dequant_gemv_i4q8(w, wLen, ws, wsLen, 32, x, xLen, y, yLen, stream),
      "quantizeDequantGemvI4Q8")

proc dequantGemvI4Q8Dev*(w: pointer, wLen: int, ws: pointer, wsLen: int, groupSize: int,
    xq: pointer, xqLen: int, xs: pointer, xsLen: int, y: pointer, yLen: int,
    stream: pointer) =
  check(lp_dequant_gemv_i4q8(w, wLen, ws, wsLen, groupSize, xq, xqLen, xs, xsLen, y, yLen,
      stream), "dequantGemvI4Q8")
