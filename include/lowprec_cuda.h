/*
 * lowprec_cuda.h -- C ABI of the B200 (sm_100a) implementation of
 * nim-lowprec's fused dequant-GEMV/GEMM hot path (liblowprec_cuda.so).
 *
 * Each entry point replaces one Nim proc of the reference and keeps its
 * argument order.  Nim's C backend passes an `openArray[T]` as a (T*, length)
 * pair, so every array argument here is a pointer followed by its element
 * count, and shapes are derived from those lengths exactly as the reference
 * derives them (m = y.len, k = x.len, gpr = k div groupSize, ...).
 *
 * Two forms per kernel:
 *   lp_*   DEVICE pointers + a CUDA stream; asynchronous, stream-ordered,
 *          allocates nothing (but see lp_batch_begin), reentrant across
 *          streams.  Activations and outputs may also be page-locked host
 *          memory, passed by the address lp_host_device_pointer gives.
 *   lph_*  HOST pointers, blocking: the literal drop-in for the Nim
 *          signature.  Stages through a cached per-thread device workspace,
 *          copies every input host->device, runs, copies the output back.
 *
 * Preconditions the reference asserts (e.g. simd/dequant.nim:768-771) return
 * LP_ERR_SHAPE here instead of raising; nothing is launched in that case.
 * Block formats are byte-compatible with the reference's packed objects:
 *   BlockQ8_0 = { uint16 d (fp16 bits); int8 qs[32] }   34 bytes (ggml.nim:26-28)
 *   BlockQ4_0 = { uint16 d (fp16 bits); uint8 qs[16] }  18 bytes (ggml.nim:30-32)
 * so a `w_len`/`xq_len` of a block array counts BLOCKS, not bytes.
 */
#ifndef LOWPREC_CUDA_H
#define LOWPREC_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status -- */
#define LP_OK 0
#define LP_ERR_SHAPE 1       /* a length precondition of the reference failed */
#define LP_ERR_ARG 2         /* null pointer, negative length, bad option */
#define LP_ERR_CUDA 3        /* a CUDA runtime call failed */
#define LP_ERR_NCCL 4        /* a collective failed */
#define LP_ERR_TIMEOUT 5     /* a bounded device-side wait ran out */
#define LP_ERR_UNSUPPORTED 6 /* shape outside what this build implements */
#define LP_ERR_NO_DEVICE 7   /* no usable CUDA device */

#define LP_QK 32
#define LP_BLOCK_Q8_0_BYTES 34
#define LP_BLOCK_Q4_0_BYTES 18

typedef void *lp_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

/* Library utilities (no counterpart in the reference, whose procs assert
 * and return nothing). */

/* Library version, e.g. 100 for 0.1.0. */
int lp_version(void);

/* Message for a status code (static string). */
const char *lp_status_string(int status);

/* Text of the last CUDA error this thread's calls hit ("" if none). */
const char *lp_last_error_detail(void);

/* Synchronise the current device, then return (and clear) the first error a
 * kernel of this library recorded on it (LP_OK if none).  Device-side
 * failures never trap; they are reported here. */
int lp_device_error(void);

/* Device address of page-locked host memory (no counterpart in the reference).
 * The device forms take any device-accessible pointer; a page-locked host
 * buffer (cudaHostAlloc / cudaMallocHost / cudaHostRegister, or a pinned
 * torch tensor) passed by this address is read and written by the kernels
 * themselves over the host link, with no copy.  LP_ERR_ARG for memory that
 * is not page-locked or not mapped. */
int lp_host_device_pointer(const void *host, void **dev);

/* Copy `bytes` from page-locked host memory (src: its lp_host_device_pointer
 * address) into device memory as a kernel of `stream` (no counterpart in the
 * reference).  For per-step inputs of a decode loop: the source is read
 * while the previous kernel in the stream finishes, dst is written after it
 * has, and a following GEMV starts streaming its weights at once.  src must
 * not be written by the kernel before it in the stream. */
int lp_copy_in(void *dst, const void *src, int64_t bytes, lp_stream_t stream);

/* Batched GEMV launches (no counterpart in the reference; the reference
 * runs each call on the CPU as it comes).  Device-form GEMVs with one output
 * per weight row -- every format: the fp32-activation ones (lp_dequant_gemv,
 * _i4, _f4, _q8_0, _q4_0, _q4_k, _q6_k) in either fp32 mode, the
 * int8-activation ones (lp_dequant_gemv_q8 / _i4q8, the fused
 * lp_quantize_dequant_gemv_q8 / _i4q8, lp_dequant_gemv_q8_0q8 / _q4_0q8),
 * and their pooled forms -- that this thread makes on `stream` between
 * begin and end are queued and run as one persistent launch per run of up to
 * 64 consecutive same-format calls: the weights of call i+1 stream while call
 * i's last rows fold, and each call's activations are staged once, by a small
 * kernel, for the whole launch.  A lone GEMV pays about 6 us of launch,
 * staging and fold latency; a decode step of many GEMVs pays it once.
 * Every call keeps its own checks and its results: bit for bit those of the
 * call made on its own, except in LP_FP32_FAST mode, whose unordered fold
 * follows the launch's row tiles, so a batched result may differ from the
 * lone call's in the last bits (within the same bound).  Argument errors
 * return at once.  Queued calls are launched at end, or earlier when this
 * thread makes any other launch of the library (stream order holds), a call
 * of another format, fp32 mode or stream, a call whose x or y meets an
 * earlier queued call's y, or a 65th call; a launch failure is returned by
 * the call that launched, or by end.  y and x pointers are read at launch, so
 * queued buffers must stay allocated until then.  Each launch stages the
 * activations in a stream-ordered allocation from a memory pool the library
 * creates per device (a few KB to 44 KB per call, freed in stream order after
 * it; up to 64 MB stay reserved for the next batch; graph memory nodes under
 * stream capture) -- the one allocation of the device forms.  Pooled calls in
 * a gather group may share a launch; the group's receive launches the queue
 * first.  begin on an open batch ends it. */
int lp_batch_begin(lp_stream_t stream);
int lp_batch_end(lp_stream_t stream);

/* ======================= fp32-activation fused dequant-GEMVs ========== */

/* Arithmetic of the fp32-activation GEMVs (process-wide, default FAST).
 *   LP_FP32_FAST   activations as block-float integers (22-bit per group,
 *                  three int8 planes), exact integer group dots: per row the
 *                  error is a few ulp of sum|w*x| (measured on config 1: at
 *                  most 4.7e-8 of it), not bit-identical to the reference's
 *                  summation order.  Where a row's dot cancels, the relative
 *                  error of that element can pass 1e-5 -- as the reference's
 *                  own fp32 order does against an fp64 dot (config 1: 195 of
 *                  11008 rows here, 99 for the reference order).  Used when
 *                  the group size is a multiple of 8.
 *   LP_FP32_EXACT  the reference scalar path's exact operation order
 *                  (simd/dequant.nim:253-256 and kin): bit-identical results.
 * No counterpart in the reference (its x86 build runs the scalar order).
 * Returns LP_ERR_ARG for an unknown mode. */
#define LP_FP32_FAST 0
#define LP_FP32_EXACT 1
int lp_set_fp32_mode(int mode);
int lp_get_fp32_mode(void);

/* dequantGemv: int8 weights M x K, scales M x (K/groupSize), fp32 x -> y.
 * Replaces simd/dequant.nim:210-257 (proc dequantGemv*). */
int lp_dequant_gemv(const int8_t *wq, int64_t wq_len, const float *scales, int64_t scales_len,
                    int64_t group_size, const float *x, int64_t x_len, float *y, int64_t y_len,
                    lp_stream_t stream);

/* dequantGemvI4: packed two's-complement int4 (low nibble = even column).
 * Replaces simd/dequant.nim:259-339 (proc dequantGemvI4*). */
int lp_dequant_gemv_i4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                       int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                       float *y, int64_t y_len, lp_stream_t stream);

/* dequantGemvF4: packed MXFP4 e2m1 codes with fp32 (E8M0-valued) scales.
 * Replaces simd/dequant.nim:341-420 (proc dequantGemvF4*). */
int lp_dequant_gemv_f4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                       int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                       float *y, int64_t y_len, lp_stream_t stream);

/* dequantGemvQ8_0: ggml Q8_0 weight blocks, M x blocksPerRow.
 * Replaces simd/dequant.nim:530-568 (proc dequantGemvQ8_0*). */
int lp_dequant_gemv_q8_0(const void *w, int64_t w_len, int64_t blocks_per_row, const float *x,
                         int64_t x_len, float *y, int64_t y_len, lp_stream_t stream);

/* dequantGemvQ4_0: ggml Q4_0 weight blocks, M x blocksPerRow.
 * Replaces simd/dequant.nim:570-622 (proc dequantGemvQ4_0*). */
int lp_dequant_gemv_q4_0(const void *w, int64_t w_len, int64_t blocks_per_row, const float *x,
                         int64_t x_len, float *y, int64_t y_len, lp_stream_t stream);

/* Fused k-quant GEMVs (GGUF Q4_K / Q6_K weights, fp32 activations): w is
 * m x superblocks_per_row super-blocks of 256 elements (Q4_K 144 bytes, Q6_K
 * 210 bytes, the layouts ggml.nim:99-213 decodes), x 256 * superblocks_per_row
 * floats.  The element values are the reference's dequantizeQ4_K /
 * dequantizeQ6_K values (ggml.nim:136-161, 163-213); the reference has no
 * fused GEMV over them, so these have no counterpart proc.  Block-float
 * arithmetic (exact integer 32-element dots, as LP_FP32_FAST) in every fp32
 * mode: within a few ulp of sum|w x| per row of the exact product. */
int lp_dequant_gemv_q4_k(const void *w, int64_t w_len, int64_t superblocks_per_row,
                         const float *x, int64_t x_len, float *y, int64_t y_len,
                         lp_stream_t stream);
int lp_dequant_gemv_q6_k(const void *w, int64_t w_len, int64_t superblocks_per_row,
                         const float *x, int64_t x_len, float *y, int64_t y_len,
                         lp_stream_t stream);

/* ======================= int8-activation GEMVs (bit-exact) ============ */

/* dequantGemvQ8: int8 weights and int8 activations, exact int32 group sums.
 * Replaces simd/dequant.nim:753-878 (proc dequantGemvQ8*). */
int lp_dequant_gemv_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                       int64_t w_scales_len, int64_t group_size, const int8_t *xq, int64_t xq_len,
                       const float *x_scales, int64_t x_scales_len, float *y, int64_t y_len,
                       lp_stream_t stream);

/* dequantGemvI4Q8: packed int4 weights, int8 activations.
 * Replaces simd/dequant.nim:968-1145 (proc dequantGemvI4Q8*). */
int lp_dequant_gemv_i4q8(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                         int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                         int64_t xq_len, const float *x_scales, int64_t x_scales_len, float *y,
                         int64_t y_len, lp_stream_t stream);

/* quantizeQ8_0 of fp32 x followed by dequantGemvQ8 / dequantGemvI4Q8, in one
 * launch: the GEMV quantizes the activations while it stages them, with the
 * arithmetic of lp_quantize_q8_0_split, so the results equal the two calls'
 * bit for bit.  The composition of ggml.nim:60-75 (quantizeQ8_0, =
 * simd/dequant.nim:1624-1641) with simd/dequant.nim:753-878 / :968-1145; no
 * single proc of the reference.  group_size must be 32 (the Q8_0 block) and
 * x_len a multiple of 32. */
int lp_quantize_dequant_gemv_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                                int64_t w_scales_len, int64_t group_size, const float *x,
                                int64_t x_len, float *y, int64_t y_len, lp_stream_t stream);
int lp_quantize_dequant_gemv_i4q8(const uint8_t *wpacked, int64_t wpacked_len,
                                  const float *w_scales, int64_t w_scales_len, int64_t group_size,
                                  const float *x, int64_t x_len, float *y, int64_t y_len,
                                  lp_stream_t stream);

/* dequantGemvQ8_0Q8: Q8_0 weight blocks x Q8_0 activation blocks.
 * Replaces simd/dequant.nim:1187-1286 (proc dequantGemvQ8_0Q8*). */
int lp_dequant_gemv_q8_0q8(const void *w, int64_t w_len, int64_t blocks_per_row, const void *xq,
                           int64_t xq_len, float *y, int64_t y_len, lp_stream_t stream);

/* dequantGemvQ4_0Q8: Q4_0 weight blocks x Q8_0 activation blocks.
 * Replaces simd/dequant.nim:1288-1365 (proc dequantGemvQ4_0Q8*). */
int lp_dequant_gemv_q4_0q8(const void *w, int64_t w_len, int64_t blocks_per_row, const void *xq,
                           int64_t xq_len, float *y, int64_t y_len, lp_stream_t stream);

/* ======================= multi-column GEMM (bit-exact) ================= */

/* dequantGemmQ8: xq is K x n column-major, x_scales n x gpr, y M x n
 * row-major.  Replaces simd/dequant.nim:1382-1458 (proc dequantGemmQ8*). */
int lp_dequant_gemm_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                       int64_t w_scales_len, int64_t group_size, const int8_t *xq, int64_t xq_len,
                       const float *x_scales, int64_t x_scales_len, int64_t n, float *y,
                       int64_t y_len, lp_stream_t stream);

/* dequantGemmI4Q8: the same over packed int4 weights.
 * Replaces simd/dequant.nim:1460-1583 (proc dequantGemmI4Q8*). */
int lp_dequant_gemm_i4q8(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                         int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                         int64_t xq_len, const float *x_scales, int64_t x_scales_len, int64_t n,
                         float *y, int64_t y_len, lp_stream_t stream);

/* ======================= FP4 x FP4 GEMMs on block-scaled tensor cores == */
/* Both operands in a 4-bit float scheme, two e2m1 codes per byte (low nibble
 * = even element): weights m rows of k/2 bytes, activations n columns of k/2
 * bytes (K x n column-major, as dequantGemmQ8 takes xq), y m x n row-major:
 *   y[r*n + c] = G * sum_b sw[r,b] * sx[c,b] * sum_{i in b} e2m1(w[r,i]) * e2m1(x[c,i])
 * The products are exact and the sums fp32 (tensor-core accumulation), so
 * results agree with an exact evaluation within fp32 rounding, not bit for bit
 * with a sequential order.  Operands 16-byte aligned; m, n, k up to 2^30. */

/* MXFP4 x MXFP4 (tcgen05.mma kind::mxf4, one E8M0 scale per 32 elements,
 * G = 1): the GEMM form of dequantGemvF4 (simd/dequant.nim:341-420, whose
 * e2m1 table and scale meaning it keeps) with the activations quantized by
 * the same scheme (calibrateMX + packF4: lp_calibrate_mx,
 * lp_quantize_f4_packed).  The scales are fp32 powers of two (calibrateMX's
 * output), m x k/32 and n x k/32; group_size must be 32.  No single proc of
 * the reference. */
int lp_dequant_gemm_f4(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                       int64_t w_scales_len, int64_t group_size, const uint8_t *xpacked,
                       int64_t xpacked_len, const float *x_scales, int64_t x_scales_len, int64_t n,
                       float *y, int64_t y_len, lp_stream_t stream);

/* NVFP4 x NVFP4 (tcgen05.mma kind::mxf4nvf4, one e4m3 scale per 16 elements,
 * G = the product of the two global decode scales, each a DEVICE float as
 * lp_quantize_nvfp4 writes it): the decode of nvfp4.nim:80-92 applied to both
 * operands of a GEMM.  Block scales m x k/16 and n x k/16 bytes; k a multiple
 * of 32.  No single proc of the reference. */
int lp_gemm_nvfp4(const uint8_t *wpacked, int64_t wpacked_len, const uint8_t *w_block_scales,
                  int64_t w_block_scales_len, const float *w_global_decode_scale,
                  const uint8_t *xpacked, int64_t xpacked_len, const uint8_t *x_block_scales,
                  int64_t x_block_scales_len, const float *x_global_decode_scale, int64_t n,
                  float *y, int64_t y_len, lp_stream_t stream);

/* ======================= encoders (bit-exact) ========================== */

/* quantizeQ8_0Batch: fp32 -> Q8_0 blocks (d = amax/127 as fp16, ties-away
 * round, clamp +-127).  Replaces simd/dequant.nim:1624-1641 (= quantizeQ8_0,
 * ggml.nim:60-75). */
int lp_quantize_q8_0_batch(const float *src, int64_t src_len, void *blocks, int64_t blocks_len,
                           lp_stream_t stream);

/* quantizeQ4_0Batch: fp32 -> Q4_0 blocks (sign-keeping max, d = max/-8).
 * Replaces simd/dequant.nim:1643-1715 (= quantizeQ4_0, ggml.nim:77-97). */
int lp_quantize_q4_0_batch(const float *src, int64_t src_len, void *blocks, int64_t blocks_len,
                           lp_stream_t stream);

/* quantizeQ8_0 with the block split into the two arrays the group-scale
 * int8 kernels take: qs (src_len int8) and d (src_len/32 floats, each the
 * fp32 value of the block's fp16 scale).  Same arithmetic as ggml.nim:60-75;
 * the split is the layout change dequantGemvQ8 needs (its xq / xScales). */
int lp_quantize_q8_0_split(const float *src, int64_t src_len, int8_t *qs, int64_t qs_len,
                           float *d, int64_t d_len, lp_stream_t stream);

/* quantizeBatch: int8 encode q = toI8(x / scales[g] + zero_points[g]) (divide,
 * then add, ties-away round, clamp [-128,127]), g = i div group_size
 * (group_size <= 0: one per-tensor scale).  zero_points_len = 0 is the
 * symmetric case (QParams with an empty zeroPoint, + 0.0); otherwise it covers
 * every group.  Replaces simd/dequant.nim:1717-1750 (proc quantizeBatch*,
 * whose zero-point case falls through to quantize[I8], quant.nim:48-60). */
int lp_quantize_batch(const float *x, int64_t x_len, const float *scales, int64_t scales_len,
                      const float *zero_points, int64_t zero_points_len, int64_t group_size,
                      int8_t *dst, int64_t dst_len, lp_stream_t stream);

/* dequantizeBatch: dst = (f32(q) - zero_points[g]) * scales[g], g = i div
 * group_size (group_size <= 0: per tensor), for int8-backed I8 and I4 values
 * stored one per byte.  zero_points_len = 0 is the symmetric case (QParams
 * with an empty zeroPoint); otherwise it covers every group.  Replaces
 * simd/dequant.nim:159-206 (proc dequantizeBatch*, both instantiations) and
 * its scalar fall-through quant.nim:62-74 (proc dequantize*). */
int lp_dequantize_batch(const int8_t *q, int64_t q_len, const float *scales, int64_t scales_len,
                        const float *zero_points, int64_t zero_points_len, int64_t group_size,
                        float *dst, int64_t dst_len, lp_stream_t stream);

/* calibrateSymmetric: scale = absmax/qmax per group (1.0 for a zero group,
 * ragged last group, group_size <= 0 = per tensor).
 * Replaces quant.nim:95-110 (proc calibrateSymmetric*). */
int lp_calibrate_symmetric(const float *x, int64_t x_len, int64_t group_size, float qmax,
                           float *scales, int64_t scales_len, lp_stream_t stream);

/* calibrateMX: E8M0-valued fp32 scale 2^clamp(floor(log2 amax) - emax, +-127)
 * per block, 1.0 for a zero block.  Replaces quant.nim:125-137. */
int lp_calibrate_mx(const float *x, int64_t x_len, int64_t block_size, int32_t elem_emax,
                    float *scales, int64_t scales_len, lp_stream_t stream);

/* quantize[I4] + packInt4: q = toI4(x/scale + 0), two per byte, low nibble =
 * even index.  Replaces quant.nim:48-60 with intx.nim:50-51 and :83-94.
 * x_len must be even. */
int lp_quantize_i4_packed(const float *x, int64_t x_len, const float *scales,
                          int64_t scales_len, int64_t group_size, uint8_t *packed,
                          int64_t packed_len, lp_stream_t stream);

/* quantize[F4E2M1] + packF4: code = toF4E2M1(x/scale + 0), two per byte.
 * Replaces quant.nim:48-60 with mxfloat.nim:52-66 and :138-149. */
int lp_quantize_f4_packed(const float *x, int64_t x_len, const float *scales,
                          int64_t scales_len, int64_t block_size, uint8_t *packed,
                          int64_t packed_len, lp_stream_t stream);

/* dequantizeQ8_0Batch / dequantizeQ4_0Batch: blocks -> fp32.
 * Replace simd/dequant.nim:446-485 and :487-526 (= ggml.nim:36-56). */
int lp_dequantize_q8_0_batch(const void *blocks, int64_t blocks_len, float *dst, int64_t dst_len,
                             lp_stream_t stream);
int lp_dequantize_q4_0_batch(const void *blocks, int64_t blocks_len, float *dst, int64_t dst_len,
                             lp_stream_t stream);

/* dequantizeQ4_K / dequantizeQ6_K: 256-element k-quant super-blocks -> fp32
 * (blocks_len in super-blocks of 144 / 210 bytes; dst_len = 256 * blocks_len).
 * Replace ggml.nim:136-161 and :163-213. */
int lp_dequantize_q4_k(const void *blocks, int64_t blocks_len, float *dst, int64_t dst_len,
                       lp_stream_t stream);
int lp_dequantize_q6_k(const void *blocks, int64_t blocks_len, float *dst, int64_t dst_len,
                       lp_stream_t stream);

/* quantizeNVFP4 / dequantizeNVFP4: e2m1 codes (one byte per element) in
 * 16-element blocks, one e4m3 decode scale per block, one fp32 global decode
 * scale (written to *global_decode_scale, a device float; the reference
 * returns it).  x_len a multiple of 16.  Replace nvfp4.nim:39-78 and :80-92. */
int lp_quantize_nvfp4(const float *x, int64_t x_len, uint8_t *codes, int64_t codes_len,
                      uint8_t *block_scales, int64_t scales_len, float *global_decode_scale,
                      lp_stream_t stream);
int lp_dequantize_nvfp4(const uint8_t *codes, int64_t codes_len, const uint8_t *block_scales,
                        int64_t scales_len, float global_decode_scale, float *dst,
                        int64_t dst_len, lp_stream_t stream);

/* ======================= host-pointer drop-in forms ==================== */
/* Same arguments and meaning as the lp_* forms above, HOST pointers, no
 * stream; blocking.  Each replaces the same reference proc as its lp_* form
 * (simd/dequant.nim, ggml.nim), with the Nim signature's host arrays. */
int lph_dequant_gemv(const int8_t *wq, int64_t wq_len, const float *scales, int64_t scales_len,
                     int64_t group_size, const float *x, int64_t x_len, float *y, int64_t y_len);
int lph_dequant_gemv_i4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                        int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                        float *y, int64_t y_len);
int lph_dequant_gemv_f4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                        int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                        float *y, int64_t y_len);
int lph_dequant_gemv_q8_0(const void *w, int64_t w_len, int64_t blocks_per_row, const float *x,
                          int64_t x_len, float *y, int64_t y_len);
int lph_dequant_gemv_q4_0(const void *w, int64_t w_len, int64_t blocks_per_row, const float *x,
                          int64_t x_len, float *y, int64_t y_len);
int lph_dequant_gemv_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                        int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                        int64_t xq_len, const float *x_scales, int64_t x_scales_len, float *y,
                        int64_t y_len);
int lph_dequant_gemv_i4q8(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                          int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                          int64_t xq_len, const float *x_scales, int64_t x_scales_len, float *y,
                          int64_t y_len);
int lph_dequant_gemv_q8_0q8(const void *w, int64_t w_len, int64_t blocks_per_row, const void *xq,
                            int64_t xq_len, float *y, int64_t y_len);
int lph_dequant_gemv_q4_0q8(const void *w, int64_t w_len, int64_t blocks_per_row, const void *xq,
                            int64_t xq_len, float *y, int64_t y_len);
int lph_dequant_gemm_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                        int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                        int64_t xq_len, const float *x_scales, int64_t x_scales_len, int64_t n,
                        float *y, int64_t y_len);
int lph_dequant_gemm_i4q8(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                          int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                          int64_t xq_len, const float *x_scales, int64_t x_scales_len, int64_t n,
                          float *y, int64_t y_len);
int lph_quantize_q8_0_batch(const float *src, int64_t src_len, void *blocks, int64_t blocks_len);
int lph_quantize_q4_0_batch(const float *src, int64_t src_len, void *blocks, int64_t blocks_len);
int lph_quantize_batch(const float *x, int64_t x_len, const float *scales, int64_t scales_len,
                       const float *zero_points, int64_t zero_points_len, int64_t group_size,
                       int8_t *dst, int64_t dst_len);
int lph_dequantize_batch(const int8_t *q, int64_t q_len, const float *scales, int64_t scales_len,
                         const float *zero_points, int64_t zero_points_len, int64_t group_size,
                         float *dst, int64_t dst_len);

/* ======================= host form that allocates nothing ============== */
/* No counterpart in the reference.  For callers that may not allocate device
 * memory during a call (real-time callbacks, hosts with a memory budget fixed
 * at start-up, embeddings that forbid cudaMalloc after initialisation):
 * dequantGemvQ4_0 with host arrays, like lph_dequant_gemv_q4_0 (same
 * arguments, same results), but its inputs and output are staged in one
 * static 32 MiB device array that every GPU loading the library holds until
 * exit, instead of a workspace grown with cudaMalloc.  No cudaMalloc, cudaFree
 * or other allocating call is made.  Shape errors return LP_ERR_SHAPE before
 * anything is copied; LP_ERR_UNSUPPORTED when the staged bytes (18 per block +
 * 4 per x and y element, each rounded up to 256) exceed 32 MiB.  The first
 * call on a device looks up the array's address (make it before any stream
 * capture).  The array is shared process-wide: calls that overlap in time race
 * on it and must be serialised by the caller. */
int lph_dequant_gemv_q4_0_static(const void *w, int64_t w_len, int64_t blocks_per_row,
                                 const float *x, int64_t x_len, float *y, int64_t y_len);

/* ======================= LpPool: row-sharded forms across GPUs ======== *
 * One process (rank) per GPU of a box.  Rank r owns the rows
 * [per*r, per*r + per) of every weight matrix, per = m div P, and the last
 * rank the remainder -- the slicing of parallel.nim:118-124, so sharded ==
 * serial bit for bit.  A pooled call takes this rank's weight (and weight
 * scale) row slice, the whole activations and the whole y; it computes the
 * slice's rows and gathers every rank's rows into y over NCCL, in stream
 * order.  Replaces LpPool / initPool / shutdown (parallel.nim:82-184) and the
 * pooled and per-call par* procs (:186-474).  NCCL is loaded when a pool is
 * created; without it these calls return LP_ERR_NCCL. */
typedef struct lp_pool *lp_pool_t;

/* The row slice of rank `rank` among `nranks` for m rows (parallel.nim:118-124). */
int lp_pool_rows(int64_t m, int nranks, int rank, int64_t *begin, int64_t *end);
/* 128-byte NCCL unique id: create on one rank, hand to all (e.g. a torch store). */
int lp_pool_unique_id(uint8_t *id128);
/* Join the pool as `rank` of `nranks` on CUDA device `device` (initPool). */
int lp_pool_init(lp_pool_t *pool, const uint8_t *id128, int nranks, int rank, int device);
/* Leave and free the pool; NULL is accepted (shutdown is idempotent). */
int lp_pool_destroy(lp_pool_t pool);
int lp_pool_size(lp_pool_t pool, int *nranks, int *rank);
/* The gather's transport (no counterpart in the reference).  By default a pool
 * whose ranks each have their own GPU maps every rank's exchange buffer over
 * NVLink (CUDA IPC, set up by lp_pool_init) and gathers with 8-byte peer
 * stores that carry the gather's sequence number beside each float (pooled
 * GEMVs store their rows from the GEMV itself), read back with bounded
 * polls; enable = 0 selects the NCCL
 * group instead.  Every rank must make the same choice before its next gather.
 * LP_ERR_UNSUPPORTED: the exchange could not be mapped on every rank. */
int lp_pool_set_p2p(lp_pool_t pool, int enable);
int lp_pool_get_p2p(lp_pool_t pool, int *enabled);
/* Gather group (no counterpart in the reference): pooled calls made between
 * begin and end whose y lies inside [y, y + y_len) (each its own row-sharded
 * part of that vector, at most 64) store their rows into the other ranks as
 * usual, and the whole vector is received once, at end, in stream order --
 * one exchange for several GEMVs (config 4: a layer's two GEMVs).  Every rank
 * makes the same calls.  On the NVLink transport a pooled call outside the
 * vector, or a 65th part, returns LP_ERR_ARG; begin returns
 * LP_ERR_UNSUPPORTED for a vector larger than the exchange (2^21 floats).
 * On the NCCL transport every call gathers on its own and end does nothing.
 * A group of 2^18 floats or more (a whole decode step) has each GEMV publish
 * its outputs in its own rank's exchange buffer and the receive read the
 * other ranks' buffers over NVLink; smaller gathers store into every other
 * rank's buffer from the GEMV.  When a group's parts are all GEMVs and some
 * are still queued in an open batch (lp_batch_begin) at end, the receive runs
 * at the end of that batch's launch, in each CTA once its rows are done,
 * instead of in a kernel of its own.  Same results either way. */
int lp_pool_group_begin(lp_pool_t pool, float *y, int64_t y_len);
int lp_pool_group_end(lp_pool_t pool, lp_stream_t stream);
/* Gather every rank's row slice of y (m rows of per_row floats) in place:
 * the output exchange inside the reference's par* procs (parallel.nim:186-474),
 * on its own. */
int lp_pool_gather_rows(lp_pool_t pool, float *y, int64_t m, int64_t per_row, lp_stream_t stream);

/* Pooled forms of the GEMVs / GEMMs above (parDequantGemv*, parDequantGemm*:
 * parallel.nim:186-474). */
int lp_pool_dequant_gemv(lp_pool_t pool, const int8_t *wq, int64_t wq_len, const float *scales,
                         int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                         float *y, int64_t y_len, lp_stream_t stream);
int lp_pool_dequant_gemv_i4(lp_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                            const float *scales, int64_t scales_len, int64_t group_size,
                            const float *x, int64_t x_len, float *y, int64_t y_len,
                            lp_stream_t stream);
int lp_pool_dequant_gemv_f4(lp_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                            const float *scales, int64_t scales_len, int64_t group_size,
                            const float *x, int64_t x_len, float *y, int64_t y_len,
                            lp_stream_t stream);
int lp_pool_dequant_gemv_q8_0(lp_pool_t pool, const void *w, int64_t w_len,
                              int64_t blocks_per_row, const float *x, int64_t x_len, float *y,
                              int64_t y_len, lp_stream_t stream);
int lp_pool_dequant_gemv_q4_0(lp_pool_t pool, const void *w, int64_t w_len,
                              int64_t blocks_per_row, const float *x, int64_t x_len, float *y,
                              int64_t y_len, lp_stream_t stream);
int lp_pool_dequant_gemv_q8(lp_pool_t pool, const int8_t *wq, int64_t wq_len,
                            const float *w_scales, int64_t w_scales_len, int64_t group_size,
                            const int8_t *xq, int64_t xq_len, const float *x_scales,
                            int64_t x_scales_len, float *y, int64_t y_len, lp_stream_t stream);
int lp_pool_dequant_gemv_i4q8(lp_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                              const float *w_scales, int64_t w_scales_len, int64_t group_size,
                              const int8_t *xq, int64_t xq_len, const float *x_scales,
                              int64_t x_scales_len, float *y, int64_t y_len, lp_stream_t stream);
/* Pooled forms of lp_quantize_dequant_gemv_q8 / _i4q8: each rank quantizes
 * the whole fp32 x to Q8_0 while staging it and runs its row slice; y is
 * assembled on every rank (parDequantGemvQ8 / parDequantGemvI4Q8 after
 * quantizeQ8_0 of the activations, parallel.nim:310-418). */
int lp_pool_quantize_dequant_gemv_q8(lp_pool_t pool, const int8_t *wq, int64_t wq_len,
                                     const float *w_scales, int64_t w_scales_len,
                                     int64_t group_size, const float *x, int64_t x_len, float *y,
                                     int64_t y_len, lp_stream_t stream);
int lp_pool_quantize_dequant_gemv_i4q8(lp_pool_t pool, const uint8_t *wpacked,
                                       int64_t wpacked_len, const float *w_scales,
                                       int64_t w_scales_len, int64_t group_size, const float *x,
                                       int64_t x_len, float *y, int64_t y_len,
                                       lp_stream_t stream);
int lp_pool_dequant_gemm_q8(lp_pool_t pool, const int8_t *wq, int64_t wq_len,
                            const float *w_scales, int64_t w_scales_len, int64_t group_size,
                            const int8_t *xq, int64_t xq_len, const float *x_scales,
                            int64_t x_scales_len, int64_t n, float *y, int64_t y_len,
                            lp_stream_t stream);
int lp_pool_dequant_gemm_i4q8(lp_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                              const float *w_scales, int64_t w_scales_len, int64_t group_size,
                              const int8_t *xq, int64_t xq_len, const float *x_scales,
                              int64_t x_scales_len, int64_t n, float *y, int64_t y_len,
                              lp_stream_t stream);

/* ======================= LpPool in one process, host arrays ========== *
 * The reference's LpPool is one process with worker threads over host
 * arrays.  Here a worker is a host thread bound to one GPU: a pooled call
 * slices the rows as the reference does (per = rows div n, worker t owns
 * [per*t, per*t + per), the last one the remainder; parallel.nim:118-124),
 * each worker runs the host form (lph_*) of its slice on its GPU, and the
 * slices of y come back into the caller's y.  Results equal the serial call
 * bit for bit.  Blocking; not safe to call concurrently on one pool
 * (parallel.nim:85-91). */
typedef struct lph_pool *lph_pool_t;

/* initPool(threads): a pool of `threads` GPUs (<= 0: every visible GPU;
 * capped at the number visible), devices 0 .. n-1.  LP_ERR_NO_DEVICE without
 * a GPU.  Replaces parallel.nim:134-151 (proc initPool*). */
int lph_pool_init(lph_pool_t *pool, int threads);
/* shutdown: stop the workers and free the pool; *pool becomes NULL, and a
 * NULL pool is accepted (idempotent).  Replaces parallel.nim:153-167. */
int lph_pool_shutdown(lph_pool_t *pool);
/* threadCount: workers (GPUs) of the pool, 0 for NULL.  Replaces
 * parallel.nim:169-171. */
int lph_pool_thread_count(lph_pool_t pool);

/* Pooled forms (serial fallback when the pool has one worker or fewer than
 * 128 rows, parallel.nim:358-360).  Replace parDequantGemvQ8 /
 * parDequantGemvI4Q8 (parallel.nim:346-374, pooled overloads) and
 * parDequantGemmQ8 / parDequantGemmI4Q8 (parallel.nim:420-474). */
int lph_pool_dequant_gemv_q8(lph_pool_t pool, const int8_t *wq, int64_t wq_len,
                             const float *w_scales, int64_t w_scales_len, int64_t group_size,
                             const int8_t *xq, int64_t xq_len, const float *x_scales,
                             int64_t x_scales_len, float *y, int64_t y_len);
int lph_pool_dequant_gemv_i4q8(lph_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                               const float *w_scales, int64_t w_scales_len, int64_t group_size,
                               const int8_t *xq, int64_t xq_len, const float *x_scales,
                               int64_t x_scales_len, float *y, int64_t y_len);
int lph_pool_dequant_gemm_q8(lph_pool_t pool, const int8_t *wq, int64_t wq_len,
                             const float *w_scales, int64_t w_scales_len, int64_t group_size,
                             const int8_t *xq, int64_t xq_len, const float *x_scales,
                             int64_t x_scales_len, int64_t n, float *y, int64_t y_len);
int lph_pool_dequant_gemm_i4q8(lph_pool_t pool, const uint8_t *wpacked, int64_t wpacked_len,
                               const float *w_scales, int64_t w_scales_len, int64_t group_size,
                               const int8_t *xq, int64_t xq_len, const float *x_scales,
                               int64_t x_scales_len, int64_t n, float *y, int64_t y_len);

/* Per-call forms par*(..., threads): shards = min(threads, rows div 64), at
 * least 1, threads <= 0 meaning every GPU (shardCount, parallel.nim:45-53),
 * over one pool of every visible GPU made on first use; one shard runs the
 * serial host form.  Replace parallel.nim:186-418 (parDequantGemv,
 * parDequantGemvI4, parDequantGemvF4, parDequantGemvQ8_0, parDequantGemvQ4_0,
 * and the per-call overloads of parDequantGemvQ8 / parDequantGemvI4Q8). */
int lph_par_dequant_gemv(const int8_t *wq, int64_t wq_len, const float *scales,
                         int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                         float *y, int64_t y_len, int threads);
int lph_par_dequant_gemv_i4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                            int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                            float *y, int64_t y_len, int threads);
int lph_par_dequant_gemv_f4(const uint8_t *wpacked, int64_t wpacked_len, const float *scales,
                            int64_t scales_len, int64_t group_size, const float *x, int64_t x_len,
                            float *y, int64_t y_len, int threads);
int lph_par_dequant_gemv_q8_0(const void *w, int64_t w_len, int64_t blocks_per_row,
                              const float *x, int64_t x_len, float *y, int64_t y_len, int threads);
int lph_par_dequant_gemv_q4_0(const void *w, int64_t w_len, int64_t blocks_per_row,
                              const float *x, int64_t x_len, float *y, int64_t y_len, int threads);
int lph_par_dequant_gemv_q8(const int8_t *wq, int64_t wq_len, const float *w_scales,
                            int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                            int64_t xq_len, const float *x_scales, int64_t x_scales_len, float *y,
                            int64_t y_len, int threads);
int lph_par_dequant_gemv_i4q8(const uint8_t *wpacked, int64_t wpacked_len, const float *w_scales,
                              int64_t w_scales_len, int64_t group_size, const int8_t *xq,
                              int64_t xq_len, const float *x_scales, int64_t x_scales_len,
                              float *y, int64_t y_len, int threads);

#ifdef __cplusplus
}
#endif

#endif /* LOWPREC_CUDA_H */
