// capi.cu -- the extern "C" boundary (include/lowprec_cuda.h).
//
// Shape rules follow the reference procs' entry asserts: m = y.len,
// k = x.len, gpr = k div groupSize, and the listed length equalities
// (e.g. simd/dequant.nim:221-226, 768-771, 1392-1400).  A failed rule
// returns LP_ERR_SHAPE before anything is launched.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "gemv.cuh"
#include "lp_internal.h"

namespace lp {

const DeviceInfo& device_info() {
  static DeviceInfo info[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = dev % kMaxDevices;
  std::call_once(once[slot], [&] {
    DeviceInfo& d = info[slot];
    d.ordinal = dev;
    cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&d.smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  });
  return info[slot];
}

namespace {
thread_local char t_detail[256] = "";
}

const char* t_detail_ptr() { return t_detail; }

void note_cuda_error(cudaError_t e) {
  snprintf(t_detail, sizeof(t_detail), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
}

void note_text(const char* text) { snprintf(t_detail, sizeof(t_detail), "%s", text); }

}  // namespace lp

using lp::GemvParams;

namespace {

#define LP_REQUIRE(cond)          \
  do {                            \
    if (!(cond)) return LP_ERR_SHAPE; \
  } while (0)

// Set by the host-staging forms: run an entry point's shape and argument
// checks only, so a bad call fails before any device work or allocation.
thread_local bool t_validate_only = false;

}  // namespace

namespace lp {
void set_validate_only(bool on) { t_validate_only = on; }
}  // namespace lp

namespace {

#define LP_VALIDATED()                   \
  do {                                   \
    if (t_validate_only) return LP_OK;   \
  } while (0)

// The stream of a launch.  S: any launch but a GEMV's -- it first launches
// the GEMVs recorded in this thread's open batch (a failure there is kept for
// lp_batch_end), so stream order holds.  SG: a GEMV, which may join the batch.
inline cudaStream_t SG(lp_stream_t s) { return static_cast<cudaStream_t>(s); }
inline cudaStream_t S(lp_stream_t s) {
  if (lp::batch_open()) lp::batch_flush_keep();
  return static_cast<cudaStream_t>(s);
}

GemvParams base(const void* w, const float* ws, const void* x, const float* xs, float* y,
                int64_t m, int64_t k, int64_t gs, int64_t gpr, int64_t row_bytes) {
  GemvParams p;
  std::memset(&p, 0, sizeof(p));
  p.w = static_cast<const uint8_t*>(w);
  p.ws = ws;
  p.x = x;
  p.xs = xs;
  p.y = y;
  p.m = static_cast<int>(m);
  p.k = static_cast<int>(k);
  p.gs = static_cast<int>(gs);
  p.gpr = static_cast<int>(gpr);
  p.row_bytes = static_cast<int>(row_bytes);
  p.neg_zero = -0.0f;
  return p;
}

constexpr int64_t kIntMax = 0x7fffffff;
// Widest GEMM (activation columns) run by the GEMV skeleton's column formats.
constexpr int64_t kGemmColsMax = 16;

std::atomic<int> g_fp32_mode{LP_FP32_FAST};

// The block-float path needs whole 8-element chunks per group.
inline bool fast_fp32(int64_t gs) { return g_fp32_mode.load() == LP_FP32_FAST && gs % 8 == 0; }

// A pointer may be null only when its array is empty.
inline bool bad(const void* p, int64_t len) { return len > 0 && p == nullptr; }

bool fits(int64_t m, int64_t k) { return m >= 0 && k >= 0 && m <= kIntMax && k <= kIntMax; }

}  // namespace

extern "C" {

int lp_version(void) { return 100; }

const char* lp_status_string(int s) {
  switch (s) {
    case LP_OK: return "ok";
    case LP_ERR_SHAPE: return "shape precondition failed";
    case LP_ERR_ARG: return "invalid argument";
    case LP_ERR_CUDA: return "CUDA error";
    case LP_ERR_NCCL: return "collective error";
    case LP_ERR_TIMEOUT: return "device-side wait timed out";
    case LP_ERR_UNSUPPORTED: return "shape not supported by this build";
    case LP_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char* lp_last_error_detail(void) { return lp::t_detail_ptr(); }

int lp_set_fp32_mode(int mode) {
  if (mode != LP_FP32_FAST && mode != LP_FP32_EXACT) return LP_ERR_ARG;
  g_fp32_mode.store(mode);
  return LP_OK;
}

int lp_get_fp32_mode(void) { return g_fp32_mode.load(); }

int lp_device_error(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return LP_ERR_CUDA;
  unsigned int e = lp::take_error_gemv();
  const unsigned int e2 = lp::take_error_gemm_tc();
  const unsigned int e3 = lp::take_error_pool();
  const unsigned int e4 = lp::take_error_gemm_fp4();
  if (!e) e = e2;
  if (!e) e = e3;
  if (!e) e = e4;
  return static_cast<int>(e);
}

int lp_batch_begin(lp_stream_t stream) { return lp::batch_begin(static_cast<cudaStream_t>(stream)); }

int lp_batch_end(lp_stream_t stream) { return lp::batch_end(static_cast<cudaStream_t>(stream)); }

int lp_host_device_pointer(const void* host, void** dev) {
  if (!host || !dev) return LP_ERR_ARG;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0) != cudaSuccess || !d) {
    cudaGetLastError();  // not page-locked here: clear the runtime's error
    return LP_ERR_ARG;
  }
  *dev = d;
  return LP_OK;
}

int lp_copy_in(void* dst, const void* src, int64_t bytes, lp_stream_t stream) {
  if (bytes < 0 || bad(dst, bytes) || bad(src, bytes)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_copy_in(dst, src, bytes, S(stream));
}

// ------------------------------------------------ fp32-activation GEMVs

static int gemv_f32_group(int fmt, const void* w, int64_t w_len, const float* scales,
                          int64_t scales_len, int64_t gs, const float* x, int64_t x_len, float* y,
                          int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len, k = x_len;
  LP_REQUIRE(gs > 0 && fits(m, k));
  const int64_t gpr = k / gs;
  const bool packed = fmt != 0;
  const int64_t rb = packed ? k / 2 : k;
  LP_REQUIRE(k % gs == 0);
  if (packed) LP_REQUIRE(k % 2 == 0);
  LP_REQUIRE(w_len == m * rb && scales_len == m * gpr);
  if (bad(w, w_len) || bad(scales, scales_len) || bad(x, x_len) || bad(y, y_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  GemvParams p = base(w, scales, x, nullptr, y, m, k, gs, gpr, rb);
  if (fast_fp32(gs)) {
    switch (fmt) {
      case 0: return lp::launch_gemv<lp::FmtI8F>(p, SG(st));
      case 1: return lp::launch_gemv<lp::FmtI4F>(p, SG(st));
      default: return lp::launch_gemv<lp::FmtF4F>(p, SG(st));
    }
  }
  switch (fmt) {
    case 0: return lp::launch_gemv<lp::FmtI8>(p, SG(st));
    case 1: return lp::launch_gemv<lp::FmtI4>(p, SG(st));
    default: return lp::launch_gemv<lp::FmtF4>(p, SG(st));
  }
}

int lp_dequant_gemv(const int8_t* wq, int64_t wq_len, const float* scales, int64_t scales_len,
                    int64_t group_size, const float* x, int64_t x_len, float* y, int64_t y_len,
                    lp_stream_t stream) {
  return gemv_f32_group(0, wq, wq_len, scales, scales_len, group_size, x, x_len, y, y_len, stream);
}
int lp_dequant_gemv_i4(const uint8_t* wp, int64_t wp_len, const float* scales, int64_t scales_len,
                       int64_t group_size, const float* x, int64_t x_len, float* y, int64_t y_len,
                       lp_stream_t stream) {
  return gemv_f32_group(1, wp, wp_len, scales, scales_len, group_size, x, x_len, y, y_len, stream);
}
int lp_dequant_gemv_f4(const uint8_t* wp, int64_t wp_len, const float* scales, int64_t scales_len,
                       int64_t group_size, const float* x, int64_t x_len, float* y, int64_t y_len,
                       lp_stream_t stream) {
  return gemv_f32_group(2, wp, wp_len, scales, scales_len, group_size, x, x_len, y, y_len, stream);
}

static int gemv_f32_blocks(int q4, const void* w, int64_t w_len, int64_t bpr, const float* x,
                           int64_t x_len, float* y, int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len;
  LP_REQUIRE(bpr >= 0 && fits(m, bpr * 32));
  LP_REQUIRE(w_len == m * bpr && x_len == bpr * 32);
  if (bad(w, w_len) || bad(x, x_len) || bad(y, y_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  const int64_t rb = bpr * (q4 ? 18 : 34);
  GemvParams p = base(w, nullptr, x, nullptr, y, m, bpr * 32, 32, bpr, rb);
  if (fast_fp32(32))
    return q4 ? lp::launch_gemv<lp::FmtQ4_0F>(p, SG(st)) : lp::launch_gemv<lp::FmtQ8_0F>(p, SG(st));
  return q4 ? lp::launch_gemv<lp::FmtQ4_0>(p, SG(st)) : lp::launch_gemv<lp::FmtQ8_0>(p, SG(st));
}

int lp_dequant_gemv_q8_0(const void* w, int64_t w_len, int64_t bpr, const float* x, int64_t x_len,
                         float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_f32_blocks(0, w, w_len, bpr, x, x_len, y, y_len, stream);
}
int lp_dequant_gemv_q4_0(const void* w, int64_t w_len, int64_t bpr, const float* x, int64_t x_len,
                         float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_f32_blocks(1, w, w_len, bpr, x, x_len, y, y_len, stream);
}

// Fused k-quant GEMVs: w is m x sbpr super-blocks (144 / 210 bytes), x is
// 256 * sbpr floats.  Always the block-float arithmetic (no reference order
// exists for a fused k-quant GEMV).
static int gemv_kquant(int q6, const void* w, int64_t w_len, int64_t sbpr, const float* x,
                       int64_t x_len, float* y, int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len;
  LP_REQUIRE(sbpr >= 0 && fits(m, sbpr * 256));
  LP_REQUIRE(w_len == m * sbpr && x_len == sbpr * 256);
  if (bad(w, w_len) || bad(x, x_len) || bad(y, y_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  const int64_t rb = sbpr * (q6 ? 210 : 144);
  GemvParams p = base(w, nullptr, x, nullptr, y, m, sbpr * 256, 32, sbpr * 8, rb);
  return q6 ? lp::launch_gemv<lp::FmtQ6_KF>(p, SG(st)) : lp::launch_gemv<lp::FmtQ4_KF>(p, SG(st));
}

int lp_dequant_gemv_q4_k(const void* w, int64_t w_len, int64_t sbpr, const float* x,
                         int64_t x_len, float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_kquant(0, w, w_len, sbpr, x, x_len, y, y_len, stream);
}
int lp_dequant_gemv_q6_k(const void* w, int64_t w_len, int64_t sbpr, const float* x,
                         int64_t x_len, float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_kquant(1, w, w_len, sbpr, x, x_len, y, y_len, stream);
}

// ------------------------------------------------ int8-activation GEMVs

static int gemv_q8_group(int i4, const void* w, int64_t w_len, const float* ws, int64_t ws_len,
                         int64_t gs, const int8_t* xq, int64_t xq_len, const float* xs,
                         int64_t xs_len, float* y, int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len, k = xq_len;
  LP_REQUIRE(gs > 0 && fits(m, k));
  const int64_t gpr = k / gs;
  const int64_t rb = i4 ? k / 2 : k;
  LP_REQUIRE(k % gs == 0);
  if (i4) LP_REQUIRE(k % 2 == 0);
  LP_REQUIRE(w_len == m * rb && ws_len == m * gpr && xs_len == gpr);
  if (bad(w, w_len) || bad(ws, ws_len) || bad(xq, xq_len) || bad(xs, xs_len) || bad(y, y_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  GemvParams p = base(w, ws, xq, xs, y, m, k, gs, gpr, rb);
  return i4 ? lp::launch_gemv<lp::FmtI4Q8>(p, SG(st)) : lp::launch_gemv<lp::FmtQ8>(p, SG(st));
}

// quantizeQ8_0 (ggml.nim:60-75) of fp32 x, then the Q8-activation GEMV, as
// one launch; Q8_0 blocks are 32 values, so the weight groups must be too.
static int gemv_q8_from_f32(int i4, const void* w, int64_t w_len, const float* ws,
                            int64_t ws_len, int64_t gs, const float* x, int64_t x_len, float* y,
                            int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len, k = x_len;
  LP_REQUIRE(gs == 32 && fits(m, k) && k % 32 == 0);
  const int64_t gpr = k / 32;
  const int64_t rb = i4 ? k / 2 : k;
  LP_REQUIRE(w_len == m * rb && ws_len == m * gpr);
  if (bad(w, w_len) || bad(ws, ws_len) || bad(x, x_len) || bad(y, y_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  GemvParams p = base(w, ws, x, nullptr, y, m, k, 32, gpr, rb);
  return i4 ? lp::launch_gemv<lp::FmtI4Q8FromF32>(p, SG(st))
            : lp::launch_gemv<lp::FmtQ8FromF32>(p, SG(st));
}

int lp_quantize_dequant_gemv_q8(const int8_t* wq, int64_t wq_len, const float* w_scales,
                                int64_t w_scales_len, int64_t group_size, const float* x,
                                int64_t x_len, float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_q8_from_f32(0, wq, wq_len, w_scales, w_scales_len, group_size, x, x_len, y, y_len,
                          stream);
}

int lp_quantize_dequant_gemv_i4q8(const uint8_t* wpacked, int64_t wpacked_len,
                                  const float* w_scales, int64_t w_scales_len, int64_t group_size,
                                  const float* x, int64_t x_len, float* y, int64_t y_len,
                                  lp_stream_t stream) {
  return gemv_q8_from_f32(1, wpacked, wpacked_len, w_scales, w_scales_len, group_size, x, x_len,
                          y, y_len, stream);
}

int lp_dequant_gemv_q8(const int8_t* wq, int64_t wq_len, const float* w_scales,
                       int64_t w_scales_len, int64_t group_size, const int8_t* xq, int64_t xq_len,
                       const float* x_scales, int64_t x_scales_len, float* y, int64_t y_len,
                       lp_stream_t stream) {
  return gemv_q8_group(0, wq, wq_len, w_scales, w_scales_len, group_size, xq, xq_len, x_scales,
                       x_scales_len, y, y_len, stream);
}
int lp_dequant_gemv_i4q8(const uint8_t* wp, int64_t wp_len, const float* w_scales,
                         int64_t w_scales_len, int64_t group_size, const int8_t* xq,
                         int64_t xq_len, const float* x_scales, int64_t x_scales_len, float* y,
                         int64_t y_len, lp_stream_t stream) {
  return gemv_q8_group(1, wp, wp_len, w_scales, w_scales_len, group_size, xq, xq_len, x_scales,
                       x_scales_len, y, y_len, stream);
}

static int gemv_q8_blocks(int q4, const void* w, int64_t w_len, int64_t bpr, const void* xq,
                          int64_t xq_len, float* y, int64_t y_len, lp_stream_t st) {
  const int64_t m = y_len;
  LP_REQUIRE(bpr >= 0 && fits(m, bpr * 32));
  LP_REQUIRE(w_len == m * bpr && xq_len == bpr);
  if (bad(w, w_len) || bad(xq, xq_len) || bad(y, y_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  const int64_t rb = bpr * (q4 ? 18 : 34);
  GemvParams p = base(w, nullptr, xq, nullptr, y, m, bpr * 32, 32, bpr, rb);
  return q4 ? lp::launch_gemv<lp::FmtQ4_0Q8>(p, SG(st)) : lp::launch_gemv<lp::FmtQ8_0Q8>(p, SG(st));
}

int lp_dequant_gemv_q8_0q8(const void* w, int64_t w_len, int64_t bpr, const void* xq,
                           int64_t xq_len, float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_q8_blocks(0, w, w_len, bpr, xq, xq_len, y, y_len, stream);
}
int lp_dequant_gemv_q4_0q8(const void* w, int64_t w_len, int64_t bpr, const void* xq,
                           int64_t xq_len, float* y, int64_t y_len, lp_stream_t stream) {
  return gemv_q8_blocks(1, w, w_len, bpr, xq, xq_len, y, y_len, stream);
}

// ------------------------------------------------------------------ GEMM

static int gemm_common(int i4, const void* w, int64_t w_len, const float* ws, int64_t ws_len,
                       int64_t gs, const int8_t* xq, int64_t xq_len, const float* xs,
                       int64_t xs_len, int64_t n, float* y, int64_t y_len, lp_stream_t st) {
  LP_REQUIRE(n > 0 && gs > 0);
  const int64_t m = y_len / n, k = xq_len / n;
  LP_REQUIRE(fits(m, k) && fits(n, n));
  const int64_t gpr = k / gs;
  const int64_t rb = i4 ? k / 2 : k;
  LP_REQUIRE(k % gs == 0);
  if (i4) LP_REQUIRE(k % 2 == 0);
  LP_REQUIRE(w_len == m * rb && ws_len == m * gpr && xq_len == n * k && xs_len == n * gpr &&
             y_len == m * n);
  if (bad(w, w_len) || bad(ws, ws_len) || bad(xq, xq_len) || bad(xs, xs_len) || bad(y, y_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  // A few columns: the GEMV skeleton with one term per (row, group, column),
  // one CTA per SM streaming its rows once (a 128-row tensor-core tile would
  // leave most SMs idle at this width).
  if (gs == 32 && n <= kGemmColsMax && m >= 1) {
    GemvParams p = base(w, ws, xq, xs, y, m, k, gs, gpr, rb);
    p.ncol = static_cast<int>(n);
    const int r = i4 ? lp::launch_gemv<lp::FmtI4Q8Cols>(p, SG(st))
                     : lp::launch_gemv<lp::FmtQ8Cols>(p, SG(st));
    if (r != LP_ERR_UNSUPPORTED) return r;
  }
  {
    const int r = lp::launch_gemm_tc(w, i4, ws, gs, xq, xs, n, y, m, k, S(st));
    if (r != LP_ERR_UNSUPPORTED) return r;
  }
  return lp::launch_gemm(static_cast<const uint8_t*>(w), i4, ws, gs, xq, xs, n, y, m, k, S(st));
}

int lp_dequant_gemm_q8(const int8_t* wq, int64_t wq_len, const float* w_scales,
                       int64_t w_scales_len, int64_t group_size, const int8_t* xq, int64_t xq_len,
                       const float* x_scales, int64_t x_scales_len, int64_t n, float* y,
                       int64_t y_len, lp_stream_t stream) {
  return gemm_common(0, wq, wq_len, w_scales, w_scales_len, group_size, xq, xq_len, x_scales,
                     x_scales_len, n, y, y_len, stream);
}
int lp_dequant_gemm_i4q8(const uint8_t* wp, int64_t wp_len, const float* w_scales,
                         int64_t w_scales_len, int64_t group_size, const int8_t* xq,
                         int64_t xq_len, const float* x_scales, int64_t x_scales_len, int64_t n,
                         float* y, int64_t y_len, lp_stream_t stream) {
  return gemm_common(1, wp, wp_len, w_scales, w_scales_len, group_size, xq, xq_len, x_scales,
                     x_scales_len, n, y, y_len, stream);
}

// ------------------------------------------ FP4 x FP4 block-scaled GEMMs

int lp_dequant_gemm_f4(const uint8_t* wp, int64_t wp_len, const float* w_scales,
                       int64_t w_scales_len, int64_t group_size, const uint8_t* xp,
                       int64_t xp_len, const float* x_scales, int64_t x_scales_len, int64_t n,
                       float* y, int64_t y_len, lp_stream_t stream) {
  LP_REQUIRE(n >= 1 && y_len >= 0 && xp_len >= 0 && y_len % n == 0 && xp_len % n == 0);
  const int64_t m = y_len / n, rb = xp_len / n, k = 2 * rb;
  LP_REQUIRE(group_size == 32 && k % 32 == 0 && fits(m, k) && fits(n, k));
  LP_REQUIRE(wp_len == m * rb && w_scales_len == m * (k / 32) && x_scales_len == n * (k / 32));
  if (bad(wp, wp_len) || bad(w_scales, w_scales_len) || bad(xp, xp_len) ||
      bad(x_scales, x_scales_len) || bad(y, y_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  if (m == 0) return LP_OK;
  if (k == 0) return lp::cuda_status(cudaMemsetAsync(y, 0, static_cast<size_t>(y_len) * 4, S(stream)));
  return lp::launch_gemm_mxf4(wp, w_scales, xp, x_scales, n, y, m, k, S(stream));
}

int lp_gemm_nvfp4(const uint8_t* wp, int64_t wp_len, const uint8_t* w_block_scales,
                  int64_t w_block_scales_len, const float* w_global_decode_scale,
                  const uint8_t* xp, int64_t xp_len, const uint8_t* x_block_scales,
                  int64_t x_block_scales_len, const float* x_global_decode_scale, int64_t n,
                  float* y, int64_t y_len, lp_stream_t stream) {
  LP_REQUIRE(n >= 1 && y_len >= 0 && xp_len >= 0 && y_len % n == 0 && xp_len % n == 0);
  const int64_t m = y_len / n, rb = xp_len / n, k = 2 * rb;
  LP_REQUIRE(k % 32 == 0 && fits(m, k) && fits(n, k));
  LP_REQUIRE(wp_len == m * rb && w_block_scales_len == m * (k / 16) &&
             x_block_scales_len == n * (k / 16));
  if (bad(wp, wp_len) || bad(w_block_scales, w_block_scales_len) || bad(xp, xp_len) ||
      bad(x_block_scales, x_block_scales_len) || bad(y, y_len) || !w_global_decode_scale ||
      !x_global_decode_scale)
    return LP_ERR_ARG;
  LP_VALIDATED();
  if (m == 0) return LP_OK;
  if (k == 0) return lp::cuda_status(cudaMemsetAsync(y, 0, static_cast<size_t>(y_len) * 4, S(stream)));
  return lp::launch_gemm_nvf4(wp, w_block_scales, w_global_decode_scale, xp, x_block_scales,
                              x_global_decode_scale, n, y, m, k, S(stream));
}

// -------------------------------------------------------------- encoders

int lp_quantize_q8_0_batch(const float* src, int64_t src_len, void* blocks, int64_t blocks_len,
                           lp_stream_t stream) {
  LP_REQUIRE(src_len >= 0 && src_len == blocks_len * 32);
  if (bad(src, src_len) || bad(blocks, blocks_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_q8_0(src, src_len, static_cast<uint8_t*>(blocks), nullptr, nullptr,
                                  S(stream));
}

int lp_quantize_q4_0_batch(const float* src, int64_t src_len, void* blocks, int64_t blocks_len,
                           lp_stream_t stream) {
  LP_REQUIRE(src_len >= 0 && src_len == blocks_len * 32);
  if (bad(src, src_len) || bad(blocks, blocks_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_q4_0(src, src_len, static_cast<uint8_t*>(blocks), S(stream));
}

int lp_quantize_q8_0_split(const float* src, int64_t src_len, int8_t* qs, int64_t qs_len,
                           float* d, int64_t d_len, lp_stream_t stream) {
  LP_REQUIRE(src_len >= 0 && src_len % 32 == 0 && qs_len == src_len && d_len == src_len / 32);
  if (bad(src, src_len) || bad(qs, qs_len) || bad(d, d_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_q8_0(src, src_len, nullptr, qs, d, S(stream));
}

static int64_t num_groups(int64_t n, int64_t gs) { return gs > 0 ? (n + gs - 1) / gs : 1; }

int lp_quantize_batch(const float* x, int64_t x_len, const float* scales, int64_t scales_len,
                      const float* zero_points, int64_t zero_points_len, int64_t group_size,
                      int8_t* dst, int64_t dst_len, lp_stream_t stream) {
  const int64_t groups = x_len ? num_groups(x_len, group_size) : 0;
  LP_REQUIRE(x_len >= 0 && x_len == dst_len);
  LP_REQUIRE(scales_len >= groups);
  LP_REQUIRE(zero_points_len == 0 || zero_points_len >= groups);
  if (bad(x, x_len) || bad(scales, scales_len) || bad(zero_points, zero_points_len) ||
      bad(dst, dst_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_batch(x, x_len, scales, zero_points_len ? zero_points : nullptr,
                                   group_size > 0 ? group_size : 0, dst, S(stream));
}

int lp_dequantize_batch(const int8_t* q, int64_t q_len, const float* scales, int64_t scales_len,
                        const float* zero_points, int64_t zero_points_len, int64_t group_size,
                        float* dst, int64_t dst_len, lp_stream_t stream) {
  const int64_t groups = q_len ? num_groups(q_len, group_size) : 0;
  LP_REQUIRE(q_len >= 0 && q_len == dst_len && scales_len >= groups);
  LP_REQUIRE(zero_points_len == 0 || zero_points_len >= groups);
  if (bad(q, q_len) || bad(scales, scales_len) || bad(dst, dst_len) ||
      bad(zero_points, zero_points_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_batch(q, q_len, scales, zero_points_len ? zero_points : nullptr,
                                     group_size > 0 ? group_size : 0, dst, S(stream));
}

int lp_calibrate_symmetric(const float* x, int64_t x_len, int64_t group_size, float qmax,
                           float* scales, int64_t scales_len, lp_stream_t stream) {
  LP_REQUIRE(x_len >= 0);
  const int64_t gs = group_size > 0 ? group_size : std::max<int64_t>(x_len, 1);
  LP_REQUIRE(scales_len == num_groups(x_len, gs) || (group_size <= 0 && scales_len == 1));
  if (bad(x, x_len) || bad(scales, scales_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_calibrate(x, x_len, gs, qmax, 0, 0, scales, scales_len, S(stream));
}

int lp_calibrate_mx(const float* x, int64_t x_len, int64_t block_size, int32_t elem_emax,
                    float* scales, int64_t scales_len, lp_stream_t stream) {
  LP_REQUIRE(x_len >= 0 && block_size > 0 && scales_len == num_groups(x_len, block_size));
  if (bad(x, x_len) || bad(scales, scales_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_calibrate(x, x_len, block_size, 0.0f, elem_emax, 1, scales, scales_len,
                              S(stream));
}

int lp_quantize_i4_packed(const float* x, int64_t x_len, const float* scales, int64_t scales_len,
                          int64_t group_size, uint8_t* packed, int64_t packed_len,
                          lp_stream_t stream) {
  LP_REQUIRE(x_len >= 0 && packed_len == (x_len + 1) / 2);
  LP_REQUIRE(scales_len >= (x_len ? num_groups(x_len, group_size) : 0));
  if (bad(x, x_len) || bad(scales, scales_len) || bad(packed, packed_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_packed(x, x_len, scales, group_size > 0 ? group_size : 0, 0, packed,
                                    S(stream));
}

int lp_quantize_f4_packed(const float* x, int64_t x_len, const float* scales, int64_t scales_len,
                          int64_t block_size, uint8_t* packed, int64_t packed_len,
                          lp_stream_t stream) {
  LP_REQUIRE(x_len >= 0 && packed_len == (x_len + 1) / 2);
  LP_REQUIRE(scales_len >= (x_len ? num_groups(x_len, block_size) : 0));
  if (bad(x, x_len) || bad(scales, scales_len) || bad(packed, packed_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_packed(x, x_len, scales, block_size > 0 ? block_size : 0, 1, packed,
                                    S(stream));
}

int lp_dequantize_q8_0_batch(const void* blocks, int64_t blocks_len, float* dst, int64_t dst_len,
                             lp_stream_t stream) {
  LP_REQUIRE(blocks_len >= 0 && dst_len == blocks_len * 32);
  if (bad(blocks, blocks_len) || bad(dst, dst_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_blocks(static_cast<const uint8_t*>(blocks), blocks_len, 0, dst,
                                      S(stream));
}

int lp_dequantize_q4_0_batch(const void* blocks, int64_t blocks_len, float* dst, int64_t dst_len,
                             lp_stream_t stream) {
  LP_REQUIRE(blocks_len >= 0 && dst_len == blocks_len * 32);
  if (bad(blocks, blocks_len) || bad(dst, dst_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_blocks(static_cast<const uint8_t*>(blocks), blocks_len, 1, dst,
                                      S(stream));
}

int lp_dequantize_q4_k(const void* blocks, int64_t blocks_len, float* dst, int64_t dst_len,
                       lp_stream_t stream) {
  LP_REQUIRE(blocks_len >= 0 && dst_len == blocks_len * 256);
  if (bad(blocks, blocks_len) || bad(dst, dst_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_kquant(static_cast<const uint8_t*>(blocks), blocks_len, 0, dst,
                                      S(stream));
}

int lp_dequantize_q6_k(const void* blocks, int64_t blocks_len, float* dst, int64_t dst_len,
                       lp_stream_t stream) {
  LP_REQUIRE(blocks_len >= 0 && dst_len == blocks_len * 256);
  if (bad(blocks, blocks_len) || bad(dst, dst_len)) return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_kquant(static_cast<const uint8_t*>(blocks), blocks_len, 1, dst,
                                      S(stream));
}

int lp_quantize_nvfp4(const float* x, int64_t x_len, uint8_t* codes, int64_t codes_len,
                      uint8_t* block_scales, int64_t scales_len, float* global_decode_scale,
                      lp_stream_t stream) {
  LP_REQUIRE(x_len >= 0 && x_len % 16 == 0 && codes_len == x_len && scales_len == x_len / 16);
  if (bad(x, x_len) || bad(codes, codes_len) || bad(block_scales, scales_len) ||
      !global_decode_scale)
    return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_quantize_nvfp4(x, x_len, codes, block_scales, global_decode_scale, S(stream));
}

int lp_dequantize_nvfp4(const uint8_t* codes, int64_t codes_len, const uint8_t* block_scales,
                        int64_t scales_len, float global_decode_scale, float* dst,
                        int64_t dst_len, lp_stream_t stream) {
  LP_REQUIRE(dst_len == codes_len && scales_len * 16 == codes_len && codes_len >= 0);
  if (bad(codes, codes_len) || bad(block_scales, scales_len) || bad(dst, dst_len))
    return LP_ERR_ARG;
  LP_VALIDATED();
  return lp::launch_dequantize_nvfp4(codes, block_scales, global_decode_scale, codes_len, dst,
                                     S(stream));
}

}  // extern "C"

// ================================================== host-staging forms ==
namespace {

// One per calling thread: a device workspace grown on demand, reused across
// calls, and a private stream.
struct HostStage {
  int device = -1;
  void* buf = nullptr;
  size_t cap = 0;
  cudaStream_t stream = nullptr;
  ~HostStage() {
    if (buf) cudaFree(buf);
    if (stream) cudaStreamDestroy(stream);
  }
};

thread_local HostStage t_stage;

struct Seg {
  const void* host;  // input to copy in (nullptr for outputs)
  size_t bytes;
  void* dev = nullptr;
};

// Lays the segments out in the workspace (256-byte aligned), copies inputs.
int stage_in(std::vector<Seg*> segs) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LP_ERR_NO_DEVICE;
  HostStage& hs = t_stage;
  if (hs.device != dev) {
    if (hs.buf) cudaFree(hs.buf);
    if (hs.stream) cudaStreamDestroy(hs.stream);
    hs.buf = nullptr;
    hs.cap = 0;
    hs.stream = nullptr;
    hs.device = dev;
    const cudaError_t e = cudaStreamCreateWithFlags(&hs.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return lp::cuda_status(e);
  }
  size_t total = 0;
  for (Seg* s : segs) total += (s->bytes + 255) & ~size_t(255);
  if (total > hs.cap) {
    if (hs.buf) cudaFree(hs.buf);
    hs.buf = nullptr;
    const size_t want = std::max(total, hs.cap * 2);
    if (cudaMalloc(&hs.buf, want) != cudaSuccess) {
      hs.cap = 0;
      return LP_ERR_CUDA;
    }
    hs.cap = want;
  }
  size_t off = 0;
  for (Seg* s : segs) {
    s->dev = static_cast<uint8_t*>(hs.buf) + off;
    off += (s->bytes + 255) & ~size_t(255);
    if (s->host && s->bytes &&
        cudaMemcpyAsync(s->dev, s->host, s->bytes, cudaMemcpyHostToDevice, hs.stream) != cudaSuccess)
      return LP_ERR_CUDA;
  }
  return LP_OK;
}

int stage_out(void* host, const Seg& s, int status) {
  HostStage& hs = t_stage;
  if (status == LP_OK && s.bytes &&
      cudaMemcpyAsync(host, s.dev, s.bytes, cudaMemcpyDeviceToHost, hs.stream) != cudaSuccess)
    status = LP_ERR_CUDA;
  if (cudaStreamSynchronize(hs.stream) != cudaSuccess && status == LP_OK) status = LP_ERR_CUDA;
  return status;
}

template <class T>
size_t nb(int64_t len) {
  return len > 0 ? static_cast<size_t>(len) * sizeof(T) : 0;
}

}  // namespace

// Runs `call` with the validate-only switch set; returns its status.
#define LPH_PRECHECK(call)                 \
  do {                                     \
    t_validate_only = true;                \
    const int pre_ = (call);               \
    t_validate_only = false;               \
    if (pre_ != LP_OK) return pre_;        \
  } while (0)

extern "C" {

#define LPH_GROUP_F32(NAME, DEVFN, WT)                                                           \
  int NAME(const WT* w, int64_t w_len, const float* scales, int64_t scales_len, int64_t gs,      \
           const float* x, int64_t x_len, float* y, int64_t y_len) {                             \
    Seg sw{w, nb<WT>(w_len)}, ss{scales, nb<float>(scales_len)}, sx{x, nb<float>(x_len)},        \
        sy{nullptr, nb<float>(y_len)};                                                            \
    LPH_PRECHECK(DEVFN(w, w_len, scales, scales_len, gs, x, x_len, y, y_len, nullptr));          \
    int st = stage_in({&sw, &ss, &sx, &sy});                                                     \
    if (st != LP_OK) return st;                                                                   \
    st = DEVFN(static_cast<const WT*>(sw.dev), w_len, static_cast<const float*>(ss.dev),         \
               scales_len, gs, static_cast<const float*>(sx.dev), x_len,                         \
               static_cast<float*>(sy.dev), y_len, t_stage.stream);                              \
    return stage_out(y, sy, st);                                                                  \
  }

LPH_GROUP_F32(lph_dequant_gemv, lp_dequant_gemv, int8_t)
LPH_GROUP_F32(lph_dequant_gemv_i4, lp_dequant_gemv_i4, uint8_t)
LPH_GROUP_F32(lph_dequant_gemv_f4, lp_dequant_gemv_f4, uint8_t)

#define LPH_BLOCKS_F32(NAME, DEVFN, BB)                                                          \
  int NAME(const void* w, int64_t w_len, int64_t bpr, const float* x, int64_t x_len, float* y,   \
           int64_t y_len) {                                                                      \
    Seg sw{w, w_len > 0 ? static_cast<size_t>(w_len) * BB : 0}, sx{x, nb<float>(x_len)},         \
        sy{nullptr, nb<float>(y_len)};                                                            \
    LPH_PRECHECK(DEVFN(w, w_len, bpr, x, x_len, y, y_len, nullptr));                             \
    int st = stage_in({&sw, &sx, &sy});                                                          \
    if (st != LP_OK) return st;                                                                   \
    st = DEVFN(sw.dev, w_len, bpr, static_cast<const float*>(sx.dev), x_len,                     \
               static_cast<float*>(sy.dev), y_len, t_stage.stream);                              \
    return stage_out(y, sy, st);                                                                  \
  }

LPH_BLOCKS_F32(lph_dequant_gemv_q8_0, lp_dequant_gemv_q8_0, 34)
LPH_BLOCKS_F32(lph_dequant_gemv_q4_0, lp_dequant_gemv_q4_0, 18)

#define LPH_GROUP_Q8(NAME, DEVFN, WT)                                                            \
  int NAME(const WT* w, int64_t w_len, const float* ws, int64_t ws_len, int64_t gs,              \
           const int8_t* xq, int64_t xq_len, const float* xs, int64_t xs_len, float* y,          \
           int64_t y_len) {                                                                      \
    Seg sw{w, nb<WT>(w_len)}, sws{ws, nb<float>(ws_len)}, sx{xq, nb<int8_t>(xq_len)},            \
        sxs{xs, nb<float>(xs_len)}, sy{nullptr, nb<float>(y_len)};                                \
    LPH_PRECHECK(DEVFN(w, w_len, ws, ws_len, gs, xq, xq_len, xs, xs_len, y, y_len, nullptr));    \
    int st = stage_in({&sw, &sws, &sx, &sxs, &sy});                                              \
    if (st != LP_OK) return st;                                                                   \
    st = DEVFN(static_cast<const WT*>(sw.dev), w_len, static_cast<const float*>(sws.dev), ws_len, \
               gs, static_cast<const int8_t*>(sx.dev), xq_len,                                   \
               static_cast<const float*>(sxs.dev), xs_len, static_cast<float*>(sy.dev), y_len,   \
               t_stage.stream);                                                                  \
    return stage_out(y, sy, st);                                                                  \
  }

LPH_GROUP_Q8(lph_dequant_gemv_q8, lp_dequant_gemv_q8, int8_t)
LPH_GROUP_Q8(lph_dequant_gemv_i4q8, lp_dequant_gemv_i4q8, uint8_t)

#define LPH_BLOCKS_Q8(NAME, DEVFN, BB)                                                           \
  int NAME(const void* w, int64_t w_len, int64_t bpr, const void* xq, int64_t xq_len, float* y,  \
           int64_t y_len) {                                                                      \
    Seg sw{w, w_len > 0 ? static_cast<size_t>(w_len) * BB : 0},                                  \
        sx{xq, xq_len > 0 ? static_cast<size_t>(xq_len) * 34 : 0},                               \
        sy{nullptr, nb<float>(y_len)};                                                            \
    LPH_PRECHECK(DEVFN(w, w_len, bpr, xq, xq_len, y, y_len, nullptr));                           \
    int st = stage_in({&sw, &sx, &sy});                                                          \
    if (st != LP_OK) return st;                                                                   \
    st = DEVFN(sw.dev, w_len, bpr, sx.dev, xq_len, static_cast<float*>(sy.dev), y_len,           \
               t_stage.stream);                                                                  \
    return stage_out(y, sy, st);                                                                  \
  }

LPH_BLOCKS_Q8(lph_dequant_gemv_q8_0q8, lp_dequant_gemv_q8_0q8, 34)
LPH_BLOCKS_Q8(lph_dequant_gemv_q4_0q8, lp_dequant_gemv_q4_0q8, 18)

#define LPH_GEMM(NAME, DEVFN, WT)                                                                \
  int NAME(const WT* w, int64_t w_len, const float* ws, int64_t ws_len, int64_t gs,              \
           const int8_t* xq, int64_t xq_len, const float* xs, int64_t xs_len, int64_t n,         \
           float* y, int64_t y_len) {                                                            \
    Seg sw{w, nb<WT>(w_len)}, sws{ws, nb<float>(ws_len)}, sx{xq, nb<int8_t>(xq_len)},            \
        sxs{xs, nb<float>(xs_len)}, sy{nullptr, nb<float>(y_len)};                                \
    LPH_PRECHECK(DEVFN(w, w_len, ws, ws_len, gs, xq, xq_len, xs, xs_len, n, y, y_len, nullptr)); \
    int st = stage_in({&sw, &sws, &sx, &sxs, &sy});                                              \
    if (st != LP_OK) return st;                                                                   \
    st = DEVFN(static_cast<const WT*>(sw.dev), w_len, static_cast<const float*>(sws.dev), ws_len, \
               gs, static_cast<const int8_t*>(sx.dev), xq_len,                                   \
               static_cast<const float*>(sxs.dev), xs_len, n, static_cast<float*>(sy.dev),       \
               y_len, t_stage.stream);                                                           \
    return stage_out(y, sy, st);                                                                  \
  }

LPH_GEMM(lph_dequant_gemm_q8, lp_dequant_gemm_q8, int8_t)
LPH_GEMM(lph_dequant_gemm_i4q8, lp_dequant_gemm_i4q8, uint8_t)

int lph_quantize_q8_0_batch(const float* src, int64_t src_len, void* blocks, int64_t blocks_len) {
  Seg ss{src, nb<float>(src_len)}, sb{nullptr, blocks_len > 0 ? static_cast<size_t>(blocks_len) * 34 : 0};
  LPH_PRECHECK(lp_quantize_q8_0_batch(src, src_len, blocks, blocks_len, nullptr));
  int st = stage_in({&ss, &sb});
  if (st != LP_OK) return st;
  st = lp_quantize_q8_0_batch(static_cast<const float*>(ss.dev), src_len, sb.dev, blocks_len,
                              t_stage.stream);
  return stage_out(blocks, sb, st);
}

int lph_quantize_q4_0_batch(const float* src, int64_t src_len, void* blocks, int64_t blocks_len) {
  Seg ss{src, nb<float>(src_len)}, sb{nullptr, blocks_len > 0 ? static_cast<size_t>(blocks_len) * 18 : 0};
  LPH_PRECHECK(lp_quantize_q4_0_batch(src, src_len, blocks, blocks_len, nullptr));
  int st = stage_in({&ss, &sb});
  if (st != LP_OK) return st;
  st = lp_quantize_q4_0_batch(static_cast<const float*>(ss.dev), src_len, sb.dev, blocks_len,
                              t_stage.stream);
  return stage_out(blocks, sb, st);
}

int lph_quantize_batch(const float* x, int64_t x_len, const float* scales, int64_t scales_len,
                       const float* zero_points, int64_t zero_points_len, int64_t group_size,
                       int8_t* dst, int64_t dst_len) {
  Seg sx{x, nb<float>(x_len)}, ss{scales, nb<float>(scales_len)},
      sz{zero_points, nb<float>(zero_points_len)}, sd{nullptr, nb<int8_t>(dst_len)};
  LPH_PRECHECK(lp_quantize_batch(x, x_len, scales, scales_len, zero_points, zero_points_len,
                                 group_size, dst, dst_len, nullptr));
  int st = stage_in({&sx, &ss, &sz, &sd});
  if (st != LP_OK) return st;
  st = lp_quantize_batch(static_cast<const float*>(sx.dev), x_len,
                         static_cast<const float*>(ss.dev), scales_len,
                         static_cast<const float*>(sz.dev), zero_points_len, group_size,
                         static_cast<int8_t*>(sd.dev), dst_len, t_stage.stream);
  return stage_out(dst, sd, st);
}

int lph_dequantize_batch(const int8_t* q, int64_t q_len, const float* scales, int64_t scales_len,
                         const float* zero_points, int64_t zero_points_len, int64_t group_size,
                         float* dst, int64_t dst_len) {
  Seg sq{q, nb<int8_t>(q_len)}, ss{scales, nb<float>(scales_len)},
      sz{zero_points, nb<float>(zero_points_len)}, sd{nullptr, nb<float>(dst_len)};
  LPH_PRECHECK(lp_dequantize_batch(q, q_len, scales, scales_len, zero_points, zero_points_len,
                                   group_size, dst, dst_len, nullptr));
  int st = stage_in({&sq, &ss, &sz, &sd});
  if (st != LP_OK) return st;
  st = lp_dequantize_batch(static_cast<const int8_t*>(sq.dev), q_len,
                           static_cast<const float*>(ss.dev), scales_len,
                           static_cast<const float*>(sz.dev), zero_points_len, group_size,
                           static_cast<float*>(sd.dev), dst_len, t_stage.stream);
  return stage_out(dst, sd, st);
}

}  // extern "C"
