// static_stage.cu -- a host form of dequantGemvQ4_0 that allocates nothing.
//
// Who needs it: code that may not allocate device memory while it runs -- a
// real-time or audio callback, a signal-safe path, a host with its memory
// budget fixed up front, or an embedding that forbids cudaMalloc after
// start-up (a cudaMalloc can synchronise the device and take unbounded time).
// lph_dequant_gemv_q4_0 stages its inputs and output through a per-thread
// device workspace that grows with cudaMalloc; this form stages them in one
// statically sized __device__ array instead, so a call performs no allocation
// at all, and it rejects calls whose staged bytes exceed the array.
//
// The array lives in every GPU that loads this library, for the life of the
// process (32 MiB each).  It is shared by every caller: calls that overlap
// in time (other threads, other streams) race on it and must be serialised by
// the caller.  Nothing in it has to start at zero: the kernel writes every
// element of y, and the inputs are copied in before the kernel runs.
//
// Set-up: the array's device address is looked up with cudaGetSymbolAddress
// on the first call on each device (with that device current) and cached; a
// failed lookup is not cached, so the next call tries again.  The cached
// address is invalid after cudaDeviceReset on that device.  Make the first
// call on a device before any stream capture.
#include <mutex>

#include "lp_internal.h"

namespace {

constexpr size_t kStaticStageBytes = size_t{32} << 20;  // 32 MiB: config 1 stages 25.4 MB

__device__ __align__(256) uint8_t g_static_stage[kStaticStageBytes];

// The array's device address on the current device (nullptr on failure).
uint8_t* static_stage() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= lp::kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  static uint8_t* base[lp::kMaxDevices];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_stage) == cudaSuccess)
      base[dev] = static_cast<uint8_t*>(p);
    else
      cudaGetLastError();  // not cached: the next call looks it up again
  }
  return base[dev];
}

inline size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

extern "C" {

int lph_dequant_gemv_q4_0_static(const void* w, int64_t w_len, int64_t blocks_per_row,
                                 const float* x, int64_t x_len, float* y, int64_t y_len) {
  // the device form's shape and argument checks, before anything is copied
  lp::set_validate_only(true);
  const int pre = lp_dequant_gemv_q4_0(w, w_len, blocks_per_row, x, x_len, y, y_len, nullptr);
  lp::set_validate_only(false);
  if (pre != LP_OK) return pre;
  const size_t wb = static_cast<size_t>(w_len) * 18, xb = static_cast<size_t>(x_len) * 4,
               yb = static_cast<size_t>(y_len) * 4;
  if (up256(wb) + up256(xb) + up256(yb) > kStaticStageBytes) {
    lp::note_text("staged bytes exceed the static stage (32 MiB)");
    return LP_ERR_UNSUPPORTED;
  }
  uint8_t* base = static_stage();
  if (!base) {
    lp::note_text("cudaGetSymbolAddress of the static stage failed");
    return LP_ERR_CUDA;
  }
  uint8_t* dw = base;
  float* dx = reinterpret_cast<float*>(base + up256(wb));
  float* dy = reinterpret_cast<float*>(base + up256(wb) + up256(xb));
  if (wb && cudaMemcpy(dw, w, wb, cudaMemcpyHostToDevice) != cudaSuccess) return LP_ERR_CUDA;
  if (xb && cudaMemcpy(dx, x, xb, cudaMemcpyHostToDevice) != cudaSuccess) return LP_ERR_CUDA;
  const int st = lp_dequant_gemv_q4_0(dw, w_len, blocks_per_row, dx, x_len, dy, y_len, nullptr);
  if (st != LP_OK) return st;
  // a copy on the legacy default stream follows the kernel and blocks
  if (yb && cudaMemcpy(y, dy, yb, cudaMemcpyDeviceToHost) != cudaSuccess) return LP_ERR_CUDA;
  return LP_OK;
}

}  // extern "C"
