// transfer.cu -- per-step inputs from page-locked host memory into device
// memory as a kernel of the stream (no counterpart in the reference).
//
// A decode loop feeds each GEMV a fresh activation vector from the host.  A
// copy-engine copy of a few KB costs several microseconds in a CUDA graph and
// cannot overlap the kernel before it; this kernel reads the source (the
// device address of page-locked memory) before its grid-dependency wait, so
// the host-link latency overlaps the previous kernel's tail, then waits for
// that kernel (which may still read the old contents of dst), stores, and
// lets the next launch (programmatic dependent launch) start streaming its
// weights at once.  The source must not be written by the previous kernel.
#include <algorithm>

#include "lp_device.cuh"
#include "lp_internal.h"

namespace lp {
namespace {

constexpr int kCopyThreads = 256;
constexpr int kMaxCopyCtas = 64;

// 16-byte units when src, dst and bytes allow, else bytes; each thread keeps
// its units in registers across the wait.
template <bool kVec>
__global__ void __launch_bounds__(kCopyThreads) k_copy_in(uint8_t* __restrict__ dst,
                                                          const uint8_t* __restrict__ src,
                                                          int64_t bytes) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  constexpr int kPer = 4;  // units held per thread before the wait
  if (kVec) {
    const int64_t n = bytes / 16;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int64_t base = 0; base < n; base += kPer * nthr) {
      uint4 v[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = base + k * nthr + tid;
        if (i < n) v[k] = s[i];
      }
      if (base == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = base + k * nthr + tid;
        if (i < n) d[i] = v[k];
      }
    }
    if (n == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int64_t i = tid; i < bytes; i += nthr) dst[i] = src[i];
  }
}

}  // namespace

int launch_copy_in(void* dst, const void* src, int64_t bytes, cudaStream_t st) {
  if (bytes == 0) return LP_OK;
  const bool vec =
      ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0;
  const int64_t units = vec ? bytes / 16 : bytes;
  const int grid = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(kMaxCopyCtas, (units + 4 * kCopyThreads - 1) /
                                                               (4 * kCopyThreads))));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kCopyThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  uint8_t* d = static_cast<uint8_t*>(dst);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  return cuda_status(vec ? cudaLaunchKernelEx(&cfg, k_copy_in<true>, d, s, bytes)
                         : cudaLaunchKernelEx(&cfg, k_copy_in<false>, d, s, bytes));
}

}  // namespace lp
