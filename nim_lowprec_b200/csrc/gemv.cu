// gemv.cu -- launch planning for the fused dequant-GEMV kernels.
#include <algorithm>
#include <mutex>

#include "gemv_formats.cuh"
#include "lp_internal.h"

namespace lp {

// The error word of this translation unit (see lp_device.cuh).
unsigned int take_error_gemv() {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return LP_ERR_CUDA;
  if (v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
  }
  return v;
}

namespace {

constexpr int kNcw = 8;                 // consumer warps per CTA
constexpr int kStageTarget = 32 * 1024; // bytes of weights+scales per stage
constexpr int kMaxStages = 8;
constexpr int kRtCap = 8;

template <class Fmt>
int x_stage_bytes(const GemvParams& p);
template <>
int x_stage_bytes<FmtI8>(const GemvParams& p) { return p.k * 4; }
template <>
int x_stage_bytes<FmtI4>(const GemvParams& p) { return p.k * 4; }
template <>
int x_stage_bytes<FmtF4>(const GemvParams& p) { return p.k * 4; }
template <>
int x_stage_bytes<FmtQ8_0>(const GemvParams& p) { return p.k * 4; }
template <>
int x_stage_bytes<FmtQ4_0>(const GemvParams& p) { return p.k * 4; }
template <>
int x_stage_bytes<FmtQ8>(const GemvParams& p) { return ((p.k + 15) & ~15) + p.gpr * 4; }
template <>
int x_stage_bytes<FmtI4Q8>(const GemvParams& p) { return ((p.k + 15) & ~15) + p.gpr * 4; }
template <>
int x_stage_bytes<FmtQ8_0Q8>(const GemvParams& p) { return ((p.k + 15) & ~15) + p.gpr * 4; }
template <>
int x_stage_bytes<FmtQ4_0Q8>(const GemvParams& p) { return ((p.k + 15) & ~15) + p.gpr * 4; }

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

}  // namespace

template <class Fmt>
int launch_gemv(GemvParams p, cudaStream_t st) {
  if (p.m == 0) return LP_OK;
  if (p.gpr == 0)  // no groups: every row is the empty fold, 0.0
    return cuda_status(cudaMemsetAsync(p.y, 0, static_cast<size_t>(p.m) * sizeof(float), st));
  const DeviceInfo& di = device_info();
  auto kern = gemv_kernel<Fmt, kNcw>;
  // Dynamic shared memory may use the opt-in maximum minus the kernel's
  // static shared memory; set once per device.
  static int dyn_max[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  const int slot = di.ordinal % kMaxDevices;
  std::call_once(once[slot], [&] {
    cudaFuncAttributes fa;
    int lim = di.max_smem_optin;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) lim -= static_cast<int>(fa.sharedSizeBytes);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess)
      lim = 48 * 1024 - 256;
    dyn_max[slot] = lim;
  });
  const int row_total = p.row_bytes + (Fmt::kScales ? p.gpr * 4 : 0);
  p.rt = std::max(1, std::min({kRtCap, kStageTarget / std::max(row_total, 1), p.m}));
  p.x_bytes = round_up(x_stage_bytes<Fmt>(p), 16);
  p.stage_w_bytes = round_up(p.rt * p.row_bytes, 16);
  p.stage_s_bytes = Fmt::kScales ? round_up(p.rt * p.gpr * 4, 16) : 0;
  p.tstride = round_up(std::max(p.gpr, 1), 32) + 4;
  const int terms_bytes = 2 * p.rt * p.tstride * 4;
  const int fixed = round_up(p.x_bytes, 128) + terms_bytes + 16 + 8 * (2 * kMaxStages + 4);
  // Two CTAs per SM when they fit (twice the consumer warps to hide the
  // fp32 chains' latency), else one.
  const int two_cta = (dyn_max[slot] - 1024) / 2 - 1024;
  int budget = dyn_max[slot];
  if (fixed + 2 * (p.stage_w_bytes + p.stage_s_bytes) <= two_cta) budget = two_cta;
  const int per_stage = p.stage_w_bytes + p.stage_s_bytes;
  p.stages = std::min(kMaxStages, (budget - fixed) / std::max(per_stage, 1));
  if (p.stages < 2) return LP_ERR_UNSUPPORTED;  // activations or rows too large for shared
  const uintptr_t wa = reinterpret_cast<uintptr_t>(p.w);
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.ws);
  p.bulk = (p.row_bytes % 16 == 0) && (wa % 16 == 0) &&
           (!Fmt::kScales || ((p.gpr % 4 == 0) && (sa % 16 == 0)));
  p.off_w = round_up(p.x_bytes, 128);
  p.off_s = p.off_w + p.stages * p.stage_w_bytes;
  p.off_t = p.off_s + p.stages * p.stage_s_bytes;
  p.off_b = round_up(p.off_t + terms_bytes, 16);
  const int smem = p.off_b + 8 * (2 * p.stages + 4);
  const int ctas_per_sm = budget < dyn_max[slot] ? 2 : 1;
  const int grid = std::min(p.m, di.sm_count * ctas_per_sm);
  // Programmatic dependent launch: this grid may start while the previous
  // kernel in the stream drains; it prefetches its weights at once and waits
  // for that kernel (griddepcontrol.wait) before it reads x or writes y.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 * (kNcw + 2));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p));
}

template int launch_gemv<FmtI8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4>(GemvParams, cudaStream_t);
template int launch_gemv<FmtF4>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8_0>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ4_0>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4Q8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8_0Q8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ4_0Q8>(GemvParams, cudaStream_t);

}  // namespace lp
