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

constexpr int kNcw = 16;         // consumer warps per CTA (512 threads)
constexpr int kMaxStages = 12;

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

// A 2-D row-major tensor map: `inner` elements per row, `rows` rows, row
// pitch `pitch` bytes, box `bi` x `br`.  Encoding is a host-side computation.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
               int64_t inner, int64_t rows, int64_t pitch, int bi, int br) {
  if (bi <= 0 || bi > 256 || br <= 0 || br > 256 || (static_cast<int64_t>(bi) * esize) % 16) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(bi), static_cast<cuuint32_t>(br)};
  const cuuint32_t estr[2] = {1, 1};
  // Resolved through the runtime, so the library has no link-time
  // dependency on the driver library (it loads on machines without a GPU).
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<EncodeFn>(fn);
  }();
  if (!encode) return false;
  return encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

template <class Fmt>
int launch_gemv(GemvParams p, cudaStream_t st) {
  if (p.m == 0) return LP_OK;
  if (p.gpr == 0)  // no groups: every row is the empty fold, 0.0
    return cuda_status(cudaMemsetAsync(p.y, 0, static_cast<size_t>(p.m) * sizeof(float), st));
  const DeviceInfo& di = device_info();
  auto kern = gemv_kernel<Fmt, kNcw>;
  // Dynamic shared memory may use the opt-in maximum minus the kernel's
  // static shared memory; set once per device.  Rows per CTA beyond
  // kMaxRowsPerPass are processed in several passes.
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
  constexpr int NC = kNcw * 32;
  const int gbytes = p.row_bytes / p.gpr + (Fmt::kScales ? 4 : 0);  // per group, rounded down
  // Chunk width: a stage is SR x G groups with SR * G = 2 * NC, i.e. one
  // row pair per consumer thread; narrower when a row has fewer groups.
  p.G = std::min(gbytes <= 24 ? 64 : 32, round_up(p.gpr, 4));
  p.SR = std::min(32, 2 * NC / p.G);    // rows per stage (one producer lane each)
  const int rows_per_cta = (p.m + std::min(p.m, di.sm_count) - 1) / std::min(p.m, di.sm_count);
  p.RP = std::min(kMaxRowsPerPass, rows_per_cta);
  p.tstride = p.G + 4;
  const int64_t slice = static_cast<int64_t>(p.G) * p.row_bytes / p.gpr;
  // Shared row pitch: 128-byte multiple, so every TMA destination (a whole
  // stage or one row of it) is 128-byte aligned; the boxes are this wide.
  p.slice_pitch = round_up(static_cast<int>(slice), 128);
  p.x_bytes = round_up(x_stage_bytes<Fmt>(p), 16);
  p.stage_w_bytes = p.SR * p.slice_pitch;
  p.spitch = round_up(p.G * 4, 128) / 4;  // scale rows: 128-byte pitch, as wide a box
  p.stage_s_bytes = Fmt::kScales ? p.SR * p.spitch * 4 : 0;
  const int terms_bytes = 2 * p.RP * p.tstride * 4;
  const int fixed = 128 + round_up(p.x_bytes, 128) + terms_bytes + 16 + 8 * (2 * kMaxStages + 4);
  const int per_stage = p.stage_w_bytes + p.stage_s_bytes;
  // All the shared memory goes to stages: the weight stream needs about a
  // microsecond of HBM bandwidth per SM in flight.
  const int budget = dyn_max[slot];
  p.stages = std::min(kMaxStages, (budget - fixed) / per_stage);
  if (p.stages < 2) return LP_ERR_UNSUPPORTED;  // activations too large for shared memory
  // Bulk copies need 16-byte aligned row slices of weights and scales.
  const uintptr_t wa = reinterpret_cast<uintptr_t>(p.w);
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.ws);
  p.bulk = (p.row_bytes % 16 == 0) && (slice % 16 == 0) && (p.slice_pitch / 8 <= 256) &&
           (wa % 16 == 0) && (!Fmt::kScales || ((p.gpr % 4 == 0) && (sa % 16 == 0)));
  if (p.bulk) {
    const bool ok =
        encode_2d(&p.tw_full, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, p.w, p.row_bytes / 8, p.m,
                  p.row_bytes, p.slice_pitch / 8, p.SR) &&
        encode_2d(&p.tw_row, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, p.w, p.row_bytes / 8, p.m,
                  p.row_bytes, p.slice_pitch / 8, 1) &&
        (!Fmt::kScales ||
         (encode_2d(&p.ts_full, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.ws, p.gpr, p.m, p.gpr * 4,
                    p.spitch, p.SR) &&
          encode_2d(&p.ts_row, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.ws, p.gpr, p.m, p.gpr * 4,
                    p.spitch, 1)));
    if (!ok) p.bulk = 0;
  }
  p.off_w = round_up(p.x_bytes, 128);
  p.off_s = p.off_w + p.stages * p.stage_w_bytes;
  p.off_t = p.off_s + p.stages * p.stage_s_bytes;
  p.off_b = round_up(p.off_t + terms_bytes, 16);
  const int smem = 128 + p.off_b + 8 * (2 * p.stages + 4);  // + base alignment slack
  const int grid = std::min(p.m, di.sm_count);
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
