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
constexpr int kTileBytes = 96 * 1024;  // weights + scales of one tile, at most
// Weight bytes in flight per CTA, at most (but at least two stages): the
// copies in flight share the SM's part of the HBM stream, so more of them
// only delay the first tile the consumers wait for (config 1: two 58 KB
// stages 9.6 us, three 10.2 us).
constexpr int kFlightBytes = 128 * 1024;
// Term-matrix bytes of two ordered-fold passes, at most.
constexpr int kFoldBytes = 100 * 1024;

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Shared bytes of the staged activations.
template <class Fmt>
int x_stage_bytes(const GemvParams& p);
inline int f32_bytes(const GemvParams& p) { return round_up(p.k, 32) * 4; }  // swizzled blocks
inline int q8_bytes(const GemvParams& p) { return round_up(p.k, 16) + p.gpr * 4; }
inline int planes_bytes(const GemvParams& p) { return 3 * round_up(p.k, 16) + 16 * p.gpr; }
template <> int x_stage_bytes<FmtI8>(const GemvParams& p) { return f32_bytes(p); }
template <> int x_stage_bytes<FmtI4>(const GemvParams& p) { return f32_bytes(p); }
template <> int x_stage_bytes<FmtF4>(const GemvParams& p) { return f32_bytes(p); }
template <> int x_stage_bytes<FmtQ8_0>(const GemvParams& p) { return f32_bytes(p); }
template <> int x_stage_bytes<FmtQ4_0>(const GemvParams& p) { return f32_bytes(p); }
template <> int x_stage_bytes<FmtI8F>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtI4F>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtF4F>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtQ8_0F>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtQ4_0F>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtQ4_KF>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtQ6_KF>(const GemvParams& p) { return planes_bytes(p); }
template <> int x_stage_bytes<FmtQ8>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtI4Q8>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtQ8_0Q8>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtQ4_0Q8>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtQ8FromF32>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtI4Q8FromF32>(const GemvParams& p) { return q8_bytes(p); }
template <> int x_stage_bytes<FmtQ8Cols>(const GemvParams& p) {
  return round_up(p.k * p.ncol, 16) + 4 * p.gpr * p.ncol;
}
template <> int x_stage_bytes<FmtI4Q8Cols>(const GemvParams& p) {
  return round_up(p.k * p.ncol, 16) + 8 * p.gpr * p.ncol;  // xs, then 8 * sum(x)
}

struct SmemLimits {
  int one = 0;  // dynamic shared bytes one CTA may use
};

}  // namespace

thread_local const PushCtx* g_push = nullptr;
thread_local int64_t g_push_off = 0;
thread_local bool g_pushed = false;

template <class Fmt>
int launch_gemv(GemvParams p, cudaStream_t st) {
  if (p.m == 0) {
    g_pushed = g_push != nullptr;  // an empty slice has nothing to send
    return LP_OK;
  }
  if (p.gpr == 0)  // no groups: every row is the empty fold, 0.0
    return cuda_status(cudaMemsetAsync(p.y, 0, static_cast<size_t>(p.m) * sizeof(float), st));
  const DeviceInfo& di = device_info();
  auto kern = gemv_kernel<Fmt, kNcw>;
  // Dynamic shared memory may use the opt-in maximum minus the kernel's
  // static shared memory; set once per device.
  static SmemLimits lim[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  const int slot = di.ordinal % kMaxDevices;
  std::call_once(once[slot], [&] {
    cudaFuncAttributes fa;
    int st_bytes = 0;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) st_bytes = static_cast<int>(fa.sharedSizeBytes);
    int one = di.max_smem_optin - st_bytes;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, one) != cudaSuccess)
      one = 48 * 1024 - 256;
    lim[slot].one = one;
  });
  constexpr int NC = kNcw * 32;
  constexpr bool kCols = ColsOf<Fmt>::value;
  const int vr = kCols ? p.ncol : 1;  // virtual rows per weight row
  const int row_total = p.row_bytes + (Fmt::kScales ? p.gpr * 4 : 0);
  if constexpr (kCols) {
    // Tile height: enough (row pair, group) units for every consumer
    // thread (one pair per thread at gpr = 128), at most 40 KB of weights +
    // scales and 64 virtual rows (rt * ncol, folded 32 at a time).
    if (p.ncol < 1 || p.ncol > 64) return LP_ERR_UNSUPPORTED;
    int rt = std::max(2, std::min(64 / p.ncol, (2 * NC) / std::max(p.gpr, 1)));
    rt = std::min(rt, std::max(1, (40 * 1024) / std::max(row_total, 1)));
    rt = std::min(rt, (p.m + di.sm_count - 1) / di.sm_count + 1);
    p.rt = rt > 1 ? rt & ~1 : 1;  // whole row pairs
  } else {
    // Tile height: as few tiles per CTA as the tile cap allows (at most 32
    // rows -- one folder lane each -- and kTileBytes of weights + scales),
    // then the CTA's rows spread evenly over them, in whole row pairs.  Each
    // tile costs the consumers a handoff and a ragged last tile idles most
    // of them, so fewer, even tiles finish sooner (config 1: 9.6 us with
    // three tiles of 26 rows, 11.0 us with five of 16; the config-4 int4
    // matrices 20.6 and 12.2 us with 96 KB tiles, 23.0 and 13.9 with 64 KB).
    const int cap = std::max(2, std::min(32, kTileBytes / std::max(row_total, 1))) & ~1;
    const int ctas = std::min(p.m, di.sm_count);
    const int rpc = (p.m + ctas - 1) / ctas;  // rows of the largest CTA
    const int nt = (rpc + cap - 1) / cap;
    const int rt = (((rpc + nt - 1) / nt) + 1) & ~1;
    p.rt = std::max(2, std::min(rt, cap));
  }
  p.tstride = round_up(p.gpr, 32) + 4;
  // Shared memory holds the staged activations, the term ring and at least
  // two weight stages; where the tile height above leaves room for fewer,
  // tiles get shorter.
  int terms_bytes = 0;
  for (;;) {
    // Ordered folds take fb tiles (<= 32 rows) per pass over a ring of two
    // passes; the unordered fold goes tile by tile over four slots.
    p.tcols = p.gpr;
    p.wred = 0;
    if (Fmt::kFold == Fold::Tree) {
      p.fb = 1;
      p.ring = 4;
      // consumer warps pre-reduce 32 groups when each warp holds 32 groups of
      // one row pair for the whole launch
      if (p.gpr % 32 == 0 && NC % p.gpr == 0) {
        p.wred = 1;
        p.tcols = p.gpr / 32;
        // a row holds only its tcols partial sums (float4-aligned rows)
        p.tstride = round_up(p.tcols, 4) + 4;
      }
    } else {
      // As many tiles per fold pass as the term budget allows: every pass is
      // a serial chain of gpr adds per row, so long rows (down projection,
      // 344 groups) fold all of a CTA's rows in one pass (4096 x 11008:
      // 12.1 us against 14.4 with a 40 KB budget).
      p.fb = std::max(1, std::min(kMaxRing / 2, 32 / (p.rt * vr)));
      while (p.fb > 1 && 2 * p.fb * p.rt * vr * p.tstride * 4 > kFoldBytes) p.fb >>= 1;
      p.ring = 2 * p.fb;
      if (kCols) {
        // one tile per fold pass; up to four slots (the consumers run ahead)
        p.fb = 1;
        p.ring = p.rt * vr * p.tstride * 4 * 4 <= 72 * 1024 ? 4 : 2;
      }
    }
    p.x_bytes = round_up(x_stage_bytes<Fmt>(p), 16);
    p.stage_w_bytes = round_up(p.rt * p.row_bytes, 128);
    p.stage_s_bytes = Fmt::kScales ? round_up(p.rt * p.gpr * 4, 128) : 0;
    terms_bytes = round_up(p.ring * p.rt * vr * p.tstride * 4, 128);
    const int fixed = 128 + round_up(p.x_bytes, 128) + terms_bytes + 8 * (2 * kMaxStages + 2 * kMaxRing);
    const int per_stage = p.stage_w_bytes + p.stage_s_bytes;
    p.stages = std::min(kMaxStages, (lim[slot].one - fixed) / per_stage);
    if (!kCols) p.stages = std::min(p.stages, std::max(2, kFlightBytes / per_stage));
    if (p.stages >= 2 || kCols || p.rt <= 2) break;
    p.rt -= 2;
  }
  if (p.stages < 2) return LP_ERR_UNSUPPORTED;  // activations too large for shared memory
  // Bulk copies need 16-byte aligned, 16-byte multiple rows of weights and scales.
  const uintptr_t wa = reinterpret_cast<uintptr_t>(p.w);
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.ws);
  p.bulk = (p.row_bytes % 16 == 0) && (wa % 16 == 0) &&
           (!Fmt::kScales || ((p.gpr % 4 == 0) && (sa % 16 == 0)));
  p.off_w = round_up(p.x_bytes, 128);
  p.off_s = p.off_w + p.stages * p.stage_w_bytes;
  p.off_t = p.off_s + p.stages * p.stage_s_bytes;
  p.off_b = p.off_t + terms_bytes;
  const int smem = 128 + p.off_b + 8 * (2 * p.stages + 2 * p.ring);  // + base alignment slack
  const int grid = std::min(p.m, di.sm_count);
  // Programmatic dependent launch: this grid may start while the previous
  // kernel in the stream drains; it prefetches its weights at once and waits
  // for that kernel (griddepcontrol.wait) before it reads x or writes y.
  // Only GEMV kernels release their dependents early, and a GEMV writes
  // nothing but y, which never aliases another GEMV's weights, so the early
  // weight stream cannot read memory still being written.
  if (g_push) {
    p.push = g_push;
    p.push_off = g_push_off;
    g_pushed = true;
  }
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
template int launch_gemv<FmtI8F>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4F>(GemvParams, cudaStream_t);
template int launch_gemv<FmtF4F>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8_0F>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ4_0F>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ4_KF>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ6_KF>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4Q8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8FromF32>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4Q8FromF32>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8_0Q8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ4_0Q8>(GemvParams, cudaStream_t);
template int launch_gemv<FmtQ8Cols>(GemvParams, cudaStream_t);
template int launch_gemv<FmtI4Q8Cols>(GemvParams, cudaStream_t);

}  // namespace lp
