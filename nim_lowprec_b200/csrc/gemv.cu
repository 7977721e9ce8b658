// gemv.cu -- launch planning for the fused dequant-GEMV kernels.
#include <algorithm>
#include <mutex>
#include <type_traits>
#include <vector>

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
static_assert(kMaxStages <= 32 && kMaxRing <= 32, "one barrier pair per lane of warp 0");
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

// ------------------------------------------------------ batched launches
// GEMV calls made between lp_batch_begin and lp_batch_end on the batch's
// stream are recorded here (this thread only) and launched as one
// gemv_batch_kernel per run of same-format calls, after one
// gemv_images_kernel that stages every job's activations.
namespace {

// Every row-folded format (the multi-column ones fold virtual rows).
template <class Fmt> struct Batchable : std::false_type {};
template <> struct Batchable<FmtI8> : std::true_type {};
template <> struct Batchable<FmtI4> : std::true_type {};
template <> struct Batchable<FmtF4> : std::true_type {};
template <> struct Batchable<FmtQ8_0> : std::true_type {};
template <> struct Batchable<FmtQ4_0> : std::true_type {};
template <> struct Batchable<FmtI8F> : std::true_type {};
template <> struct Batchable<FmtI4F> : std::true_type {};
template <> struct Batchable<FmtF4F> : std::true_type {};
template <> struct Batchable<FmtQ8_0F> : std::true_type {};
template <> struct Batchable<FmtQ4_0F> : std::true_type {};
template <> struct Batchable<FmtQ4_KF> : std::true_type {};
template <> struct Batchable<FmtQ6_KF> : std::true_type {};
template <> struct Batchable<FmtQ8> : std::true_type {};
template <> struct Batchable<FmtI4Q8> : std::true_type {};
template <> struct Batchable<FmtQ8FromF32> : std::true_type {};
template <> struct Batchable<FmtI4Q8FromF32> : std::true_type {};
template <> struct Batchable<FmtQ8_0Q8> : std::true_type {};
template <> struct Batchable<FmtQ4_0Q8> : std::true_type {};

constexpr int kNotRecorded = -1000;
// Weights + scales of one tile, at most.  Fewer, larger copies stream
// faster per SM: on the config-4 sweep (one GPU), 80 KB tiles x 2 stages ran
// 25.7 us per layer, 60 KB x 2 30.4 us, 40 KB x 4 32.8 us.  76 KB leaves room
// for three activation buffers next to two stages (see launch_batch).
constexpr int kBatchTile = 76 * 1024;
constexpr int kBatchTerms = 48 * 1024;    // term slots, at most
constexpr int kBatchFlight = 160 * 1024;  // weight stages, at most

struct Range {
  uintptr_t lo, hi;
  bool meets(const Range& o) const { return lo < o.hi && o.lo < hi; }
};

struct BatchState {
  bool open = false;
  cudaStream_t st = nullptr;
  const void* fmt = nullptr;  // launcher of the recorded format
  int (*launch)(std::vector<GemvParams>&, cudaStream_t) = nullptr;
  int (*single)(GemvParams, cudaStream_t) = nullptr;
  std::vector<GemvParams> jobs;
  std::vector<Range> outs;    // the recorded jobs' y
  int kept = LP_OK;           // first failed flush made on another call's behalf
  const RecvSegs* recv = nullptr;  // a gather riding in the next launch (batch_flush_recv)
  float* recv_y = nullptr;
  bool recv_taken = false;
};
thread_local BatchState g_batch;

// The images' memory pool of a device: the library's own (the device's
// default pool is left as it is), keeping what it has reserved across
// synchronisations so an eager decode loop does not map memory every step.
cudaMemPool_t image_pool(int device) {
  static cudaMemPool_t pools[kMaxDevices];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  cudaMemPool_t& pool = pools[device % kMaxDevices];
  if (!pool) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      pool = nullptr;
      return nullptr;
    }
    uint64_t keep = 64ull << 20;  // up to 64 MB stays reserved
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  return pool;
}

// Plan the batch's common layout and launch the images and batch kernels;
// LP_ERR_UNSUPPORTED when the jobs do not share one layout in shared memory.
template <class Fmt>
int launch_batch(std::vector<GemvParams>& jobs, cudaStream_t st) {
  const DeviceInfo& di = device_info();
  auto kern = gemv_batch_kernel<Fmt, kNcw>;
  static int one[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  const int slot = di.ordinal % kMaxDevices;
  std::call_once(once[slot], [&] {
    cudaFuncAttributes fa;
    int st_bytes = 0;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) st_bytes = static_cast<int>(fa.sharedSizeBytes);
    one[slot] = di.max_smem_optin - st_bytes;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, one[slot]) !=
        cudaSuccess)
      one[slot] = 0;
  });
  static thread_local GemvBatch b;
  b.n = static_cast<int>(jobs.size());
  b.push = nullptr;
  b.rs.n = 0;
  b.ry = nullptr;
  // The jobs' rows laid end to end, each weighted by its bytes times the
  // consumers' slowdown on it: a thread keeps one group of the row, so when
  // the consumer count is not a multiple of the row's groups some threads
  // idle (344 groups: 344 of 512 busy, and such rows took 1.46x as long per
  // byte, measured per CTA).  Equal shares of this weight finish together.
  constexpr int NC = kNcw * 32;
  int64_t at = 0;
  for (int j = 0; j < b.n; ++j) {
    GemvParams& p = jobs[j];
    const int row_total = p.row_bytes + (Fmt::kScales ? p.gpr * 4 : 0);
    const int busy = p.gpr <= NC ? (NC / p.gpr) * p.gpr : NC;
    const int64_t weight = (static_cast<int64_t>(row_total) * NC + busy - 1) / busy;
    p.boff = at;
    p.bend = at + static_cast<int64_t>(p.m) * weight;
    at = p.bend;
    if (p.push && !b.push) b.push = p.push;
    p.x_bytes = round_up(x_stage_bytes<Fmt>(p), 16);
    const uintptr_t wa = reinterpret_cast<uintptr_t>(p.w);
    const uintptr_t sa = reinterpret_cast<uintptr_t>(p.ws);
    p.bulk = (p.row_bytes % 16 == 0) && (wa % 16 == 0) &&
             (!Fmt::kScales || ((p.gpr % 4 == 0) && (sa % 16 == 0)));
  }
  b.total = at;
  // The common layout, with tiles of at most kBatchTile bytes, or smaller
  // where the activation buffers (fp32 formats at long rows) leave no room
  // for two stages of them.
  int sw = 0, ss = 0, tslot = 0, xs = 0, ring = 2, p_off = 0, xbufs = 0, stages = 0;
  for (int tile = kBatchTile; tile >= 16 * 1024; tile -= 8 * 1024) {
    sw = ss = tslot = xs = 0;
    int fbmax = 1;
    for (auto& p : jobs) {
      // Rows per tile: what fits the tile (at most 32, one folder lane
      // each), in whole row pairs.
      const int row_total = p.row_bytes + (Fmt::kScales ? p.gpr * 4 : 0);
      int rt = std::min(32, std::max(1, tile / std::max(row_total, 1)));
      rt = rt >= 2 ? rt & ~1 : 1;
      p.rt = rt;
      p.tstride = round_up(p.gpr, 32) + 4;
      p.tcols = p.gpr;
      p.wred = 0;
      p.fb = std::max(1, std::min(kMaxRing / 2, 32 / rt));
      if (Fmt::kFold == Fold::Tree) {
        // the unordered fold goes tile by tile; consumer warps pre-reduce
        // 32 groups when each warp holds 32 groups of one row pair (as
        // planned for gemv_kernel)
        p.fb = 1;
        if (p.gpr % 32 == 0 && NC % p.gpr == 0) {
          p.wred = 1;
          p.tcols = p.gpr / 32;
          p.tstride = round_up(p.tcols, 4) + 4;
        }
      }
      sw = std::max(sw, round_up(rt * p.row_bytes, 128));
      ss = std::max(ss, Fmt::kScales ? round_up(rt * p.gpr * 4, 128) : 0);
      tslot = std::max(tslot, round_up(rt * p.tstride, 32));
      xs = std::max(xs, round_up(p.x_bytes, 16));
      fbmax = std::max(fbmax, p.fb);
    }
    // term ring: two passes of the longest fold batch (four tiles for the
    // unordered fold, which lets the consumers run ahead), within kBatchTerms
    const int want = Fmt::kFold == Fold::Tree ? 4 : 2 * fbmax;
    ring = 2;
    while (ring < want && 2 * ring * tslot * 4 <= kBatchTerms) ring *= 2;
    for (auto& p : jobs) p.fb = std::min(p.fb, ring / 2);
    // each image: the staged activations, then the job's parameters
    p_off = round_up(xs, 16);
    xs = round_up(p_off + static_cast<int>(sizeof(GemvParams)), 128);
    const int per_stage = sw + ss;
    for (xbufs = 3; xbufs >= 2; --xbufs) {
      const int fixed =
          128 + xbufs * xs + ring * tslot * 4 + 8 * (2 * kMaxStages + 2 * ring + 2 * xbufs);
      stages = std::min(kMaxStages, (one[slot] - fixed) / per_stage);
      stages = std::min(stages, std::max(2, kBatchFlight / per_stage));
      if (stages >= 2) break;
    }
    if (stages >= 2) break;
  }
  if (stages < 2 || one[slot] <= 0) return LP_ERR_UNSUPPORTED;
  b.stages = stages;
  b.ring = ring;
  b.xbufs = xbufs;
  b.stage_w_bytes = sw;
  b.stage_s_bytes = ss;
  b.tslot = tslot;
  b.x_stride = xs;
  b.p_off = p_off;
  b.off_w = xbufs * xs;
  b.off_s = b.off_w + stages * sw;
  b.off_t = b.off_s + stages * ss;
  b.off_b = b.off_t + ring * tslot * 4;
  const int smem = 128 + b.off_b + 8 * (2 * stages + 2 * ring + 2 * xbufs);
  for (int j = 0; j < b.n; ++j) b.job[j] = jobs[j];
  if (g_batch.recv && b.push) {
    b.rs = *g_batch.recv;
    b.ry = g_batch.recv_y;
  }
  // The images live for this launch only: a stream-ordered allocation (from
  // the library's pool), freed in stream order after the batch kernel (graph
  // memory nodes when the stream is being captured), so batches on other
  // streams or in other graphs never share them.
  void* img = nullptr;
  cudaMemPool_t ipool = image_pool(di.ordinal);
  int r = ipool ? cuda_status(cudaMallocFromPoolAsync(&img, static_cast<size_t>(b.n) * xs, ipool, st))
                : cuda_status(cudaMallocAsync(&img, static_cast<size_t>(b.n) * xs, st));
  if (r != LP_OK) return r;
  b.img = static_cast<uint8_t*>(img);

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(b.n);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  r = cuda_status(cudaLaunchKernelEx(&cfg, gemv_images_kernel<Fmt>, b));
  if (r == LP_OK) {
    cfg.gridDim = dim3(di.sm_count);  // one CTA per SM, each a 1/148 share of the bytes
    cfg.blockDim = dim3(32 * (kNcw + 3));  // + the image loader warp
    cfg.dynamicSmemBytes = smem;
    r = cuda_status(cudaLaunchKernelEx(&cfg, kern, b));
  }
  const int rf = cuda_status(cudaFreeAsync(img, st));
  return r != LP_OK ? r : rf;
}

// Record a GEMV into the open batch (flushing first when it cannot join the
// recorded jobs); kNotRecorded for a call on another stream.
template <class Fmt>
int batch_record(GemvParams p, cudaStream_t st) {
  BatchState& bs = g_batch;
  if (st != bs.st) return kNotRecorded;
  const void* fmt = reinterpret_cast<const void*>(&launch_batch<Fmt>);
  // The images kernel reads every job's activations before any job writes:
  // a call reading an earlier call's output, writing where one writes, or
  // pushing into another pool's exchange starts a new launch.
  const int xb = std::max(p.k * 4, 1);
  const Range xr{reinterpret_cast<uintptr_t>(p.x), reinterpret_cast<uintptr_t>(p.x) + xb};
  const Range sr{reinterpret_cast<uintptr_t>(p.xs),
                 reinterpret_cast<uintptr_t>(p.xs) + (p.xs ? p.gpr * 4 : 0)};
  const Range yr{reinterpret_cast<uintptr_t>(p.y),
                 reinterpret_cast<uintptr_t>(p.y) + static_cast<uintptr_t>(p.m) * 4};
  bool join = bs.fmt == fmt && static_cast<int>(bs.jobs.size()) < kMaxBatch;
  for (size_t i = 0; join && i < bs.outs.size(); ++i)
    join = !bs.outs[i].meets(xr) && !bs.outs[i].meets(sr) && !bs.outs[i].meets(yr);
  if (join && g_push && !bs.jobs.empty() && bs.jobs[0].push && bs.jobs[0].push != g_push) join = false;
  if (!join && !bs.jobs.empty()) {
    const int r = batch_flush();
    if (r != LP_OK) return r;
  }
  if (g_push) {
    p.push = g_push;
    p.push_off = g_push_off;
    g_pushed = true;
  }
  bs.fmt = fmt;
  bs.launch = &launch_batch<Fmt>;
  bs.single = &launch_gemv<Fmt>;
  bs.jobs.push_back(p);
  bs.outs.push_back(yr);
  return LP_OK;
}

}  // namespace

bool batch_open() { return g_batch.open; }

int batch_flush() {
  BatchState& bs = g_batch;
  if (bs.jobs.empty()) return LP_OK;
  std::vector<GemvParams> jobs;
  jobs.swap(bs.jobs);
  bs.outs.clear();
  auto launch = bs.launch;
  auto single = bs.single;
  bs.fmt = nullptr;
  int r = launch(jobs, bs.st);
  bs.recv_taken = r == LP_OK && bs.recv != nullptr;
  if (r == LP_ERR_UNSUPPORTED) {
    // no common layout: one launch per job, planned as a lone call (the
    // recorded jobs keep their push context)
    bs.open = false;
    r = LP_OK;
    for (size_t i = 0; i < jobs.size() && r == LP_OK; ++i) r = single(jobs[i], bs.st);
    bs.open = true;
  }
  return r;
}

bool batch_takes_recv(const PushCtx* push, cudaStream_t st) {
  const BatchState& bs = g_batch;
  if (!bs.open || st != bs.st || !push) return false;
  for (const auto& j : bs.jobs)
    if (j.push == push) return true;  // a batch's jobs share one context (batch_record)
  return false;
}

int batch_flush_recv(float* y, const RecvSegs& segs, bool* taken) {
  BatchState& bs = g_batch;
  bs.recv = &segs;
  bs.recv_y = y;
  bs.recv_taken = false;
  const int r = batch_flush();
  *taken = bs.recv_taken;
  bs.recv = nullptr;
  bs.recv_y = nullptr;
  bs.recv_taken = false;
  return r;
}

void batch_flush_keep() {
  const int r = batch_flush();
  if (r != LP_OK && g_batch.kept == LP_OK) g_batch.kept = r;
}

int batch_begin(cudaStream_t st) {
  const int r = batch_end(nullptr);
  g_batch.open = true;
  g_batch.st = st;
  return r;
}

int batch_end(cudaStream_t st) {
  (void)st;
  int r = batch_flush();
  if (r == LP_OK) r = g_batch.kept;
  g_batch.kept = LP_OK;
  g_batch.open = false;
  g_batch.st = nullptr;
  return r;
}

thread_local const PushCtx* g_push = nullptr;
thread_local int64_t g_push_off = 0;
thread_local bool g_pushed = false;

template <class Fmt>
int launch_gemv(GemvParams p, cudaStream_t st) {
  if (batch_open()) {
    if constexpr (Batchable<Fmt>::value)
      if (p.m > 0 && p.gpr > 0) {
        const int r = batch_record<Fmt>(p, st);
        if (r != kNotRecorded) return r;
      }
    const int r = batch_flush();
    if (r != LP_OK) return r;
  }
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
