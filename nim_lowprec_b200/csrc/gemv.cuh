// gemv.cuh -- the fused dequant-GEMV skeleton for sm_100a.
//
// Every GEMV of nim-lowprec has the same shape: output row m is an ordered
// fold over the row's groups (blocks) g of a per-group term,
//     y[m] = fold_g term(m, g)
// where term(m, g) needs only group g of row m plus the activations of group g:
//   fp32 activations  term = (sequential fp32 sum over the group of w*x) * s
//                     (simd/dequant.nim:253-256, 329-338, 410-419, 564-567,
//                      616-621)
//   int8 activations  term = (f32(exact int32 group dot) * ws) * xs
//                     (applyScales, simd/dequant.nim:654-657)
//   ggml int8 acts    term = f32(isum) * (wd * xd), folded into 4 lanes by
//                     block index mod 4 (simd/dequant.nim:1275-1286)
// and the fold is either serial from 0.0 or that 4-lane discipline.  Terms
// parallelise freely; the fold must keep its order to stay bit-exact.
//
// Work layout.  Each CTA owns a contiguous, balanced range of rows (one CTA
// per SM; under programmatic dependent launch the next launch's CTA takes
// the SM as soon as this one exits and streams its weights at once).  It walks its
// rows in tiles of RT consecutive rows -- one contiguous stretch of HBM, so
// one large bulk copy (per-SM copy throughput on B200 grows with copy size:
// copies of 16 KB and up are needed to stream at full HBM bandwidth).
//
//   warp 0   producer: per tile one 1-D bulk copy (TMA) of the weight rows and
//            one of their scale rows, HBM -> shared, `stages` deep, tracked
//            by mbarriers.  Rows that are not 16-byte multiples take a
//            plain-load staging path.  It releases the next launch in the
//            stream at once and starts before the activations are staged.
//   warps 2+ consumers: the terms of row pairs x groups into a ring of
//            per-tile term matrices (`ring` tiles deep).
//   warp 1   folder: reduces each finished row to y.  Ordered folds (the
//            bit-exact paths) give each lane one row and take `fb` tiles at a
//            time so up to 32 independent chains run together; the
//            unordered fold of the block-float path sums a row across lanes.
#pragma once
#include <type_traits>

#include "lp_device.cuh"
#include "lp_internal.h"

namespace lp {

enum class Fold { Serial, Lanes4, Tree };

constexpr int kMaxRing = 16;  // term-ring slots (tiles), at most

struct GemvParams {
  const uint8_t* w;   // weight rows, row_bytes each
  const float* ws;    // per-row group scales (M x gpr) or nullptr
  const void* x;      // activations (format-specific)
  const float* xs;    // activation group scales or nullptr
  float* y;
  int m, k, gs, gpr;  // gpr: groups (ggml: blocks) per row
  int row_bytes;
  int rt;             // rows per tile (<= 32: one folder lane each)
  int stages;
  int bulk;           // 1: bulk-copy staging, 0: plain loads
  int tstride;        // floats per term-matrix row
  int x_bytes;        // shared bytes for the staged activations
  int fb;             // tiles per ordered fold batch (fb * rt <= 32)
  int ring;           // term-ring slots, a multiple of fb
  int wred;           // 1: unordered fold pre-reduced by consumer warps (32 groups each)
  int tcols;          // term columns per row the folder sums (gpr, or gpr / 32)
  int off_w, off_s, off_t, off_b;  // shared-memory offsets (128-byte aligned)
  int stage_w_bytes, stage_s_bytes;
  float neg_zero;     // -0.0f, passed at run time (see mul2_rn)
  int ncol;           // activation columns (the small-n GEMM formats); else unused
  const PushCtx* push;  // pooled call: also store every output into the other ranks
  int64_t push_off;     // this slice's first element in the whole y
  // batched launches: the job's rows in the batch's rows laid end to end,
  // as a range [boff, bend) of work units (bytes weighted by consumer cost)
  int64_t boff, bend;
};

// The pooled form's stores: out value v of y element idx (of this slice) goes
// out as one 8-byte word tagged with the gather number, which the receiver
// polls (pool.cu): into every other rank's exchange buffer, or, for a large
// gather, into this rank's own buffer for the others to read.
struct PushTag {
  uint64_t tag = 0;
  int64_t half = 0;
};
__device__ __forceinline__ PushTag push_tag(const PushCtx* push) {
  PushTag t;
  if (push) {
    const uint32_t e = *reinterpret_cast<volatile const uint32_t*>(push->state) + 1u;
    t.tag = static_cast<uint64_t>(e) << 32;
    t.half = (e & 1u) * kXchgWords;
  }
  return t;
}
// Pull form: one local store per output, whatever the rank count, so the
// fold never waits on remote writes (the receivers pay the NVLink reads, in
// bulk, once per gather).  Push form: the receive is a local read, the better
// trade for small gathers that come one after another.
__device__ __forceinline__ void push_out(const GemvParams& p, const PushTag& t, int64_t idx,
                                         float v) {
  const uint64_t w = t.tag | __float_as_uint(v);
  const int nr = p.push->nranks, me = p.push->rank;
  if (p.push->pull) {
    uint64_t* a = reinterpret_cast<uint64_t*>(p.push->peers[me]) + t.half + p.push_off + idx;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
    return;
  }
  for (int q = 0; q < nr; ++q) {
    if (q == me) continue;
    uint64_t* a = reinterpret_cast<uint64_t*>(p.push->peers[q]) + t.half + p.push_off + idx;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
  }
}

// Formats with a column dimension (kCols) compute, per (row, group), one term
// for each of p.ncol activation columns.  The skeleton treats (row r, column
// c) of a tile as virtual row r * ncol + c: that is y's own row-major index
// (y is M x ncol), so tiles, folds and stores stay those of a GEMV with
// rt * ncol rows.
template <class F, class = void>
struct ColsOf : std::false_type {};
template <class F>
struct ColsOf<F, std::void_t<decltype(F::kCols)>> : std::bool_constant<F::kCols> {};

// ------------------------------------------------------------ x staging
// Cooperative copy of `bytes` bytes global -> shared (activations are tiny
// next to the weights and are staged once per CTA).
__device__ __forceinline__ void copy_bytes(uint8_t* dst, const uint8_t* src, int bytes, int tid,
                                           int nthr) {
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    const int n16 = bytes >> 4;
    for (int i = tid; i < n16; i += nthr)
      reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    for (int i = (n16 << 4) + tid; i < bytes; i += nthr) dst[i] = src[i];
  } else {
    for (int i = tid; i < bytes; i += nthr) dst[i] = src[i];
  }
}

// ------------------------------------------------------------- folds
// Row folds in group order.  Terms come in 32 at a time, the next batch
// loaded while the current one is added, so the add chain (the only true
// dependency) never waits on shared-memory latency.
__device__ __forceinline__ void load32(const float* T, int g, int g4, float4 (&v)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    v[k] = (g + 4 * k < g4) ? *reinterpret_cast<const float4*>(T + g + 4 * k)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
}

// total = ((0 + t0) + t1) + ... (simd/dequant.nim:877 and kin), or with
// four lanes lane[g & 3] += t_g, then (l0 + l1) + (l2 + l3)
// (simd/dequant.nim:1275-1286).
template <Fold F>
__device__ __forceinline__ float fold_row(const float* T, int gpr) {
  const int g4 = gpr & ~3;
  float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
  float4 a[8], b[8];
  load32(T, 0, g4, a);
  for (int g = 0; g < g4; g += 32) {
    load32(T, g + 32, g4, b);
    const int n4 = min(8, (g4 - g) >> 2);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < n4) {
        if (F == Fold::Serial) {
          l0 = fadd(l0, a[k].x);
          l0 = fadd(l0, a[k].y);
          l0 = fadd(l0, a[k].z);
          l0 = fadd(l0, a[k].w);
        } else {
          l0 = fadd(l0, a[k].x);
          l1 = fadd(l1, a[k].y);
          l2 = fadd(l2, a[k].z);
          l3 = fadd(l3, a[k].w);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = b[k];
  }
  for (int g = g4; g < gpr; ++g) {
    if (F == Fold::Serial) {
      l0 = fadd(l0, T[g]);
    } else {
      const int l = g & 3;
      if (l == 0) l0 = fadd(l0, T[g]);
      else if (l == 1) l1 = fadd(l1, T[g]);
      else l2 = fadd(l2, T[g]);
    }
  }
  return F == Fold::Serial ? l0 : fadd(fadd(l0, l1), fadd(l2, l3));
}

// Unordered row sums (block-float path): L lanes per row, L the largest
// power of two with L * rows <= 32; each lane sums 4-term slices of the row
// (four 16-byte loads in flight), then the L partial sums meet by shuffles.
__device__ __forceinline__ void tree_fold(const float* T, int tstride, int rows, int gpr,
                                          float* y, int lane, const GemvParams& p,
                                          const PushTag& pt, int64_t y0) {
  int lg = 5;
  while (lg > 0 && (rows << lg) > 32) --lg;
  const int L = 1 << lg;
  const int r = lane >> lg, sub = lane & (L - 1);
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  if (r < rows) {
    const float* row = T + r * tstride;
    const int g4 = gpr & ~3;
    int g = 4 * sub;
    for (; g + 12 * L < g4; g += 16 * L) {
      const float4 a = *reinterpret_cast<const float4*>(row + g);
      const float4 b = *reinterpret_cast<const float4*>(row + g + 4 * L);
      const float4 c = *reinterpret_cast<const float4*>(row + g + 8 * L);
      const float4 d = *reinterpret_cast<const float4*>(row + g + 12 * L);
      s0 = fadd(s0, fadd(fadd(a.x, b.x), fadd(c.x, d.x)));
      s1 = fadd(s1, fadd(fadd(a.y, b.y), fadd(c.y, d.y)));
      s2 = fadd(s2, fadd(fadd(a.z, b.z), fadd(c.z, d.z)));
      s3 = fadd(s3, fadd(fadd(a.w, b.w), fadd(c.w, d.w)));
    }
    for (; g < g4; g += 4 * L) {
      const float4 a = *reinterpret_cast<const float4*>(row + g);
      s0 = fadd(s0, a.x);
      s1 = fadd(s1, a.y);
      s2 = fadd(s2, a.z);
      s3 = fadd(s3, a.w);
    }
    if (sub == 0)
      for (int t = g4; t < gpr; ++t) s0 = fadd(s0, row[t]);
  }
  float s = fadd(fadd(s0, s1), fadd(s2, s3));
  for (int o = L >> 1; o > 0; o >>= 1) s = fadd(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (r < rows && sub == 0) {
    y[r] = s;
    if (p.push) push_out(p, pt, y0 + r, s);
  }
}

// Unordered fold, first stage, in a consumer warp whose 32 lanes hold 32
// consecutive groups of the same four rows (t0..t3 = rows ra, ra+1, rc,
// rc+1): a reduce-scatter over the lanes (6 shuffles for the 4 rows) leaves
// each row's 32-group sum in lanes 0, 8, 16 and 24, stored as column `col`
// of the term matrix.  rc < 0: only rows ra, ra+1 exist.
__device__ __forceinline__ void store_warp_sums(float* T, int tstride, int rows, int ra, int rc,
                                                float t0, float t1, float t2, float t3, int col,
                                                int lane) {
  const bool h16 = lane & 16, h8 = lane & 8;
  float ka = h16 ? t2 : t0, kb = h16 ? t3 : t1;
  const float sa = h16 ? t0 : t2, sb = h16 ? t1 : t3;
  ka = fadd(ka, __shfl_xor_sync(0xffffffffu, sa, 16));
  kb = fadd(kb, __shfl_xor_sync(0xffffffffu, sb, 16));
  float k = h8 ? kb : ka;
  const float sd = h8 ? ka : kb;
  k = fadd(k, __shfl_xor_sync(0xffffffffu, sd, 8));
  k = fadd(k, __shfl_xor_sync(0xffffffffu, k, 4));
  k = fadd(k, __shfl_xor_sync(0xffffffffu, k, 2));
  k = fadd(k, __shfl_xor_sync(0xffffffffu, k, 1));
  if ((lane & 7) == 0) {
    const int slot = lane >> 3;
    const int row = (slot < 2 ? ra : rc) + (slot & 1);
    if ((slot < 2 || rc >= 0) && row < rows) T[row * tstride + col] = k;
  }
}

// ----------------------------------------------------------- the kernel
template <class Fmt, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 2), 1) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ volatile int s_abort;
  // Every bulk-copy destination is a 128-byte multiple from this base.
  uint8_t* smem = smem_raw + ((128u - (saddr(smem_raw) & 127u)) & 127u);
  uint8_t* xsm = smem;
  uint8_t* stw = smem + p.off_w;
  uint8_t* sts = smem + p.off_s;
  float* terms = reinterpret_cast<float*>(smem + p.off_t);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_b);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* tfull = bars + 2 * p.stages;
  uint64_t* tempty = tfull + p.ring;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row_begin = static_cast<int>((static_cast<int64_t>(p.m) * blockIdx.x) / gridDim.x);
  const int row_end = static_cast<int>((static_cast<int64_t>(p.m) * (blockIdx.x + 1)) / gridDim.x);
  const int ntiles = (row_end - row_begin + p.rt - 1) / p.rt;

  // one barrier pair per lane of warp 0 (stages <= 12, ring <= 16)
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    if (i < p.stages) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    if (i < p.ring) {
      mbar_init(&tfull[i], NCW);
      mbar_init(&tempty[i], 1);
    }
    if (i == 0) s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (ntiles <= 0) return;

  if (warp == 0) {
    // ------------------------------------------------------ producer
    // The next launch in the stream may start now: it streams only its own
    // weights before its grid-dependency wait, and no GEMV writes weights.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint64_t pol = l2_evict_first();
    int t = 0;
    for (; t < ntiles; ++t) {
      const int s = t % p.stages;
      if (t >= p.stages && !mbar_wait_idle(&empty[s], ((t / p.stages) - 1) & 1, &s_abort)) break;
      if (s_abort) break;
      const int r0 = row_begin + t * p.rt;
      const int rows = min(p.rt, row_end - r0);
      const uint32_t bw = static_cast<uint32_t>(rows) * p.row_bytes;
      const uint32_t bs = Fmt::kScales ? static_cast<uint32_t>(rows) * p.gpr * 4u : 0u;
      const uint8_t* gw = p.w + static_cast<int64_t>(r0) * p.row_bytes;
      const float* gsc = Fmt::kScales ? p.ws + static_cast<int64_t>(r0) * p.gpr : nullptr;
      uint8_t* dw = stw + s * p.stage_w_bytes;
      uint8_t* ds = sts + s * p.stage_s_bytes;
      if (p.bulk) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], bw + bs);
          bulk_g2s(dw, gw, bw, &full[s], pol);
          if (Fmt::kScales) bulk_g2s(ds, gsc, bs, &full[s], pol);
        }
      } else {
        for (uint32_t i = lane; i < bw; i += 32) dw[i] = gw[i];
        if constexpr (Fmt::kScales)
          for (uint32_t i = lane; i < bs / 4; i += 32) reinterpret_cast<float*>(ds)[i] = gsc[i];
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
    }
    // Drain: never leave the CTA with a bulk copy still landing in shared.
    if (p.bulk && lane == 0) {
      for (int u = max(0, t - p.stages); u < t; ++u)
        mbar_wait(&full[u % p.stages], (u / p.stages) & 1);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- folder
    // a pooled call's gather number is final once the previous kernel in the
    // stream (the previous gather) has completed
    PushTag pt;
    if (p.push) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      pt = push_tag(p.push);
    }
    if constexpr (Fmt::kFold == Fold::Tree) {
      for (int t = 0; t < ntiles; ++t) {
        const int slot = t % p.ring;
        if (!mbar_wait_idle(&tfull[slot], (t / p.ring) & 1, &s_abort)) break;
        if (s_abort) break;
        const int r0 = row_begin + t * p.rt;
        const int rows = min(p.rt, row_end - r0);
        tree_fold(terms + slot * p.rt * p.tstride, p.tstride, rows, p.tcols, p.y + r0, lane, p, pt,
                  r0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
      }
    } else if constexpr (ColsOf<Fmt>::value) {
      // one tile per pass; its rows * ncol virtual rows 32 at a time
      for (int t = 0; t < ntiles; ++t) {
        const int slot = t % p.ring;
        if (!mbar_wait_idle(&tfull[slot], (t / p.ring) & 1, &s_abort)) break;
        if (s_abort) break;
        const int r0 = row_begin + t * p.rt;
        const int nv = min(p.rt, row_end - r0) * p.ncol;
        const float* T = terms + slot * p.rt * p.ncol * p.tstride;
        for (int v = lane; v < nv; v += 32) {
          const int64_t idx = static_cast<int64_t>(r0) * p.ncol + v;
          const float val = fold_row<Fmt::kFold>(T + v * p.tstride, p.gpr);
          p.y[idx] = val;
          if (p.push) push_out(p, pt, idx, val);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
      }
    } else {
      // Lane l folds (virtual) row l % (rt * vr) of tile t0 + l / (rt * vr)
      // of each batch.
      constexpr bool kCols = ColsOf<Fmt>::value;
      const int vr = kCols ? p.ncol : 1;
      const int vt = p.rt * vr;
      const int ti = lane / vt, r = lane - ti * vt;
      for (int t0 = 0; t0 < ntiles; t0 += p.fb) {
        const int nt = min(p.fb, ntiles - t0);
        bool ok = true;
        for (int i = 0; i < nt && ok; ++i)
          ok = mbar_wait_idle(&tfull[(t0 + i) % p.ring], ((t0 + i) / p.ring) & 1, &s_abort);
        if (!ok || s_abort) break;
        if (ti < nt) {
          const int t = t0 + ti;
          const int r0 = row_begin + t * p.rt;
          if (r < min(p.rt, row_end - r0) * vr) {
            const int64_t idx = static_cast<int64_t>(r0) * vr + r;
            const float val = fold_row<Fmt::kFold>(terms + ((t % p.ring) * vt + r) * p.tstride, p.gpr);
            p.y[idx] = val;
            if (p.push) push_out(p, pt, idx, val);
          }
        }
        __syncwarp();
        if (lane == 0)
          for (int i = 0; i < nt; ++i) mbar_arrive(&tempty[(t0 + i) % p.ring]);
      }
    }
  } else {
    // ------------------------------------------------------ consumers
    const int ct = threadIdx.x - 64;
    constexpr int NC = NCW * 32;
    // The activations (and y, written by the folder after these warps
    // signal) may belong to the previous kernel in the stream.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    Fmt::stage_x(xsm, p, ct, NC);
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    Fmt f;
    // Unit q = pair * gpr + g.  When gpr <= NC a thread keeps one group for
    // the whole launch (activations in registers) and takes two row pairs per
    // step, two independent straight-line term2 calls the compiler
    // interleaves; longer rows walk q = ct, ct + NC, ... without a division
    // per unit.
    const int dpr = NC / p.gpr, dg = NC - dpr * p.gpr;
    const int pr0 = ct / p.gpr, g0 = ct - pr0 * p.gpr;
    // Whenever a row's groups fit the consumers (gpr <= NC) a thread keeps
    // one group for the whole launch; when NC is not a multiple of gpr the
    // threads past the last whole multiple have no unit.
    const bool fixed = dpr >= 1;
    const bool idle = fixed && ct >= dpr * p.gpr;
    if constexpr (!ColsOf<Fmt>::value)
      if (fixed && !idle) f.prepare(p, xsm, g0);
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % p.stages;
      const int tb = t % p.ring;
      bool ok = mbar_wait(&full[s], (t / p.stages) & 1, &s_abort);
      if (ok && t >= p.ring) ok = mbar_wait(&tempty[tb], ((t / p.ring) - 1) & 1, &s_abort);
      if (!ok || s_abort) break;
      const int r0 = row_begin + t * p.rt;
      const int rows = min(p.rt, row_end - r0);
      const uint8_t* W = stw + s * p.stage_w_bytes;
      const float* S = reinterpret_cast<const float*>(sts + s * p.stage_s_bytes);
      float* T = terms + tb * p.rt * p.tstride;
      const int npairs = (rows + 1) >> 1;
      if constexpr (ColsOf<Fmt>::value) {
        // one (row pair, group) unit at a time, all columns of it: each
        // column's activations are read once for both rows
        T = terms + tb * p.rt * p.ncol * p.tstride;
        for (int q = ct; q < npairs * p.gpr; q += NC) {
          const int pr = q / p.gpr, g = q - pr * p.gpr;
          const int ra = 2 * pr, rb = min(ra + 1, rows - 1);
          f.termcols2(p, xsm, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                      S + rb * p.gpr, g, T + ra * p.ncol * p.tstride,
                      ra + 1 < rows ? T + (ra + 1) * p.ncol * p.tstride : nullptr, p.tstride);
        }
      } else if (fixed) {
        const int g = g0;
        int pr = idle ? npairs : pr0;
        for (; Fmt::kTwoPairs && pr + dpr < npairs; pr += 2 * dpr) {
          const int ra = 2 * pr, rc = 2 * (pr + dpr);
          const int rb = min(ra + 1, rows - 1), rd = min(rc + 1, rows - 1);
          float t0, t1, t2, t3;
          f.term2(p, xsm, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                  S + rb * p.gpr, g, t0, t1);
          f.term2(p, xsm, W + rc * p.row_bytes, W + rd * p.row_bytes, S + rc * p.gpr,
                  S + rd * p.gpr, g, t2, t3);
          if constexpr (Fmt::kFix) {
            f.fix2(p, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                   S + rb * p.gpr, g, t0, t1);
            f.fix2(p, W + rc * p.row_bytes, W + rd * p.row_bytes, S + rc * p.gpr,
                   S + rd * p.gpr, g, t2, t3);
          }
          if (Fmt::kFold == Fold::Tree && p.wred) {
            store_warp_sums(T, p.tstride, rows, ra, rc, t0, t1, t2, t3, g >> 5, lane);
            continue;
          }
          T[ra * p.tstride + g] = t0;
          if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
          T[rc * p.tstride + g] = t2;
          if (rc + 1 < rows) T[(rc + 1) * p.tstride + g] = t3;
        }
        for (; pr < npairs; pr += dpr) {  // the rest one pair at a time
          const int ra = 2 * pr;
          const int rb = min(ra + 1, rows - 1);
          float t0, t1;
          f.term2(p, xsm, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                  S + rb * p.gpr, g, t0, t1);
          if constexpr (Fmt::kFix)
            f.fix2(p, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                   S + rb * p.gpr, g, t0, t1);
          if (Fmt::kFold == Fold::Tree && p.wred) {
            store_warp_sums(T, p.tstride, rows, ra, -1, t0, t1, 0.0f, 0.0f, g >> 5, lane);
          } else {
            T[ra * p.tstride + g] = t0;
            if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
          }
        }
      } else {
        int g = g0;
        for (int pr = pr0; pr < npairs;) {
          const int ra = 2 * pr;
          const int rb = min(ra + 1, rows - 1);
          float t0, t1;
          f.prepare(p, xsm, g);
          f.term2(p, xsm, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                  S + rb * p.gpr, g, t0, t1);
          if constexpr (Fmt::kFix)
            f.fix2(p, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                   S + rb * p.gpr, g, t0, t1);
          T[ra * p.tstride + g] = t0;
          if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
          g += dg;
          pr += dpr;
          if (g >= p.gpr) {
            g -= p.gpr;
            ++pr;
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&tfull[tb]);
      }
    }
  }
}


// ------------------------------------------------------ batched launches
// Several GEMVs of one format in one persistent launch (lp_batch_begin ..
// lp_batch_end).  A lone GEMV pays, per launch, the CTA start, the
// activation staging after its grid-dependency wait, the first copy's
// latency and the last tile's fold -- about 5.7 us at K = 4096 and 8.1 us at
// K = 11008 with one row per SM, more than a 4800 x 4096 int4 slice takes
// to stream.  Here the producer streams job after job without a break, the
// folder trails the consumers across job boundaries, and each job's staged
// activations come from an image a small kernel builds once for the whole
// batch (byte for byte what the job's consumers would have staged), copied
// by a loader warp into one of `xbufs` buffers while earlier jobs compute.
//
// Common layout: every job uses the same weight stages, term slots and
// activation buffers, so the barriers' phases run on over the whole batch
// (tile counter tg across jobs).  Per job: rows per tile rt, term stride
// tstride, fold batch fb (<= ring / 2) and its image's byte count x_bytes.
// Ordered folds go fb tiles per pass; the unordered (block-float) fold goes
// tile by tile, from the consumer warps' 32-group partial sums where the job
// allows them (wred), as in gemv_kernel.
constexpr int kMaxBatch = 64;

struct GemvBatch {
  int n;                     // jobs
  int stages, ring, xbufs;   // weight stages, term slots, activation buffers
  int stage_w_bytes, stage_s_bytes;
  int tslot;                 // floats per term slot
  int x_stride;              // bytes per activation buffer and per image (128-multiple)
  int p_off;                 // the job's GemvParams inside its image (after the activations)
  int off_w, off_s, off_t, off_b;  // activation buffers from 0, x_stride apart
  uint8_t* img;              // n images, x_stride apart
  int64_t total;             // work units of all jobs' rows (job[n - 1].bend)
  const PushCtx* push;       // the pooled jobs' exchange (one per batch), or null
  GemvParams job[kMaxBatch];
  // A gather riding in this launch (rs.n > 0): every other rank's
  // rows of the group's vector ry, read by each CTA once its rows are done;
  // the launch then completes the gather (see batch_receive).
  RecvSegs rs;
  float* ry;
};

static_assert(sizeof(GemvParams) % 16 == 0, "job parameters are copied in 16-byte pieces");

// Work split.  The jobs' rows, laid end to end in work units (bytes weighted
// by the consumers' cost per byte, see launch_batch), are cut into one
// contiguous range per CTA, [cs, ce); a row belongs to the CTA whose range
// holds its first unit.  So a CTA streams one stretch of HBM and meets only
// the one to three jobs its range touches, whatever their number or size:
// a job boundary costs its activations, its parameters and its first tile's
// latency, which 64 small per-job slices per CTA (a sweep's share on 8 GPUs)
// would pay 64 times.
struct CtaRange {
  int64_t cs, ce;
};
__device__ __forceinline__ CtaRange cta_range(int64_t total) {
  return {total * blockIdx.x / gridDim.x, total * (blockIdx.x + 1) / gridDim.x};
}

// This CTA's rows of a job: [rb, re) in tiles of p.rt (nt = 0: none).
__device__ __forceinline__ int batch_rows(const GemvParams& p, const CtaRange& c, int& rb,
                                          int& nt) {
  const int64_t rtot = (p.bend - p.boff) / p.m;  // units per row
  auto first_row = [&](int64_t at) -> int {      // first row starting at or after `at`
    if (at <= p.boff) return 0;
    return static_cast<int>(min((at - p.boff + rtot - 1) / rtot, static_cast<int64_t>(p.m)));
  };
  rb = first_row(c.cs);
  const int re = first_row(c.ce);
  nt = (re - rb + p.rt - 1) / p.rt;
  return re;
}

// The first job whose byte range reaches past cs (jobs are contiguous).
__device__ __forceinline__ int first_job(const GemvBatch& b, const CtaRange& c) {
  int lo = 0, hi = b.n;  // first j with job[j].bend > cs
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (b.job[mid].bend > c.cs) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// One block per job: the job's staged activations, written to its image.
template <class Fmt>
__global__ void __launch_bounds__(512) gemv_images_kernel(const __grid_constant__ GemvBatch b) {
  // the batch kernel may start streaming weights now; it reads the images
  // only after this grid has completed (its own grid-dependency wait)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int j = blockIdx.x;
  if (j >= b.n) return;
  uint8_t* img = b.img + static_cast<int64_t>(j) * b.x_stride;
  Fmt::stage_x(img, b.job[j], threadIdx.x, blockDim.x);
  // the job's own parameters ride along: the consumers read them from
  // shared memory instead of the kernel's parameter block
  const uint32_t* src = reinterpret_cast<const uint32_t*>(&b.job[j]);
  for (int i = threadIdx.x; i < static_cast<int>(sizeof(GemvParams) / 4); i += blockDim.x)
    reinterpret_cast<uint32_t*>(img + b.p_off)[i] = src[i];
}

// The receive of a batch that carries a gather, run by all of a CTA's
// threads once its GEMV rows are done.  The segments laid end to end
// are split evenly over the CTAs, in part order, so CTA c reads roughly the
// parts that the other ranks' CTA c made, which are done about when its own
// are.  Each thread keeps 8 words in flight; a word whose tag is not yet this
// gather's is polled again (bounded, with a short sleep).  Only other GPUs'
// outputs are waited on, and their kernels wait on nothing before making
// them, so every wait ends.  (One extra warp per CTA reading the same words
// while the GEMVs still streamed weights made the config-4 sweep on 2 GPUs
// 1.7x slower; at the tail the exchange costs 0.79 us per layer there,
// against 0.94 for a receive kernel after the batch.)
__device__ __forceinline__ uint64_t ld_sys(const uint64_t* a) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
static __device__ __noinline__ void batch_receive(const GemvBatch& b, const PushTag& t, int tid,
                                                  int nthr) {
  const RecvSegs& segs = b.rs;
  const uint32_t e = static_cast<uint32_t>(t.tag >> 32);
  const int64_t total = segs.start[segs.n];
  const int64_t C = gridDim.x;
  const int64_t per = (total + C - 1) / C;
  const int64_t lo = min(total, static_cast<int64_t>(blockIdx.x) * per), hi = min(total, lo + per);
  int sg = 0;  // the segment of index lo + tid, advanced as the index grows
  {
    int a = 0, z = segs.n;
    const int64_t i = lo + tid;
    while (z - a > 1) {
      const int mid = (a + z) >> 1;
      if (segs.start[mid] <= i) a = mid; else z = mid;
    }
    sg = a;
  }
  // pull form: the words wait in their owner's buffer; push form: the
  // owners stored them into this rank's buffer from their folds
  const int pull = b.push->pull, me = b.push->rank;
  bool ok = true;
  const uint64_t t0 = global_ns();
  constexpr int kF = 8;
  for (int64_t i0 = lo + tid; i0 < hi && ok; i0 += kF * nthr) {
    uint64_t w[kF];
    int64_t at[kF];  // the word's element in ry and in its owner's exchange half
    int src[kF];     // its owner
#pragma unroll
    for (int k = 0; k < kF; ++k) {
      const int64_t i = i0 + k * nthr;
      at[k] = -1;
      w[k] = 0;
      src[k] = 0;
      if (i < hi) {
        while (sg + 1 < segs.n && segs.start[sg + 1] <= i) ++sg;
        at[k] = segs.off[sg] + (i - segs.start[sg]);
        src[k] = pull ? segs.src[sg] : me;
        w[k] = ld_sys(reinterpret_cast<const uint64_t*>(b.push->peers[src[k]]) + t.half + at[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < kF; ++k) {
      if (at[k] < 0 || !ok) continue;
      for (uint32_t n = 1; (w[k] >> 32) != e; ++n) {
        if ((n & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
          raise_error(LP_ERR_TIMEOUT);
          ok = false;
          break;
        }
        __nanosleep(128);
        w[k] = ld_sys(reinterpret_cast<const uint64_t*>(b.push->peers[src[k]]) + t.half + at[k]);
      }
      if (ok) b.ry[at[k]] = __uint_as_float(static_cast<uint32_t>(w[k]));
    }
  }
}

template <class Fmt, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 3), 1)
    gemv_batch_kernel(const __grid_constant__ GemvBatch b) {
  static_assert(!ColsOf<Fmt>::value, "row folds only");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ volatile int s_abort;
  __shared__ uint32_t s_gather;  // the gather number a carried receive completes
  uint8_t* smem = smem_raw + ((128u - (saddr(smem_raw) & 127u)) & 127u);
  uint8_t* stw = smem + b.off_w;
  uint8_t* sts = smem + b.off_s;
  float* terms = reinterpret_cast<float*>(smem + b.off_t);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + b.off_b);
  uint64_t* empty = full + b.stages;
  uint64_t* tfull = empty + b.stages;
  uint64_t* tempty = tfull + b.ring;
  uint64_t* xfull = tempty + b.ring;  // image landed in buffer i (the loader warp's 32 lanes)
  uint64_t* xempty = xfull + b.xbufs; // every consumer warp done with buffer i

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // one barrier pair per lane of warp 0 (stages <= 12, ring <= 16, xbufs <= 3)
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    if (i < b.stages) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    if (i < b.ring) {
      mbar_init(&tfull[i], NCW);
      mbar_init(&tempty[i], 1);
    }
    if (i < b.xbufs) {
      mbar_init(&xfull[i], 32);
      mbar_init(&xempty[i], NCW);
    }
    if (i == 0) s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------ producer
    // Weights are never written by kernels this launch may overlap (see
    // gemv_kernel), so the stream starts before the grid-dependency wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint64_t pol = l2_evict_first();
    const CtaRange cr = cta_range(b.total);
    int tg = 0;
    bool stop = false;
    for (int j = first_job(b, cr); j < b.n && b.job[j].boff < cr.ce && !stop; ++j) {
      const GemvParams& p = b.job[j];
      int rb, nt;
      const int re = batch_rows(p, cr, rb, nt);
      for (int t = 0; t < nt; ++t, ++tg) {
        const int s = tg % b.stages;
        if (tg >= b.stages && !mbar_wait_idle(&empty[s], ((tg / b.stages) - 1) & 1, &s_abort)) {
          stop = true;
          break;
        }
        if (s_abort) {
          stop = true;
          break;
        }
        const int r0 = rb + t * p.rt;
        const int rows = min(p.rt, re - r0);
        const uint32_t bw = static_cast<uint32_t>(rows) * p.row_bytes;
        const uint32_t bs = Fmt::kScales ? static_cast<uint32_t>(rows) * p.gpr * 4u : 0u;
        const uint8_t* gw = p.w + static_cast<int64_t>(r0) * p.row_bytes;
        const float* gsc = Fmt::kScales ? p.ws + static_cast<int64_t>(r0) * p.gpr : nullptr;
        uint8_t* dw = stw + s * b.stage_w_bytes;
        uint8_t* ds = sts + s * b.stage_s_bytes;
        if (p.bulk) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[s], bw + bs);
            bulk_g2s(dw, gw, bw, &full[s], pol);
            if (Fmt::kScales) bulk_g2s(ds, gsc, bs, &full[s], pol);
          }
        } else {
          for (uint32_t i = lane; i < bw; i += 32) dw[i] = gw[i];
          if constexpr (Fmt::kScales)
            for (uint32_t i = lane; i < bs / 4; i += 32) reinterpret_cast<float*>(ds)[i] = gsc[i];
          __threadfence_block();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      }
    }
    // never leave the CTA with a bulk copy still landing in shared memory
    if (lane == 0)
      for (int u = max(0, tg - b.stages); u < tg; ++u)
        mbar_wait(&full[u % b.stages], (u / b.stages) & 1);
  } else if (warp == 1) {
    // --------------------------------------------------------- folder
    // Lane l folds row l % rt of tile l / rt of each pass of fb tiles (the
    // unordered fold: all lanes on each tile in turn).  The jobs of a pooled
    // batch share one exchange and one gather number.
    PushTag pt;
    if (b.push) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      pt = push_tag(b.push);
      if (lane == 0) s_gather = static_cast<uint32_t>(pt.tag >> 32);
    }
    const CtaRange cr = cta_range(b.total);
    int tg = 0;
    bool stop = false;
    for (int j = first_job(b, cr); j < b.n && b.job[j].boff < cr.ce && !stop; ++j) {
      const GemvParams& p = b.job[j];
      int rb, nt;
      const int re = batch_rows(p, cr, rb, nt);
      if constexpr (Fmt::kFold == Fold::Tree) {
        for (int t = 0; t < nt; ++t) {
          const int slot = (tg + t) % b.ring;
          if (!mbar_wait_idle(&tfull[slot], ((tg + t) / b.ring) & 1, &s_abort) || s_abort) {
            stop = true;
            break;
          }
          const int r0 = rb + t * p.rt;
          tree_fold(terms + slot * b.tslot, p.tstride, min(p.rt, re - r0), p.tcols, p.y + r0,
                    lane, p, pt, r0);
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[slot]);
        }
        tg += nt;
        continue;
      }
      const int ti = lane / p.rt, r = lane - ti * p.rt;
      for (int t0 = 0; t0 < nt; t0 += p.fb) {
        const int nb = min(p.fb, nt - t0);
        bool ok = true;
        for (int i = 0; i < nb && ok; ++i)
          ok = mbar_wait_idle(&tfull[(tg + t0 + i) % b.ring], ((tg + t0 + i) / b.ring) & 1,
                              &s_abort);
        if (!ok || s_abort) {
          stop = true;
          break;
        }
        if (ti < nb) {
          const int t = t0 + ti;
          const int r0 = rb + t * p.rt;
          if (r < min(p.rt, re - r0)) {
            const int64_t idx = static_cast<int64_t>(r0) + r;
            const float val = fold_row<Fmt::kFold>(
                terms + ((tg + t) % b.ring) * b.tslot + r * p.tstride, p.gpr);
            p.y[idx] = val;
            if (p.push) push_out(p, pt, idx, val);
          }
        }
        __syncwarp();
        if (lane == 0)
          for (int i = 0; i < nb; ++i) mbar_arrive(&tempty[(tg + t0 + i) % b.ring]);
      }
      tg += nt;
    }
  } else if (warp < NCW + 2) {
    // ------------------------------------------------------ consumers
    const int ct = threadIdx.x - 64;
    constexpr int NC = NCW * 32;
    const CtaRange cr = cta_range(b.total);
    int tg = 0;
    // The loader fills the buffers with this CTA's jobs in order, then one
    // whose parameters say m < 0: the end.
    for (int jl = 0;; ++jl) {
      const int buf = jl % b.xbufs;
      if (!mbar_wait(&xfull[buf], (jl / b.xbufs) & 1, &s_abort) || s_abort) break;
      const uint8_t* xsm = smem + buf * b.x_stride;
      const GemvParams& p = *reinterpret_cast<const GemvParams*>(xsm + b.p_off);
      if (p.m < 0) break;
      int rb, nt;
      const int re = batch_rows(p, cr, rb, nt);
      Fmt f;
      const int dpr = NC / p.gpr, dg = NC - dpr * p.gpr;
      const int pr0 = ct / p.gpr, g0 = ct - pr0 * p.gpr;
      const bool fixed = dpr >= 1;
      const bool idle = fixed && ct >= dpr * p.gpr;
      if (fixed && !idle) f.prepare(p, xsm, g0);
      bool stop = false;
      for (int t = 0; t < nt; ++t, ++tg) {
        const int s = tg % b.stages;
        const int tb = tg % b.ring;
        bool ok = mbar_wait(&full[s], (tg / b.stages) & 1, &s_abort);
        if (ok && tg >= b.ring) ok = mbar_wait(&tempty[tb], ((tg / b.ring) - 1) & 1, &s_abort);
        if (!ok || s_abort) {
          stop = true;
          break;
        }
        const int r0 = rb + t * p.rt;
        const int rows = min(p.rt, re - r0);
        const uint8_t* W = stw + s * b.stage_w_bytes;
        const float* S = reinterpret_cast<const float*>(sts + s * b.stage_s_bytes);
        float* T = terms + tb * b.tslot;
        const int npairs = (rows + 1) >> 1;
        if (fixed) {
          const int g = g0;
          int pr = idle ? npairs : pr0;
          for (; Fmt::kTwoPairs && pr + dpr < npairs; pr += 2 * dpr) {
            const int ra = 2 * pr, rc = 2 * (pr + dpr);
            const int rb2 = min(ra + 1, rows - 1), rd = min(rc + 1, rows - 1);
            float t0, t1, t2, t3;
            f.term2(p, xsm, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                    S + rb2 * p.gpr, g, t0, t1);
            f.term2(p, xsm, W + rc * p.row_bytes, W + rd * p.row_bytes, S + rc * p.gpr,
                    S + rd * p.gpr, g, t2, t3);
            if constexpr (Fmt::kFix) {
              f.fix2(p, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                     S + rb2 * p.gpr, g, t0, t1);
              f.fix2(p, W + rc * p.row_bytes, W + rd * p.row_bytes, S + rc * p.gpr,
                     S + rd * p.gpr, g, t2, t3);
            }
            if (Fmt::kFold == Fold::Tree && p.wred) {
              store_warp_sums(T, p.tstride, rows, ra, rc, t0, t1, t2, t3, g >> 5, lane);
              continue;
            }
            T[ra * p.tstride + g] = t0;
            if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
            T[rc * p.tstride + g] = t2;
            if (rc + 1 < rows) T[(rc + 1) * p.tstride + g] = t3;
          }
          for (; pr < npairs; pr += dpr) {
            const int ra = 2 * pr;
            const int rb2 = min(ra + 1, rows - 1);
            float t0, t1;
            f.term2(p, xsm, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                    S + rb2 * p.gpr, g, t0, t1);
            if constexpr (Fmt::kFix)
              f.fix2(p, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                     S + rb2 * p.gpr, g, t0, t1);
            if (Fmt::kFold == Fold::Tree && p.wred) {
              store_warp_sums(T, p.tstride, rows, ra, -1, t0, t1, 0.0f, 0.0f, g >> 5, lane);
              continue;
            }
            T[ra * p.tstride + g] = t0;
            if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
          }
        } else {
          int g = g0;
          for (int pr = pr0; pr < npairs;) {
            const int ra = 2 * pr;
            const int rb2 = min(ra + 1, rows - 1);
            float t0, t1;
            f.prepare(p, xsm, g);
            f.term2(p, xsm, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                    S + rb2 * p.gpr, g, t0, t1);
            if constexpr (Fmt::kFix)
              f.fix2(p, W + ra * p.row_bytes, W + rb2 * p.row_bytes, S + ra * p.gpr,
                     S + rb2 * p.gpr, g, t0, t1);
            T[ra * p.tstride + g] = t0;
            if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = t1;
            g += dg;
            pr += dpr;
            if (g >= p.gpr) {
              g -= p.gpr;
              ++pr;
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty[s]);
          mbar_arrive(&tfull[tb]);
        }
      }
      if (stop) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xempty[buf]);
    }
  } else if (warp == NCW + 2) {
    // ------------------------------------------------- image loader
    // Each job's staged activations, copied by this warp's 32 lanes with
    // 16-byte cp.async (the load path, not the bulk-copy engine: an image
    // copied in bulk waits behind the weight tiles this SM has in flight)
    // into the buffer the consumers freed, up to xbufs jobs ahead.  The
    // images were written by the kernel before this one.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const CtaRange cr = cta_range(b.total);
    int jl = 0;  // jobs handed to the consumers
    bool stop = false;
    for (int j = first_job(b, cr); j < b.n && b.job[j].boff < cr.ce; ++j) {
      int rb, nt;
      batch_rows(b.job[j], cr, rb, nt);
      if (nt == 0) continue;  // the range holds no row start of this job
      const int buf = jl % b.xbufs;
      if (jl >= b.xbufs &&
          !mbar_wait_idle(&xempty[buf], ((jl / b.xbufs) - 1) & 1, &s_abort)) {
        stop = true;
        break;
      }
      if (s_abort) {
        stop = true;
        break;
      }
      ++jl;
      const uint8_t* src = b.img + static_cast<int64_t>(j) * b.x_stride;
      uint8_t* dst = smem + buf * b.x_stride;
      for (int o = lane * 16; o < b.job[j].x_bytes; o += 32 * 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst + o)),
                     "l"(src + o)
                     : "memory");
      // and the job's parameters
      for (int o = lane * 16; o < static_cast<int>(sizeof(GemvParams)); o += 32 * 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst + b.p_off + o)),
                     "l"(src + b.p_off + o)
                     : "memory");
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(saddr(&xfull[buf]))
                   : "memory");
    }
    // the end marker: a buffer whose parameters say m = -1
    const int buf = jl % b.xbufs;
    if (!stop && (jl < b.xbufs ||
                  mbar_wait_idle(&xempty[buf], ((jl / b.xbufs) - 1) & 1, &s_abort))) {
      if (lane == 0)
        reinterpret_cast<GemvParams*>(smem + buf * b.x_stride + b.p_off)->m = -1;
      __syncwarp();
      mbar_arrive(&xfull[buf]);  // all 32 lanes: the phase's count
    }
    // never leave with a copy still landing in shared memory
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  if (b.rs.n > 0) {
    // The other ranks' rows, then the gather is complete on this rank once
    // every CTA's folds (this rank's rows) and receive are done: the last
    // CTA to get here publishes its number, which the next gather's kernels
    // read.  (The folder took the number after its grid-dependency wait.)
    __syncthreads();
    PushTag t;
    t.tag = static_cast<uint64_t>(s_gather) << 32;
    t.half = (s_gather & 1u) * kXchgWords;
    batch_receive(b, t, threadIdx.x, blockDim.x);
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      uint32_t* state = b.push->state;
      if (atomicAdd(state + 1, 1u) == gridDim.x - 1) {
        state[1] = 0;
        __threadfence();
        atomicExch(state, s_gather);
      }
    }
  }
}

}  // namespace lp
