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
// per SM; the planner sizes it so two fit on an SM, which lets the next
// launch in the stream start streaming while this one drains).  It walks its
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
#include "lp_device.cuh"

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
  int off_w, off_s, off_t, off_b;  // shared-memory offsets (128-byte aligned)
  int stage_w_bytes, stage_s_bytes;
  float neg_zero;     // -0.0f, passed at run time (see mul2_rn)
};

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
// power of two with L * rows <= 32; each lane sums a strided subset of the
// row's terms in four chains, then the L partial sums meet by shuffles.
__device__ __forceinline__ void tree_fold(const float* T, int tstride, int rows, int gpr,
                                          float* y, int lane) {
  int lg = 5;
  while (lg > 0 && (rows << lg) > 32) --lg;
  const int L = 1 << lg;
  const int r = lane >> lg, sub = lane & (L - 1);
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  if (r < rows) {
    const float* row = T + r * tstride;
    int g = sub;
    for (; g + 3 * L < gpr; g += 4 * L) {
      s0 = fadd(s0, row[g]);
      s1 = fadd(s1, row[g + L]);
      s2 = fadd(s2, row[g + 2 * L]);
      s3 = fadd(s3, row[g + 3 * L]);
    }
    for (; g < gpr; g += L) s0 = fadd(s0, row[g]);
  }
  float s = fadd(fadd(s0, s1), fadd(s2, s3));
  for (int o = L >> 1; o > 0; o >>= 1) s = fadd(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (r < rows && sub == 0) y[r] = s;
}

// ----------------------------------------------------------- the kernel
template <class Fmt, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 2), 2) gemv_kernel(const GemvParams p) {
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    for (int b = 0; b < p.ring; ++b) {
      mbar_init(&tfull[b], NCW);
      mbar_init(&tempty[b], 1);
    }
    s_abort = 0;
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
      if (t >= p.stages && !mbar_wait(&empty[s], ((t / p.stages) - 1) & 1, &s_abort)) break;
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
    if constexpr (Fmt::kFold == Fold::Tree) {
      for (int t = 0; t < ntiles; ++t) {
        const int slot = t % p.ring;
        if (!mbar_wait(&tfull[slot], (t / p.ring) & 1, &s_abort)) break;
        if (s_abort) break;
        const int r0 = row_begin + t * p.rt;
        const int rows = min(p.rt, row_end - r0);
        tree_fold(terms + slot * p.rt * p.tstride, p.tstride, rows, p.gpr, p.y + r0, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
      }
    } else {
      // Lane l folds row l % rt of tile t0 + l / rt of each batch.
      const int ti = lane / p.rt, r = lane - ti * p.rt;
      for (int t0 = 0; t0 < ntiles; t0 += p.fb) {
        const int nt = min(p.fb, ntiles - t0);
        bool ok = true;
        for (int i = 0; i < nt && ok; ++i)
          ok = mbar_wait(&tfull[(t0 + i) % p.ring], ((t0 + i) / p.ring) & 1, &s_abort);
        if (!ok || s_abort) break;
        if (ti < nt) {
          const int t = t0 + ti;
          const int r0 = row_begin + t * p.rt;
          if (r < min(p.rt, row_end - r0))
            p.y[r0 + r] =
                fold_row<Fmt::kFold>(terms + ((t % p.ring) * p.rt + r) * p.tstride, p.gpr);
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
    f.init(p, xsm);
    // Unit q = pair * gpr + g walks q = ct, ct + NC, ...; stepped without a
    // division per unit.
    const int dpr = NC / p.gpr, dg = NC - dpr * p.gpr;
    const int pr0 = ct / p.gpr, g0 = ct - pr0 * p.gpr;
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
      int g = g0;
      for (int pr = pr0; pr < npairs;) {
        const int ra = 2 * pr;
        const int rb = min(ra + 1, rows - 1);
        float ta, tbv;
        f.term2(p, xsm, W + ra * p.row_bytes, W + rb * p.row_bytes, S + ra * p.gpr,
                S + rb * p.gpr, g, ta, tbv);
        T[ra * p.tstride + g] = ta;
        if (ra + 1 < rows) T[(ra + 1) * p.tstride + g] = tbv;
        g += dg;
        pr += dpr;
        if (g >= p.gpr) {
          g -= p.gpr;
          ++pr;
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

}  // namespace lp
