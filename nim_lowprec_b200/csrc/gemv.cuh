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
// per SM, sixteen consumer warps).  K is cut into chunks of G groups; a stage is SR rows x one chunk,
// where SR * G / 2 equals the consumer thread count, so every consumer
// thread computes exactly one row pair of one group per stage.  Stages run
// chunk-major over the CTA's rows (all rows of chunk 0, then chunk 1, ...),
// so each row's terms arrive in group order, one chunk at a time.
//
//   warp 0   producer: per stage one 2-D tiled TMA load of the weight box
//            (SR rows x one chunk) and one of the scale box, HBM -> shared,
//            `stages` deep, tracked by mbarriers (a CTA's last rows come in
//            single-row boxes so no other CTA's rows are fetched).  Few large
//            copies keep enough bytes in flight per SM; one small copy per
//            row does not.  Shapes whose rows are not 16-byte aligned take a
//            plain-load staging path.  It starts before the activations are
//            staged and, under programmatic dependent launch, before the
//            previous kernel in the stream has finished.
//   warps 2+ consumers: per stage, the terms of one row pair x one group
//            (two rows run as one packed f32x2 chain on the fp32 paths) into
//            the chunk's term matrix (double-buffered by chunk).
//   warp 1   folder: once a chunk's terms are complete, each lane folds the
//            chunk into the running totals of its rows (up to four rows per
//            lane, independent chains) and writes y after the last chunk.
//            Chains are one chunk long, so the fold trails the consumers by
//            about one chunk and the kernel tail is one short fold.
#pragma once
#include "lp_device.cuh"

namespace lp {

enum class Fold { Serial, Lanes4 };

struct alignas(64) GemvParams {
  // 2-D tensor maps over the weight rows (uint64 elements, row_bytes / 8 per
  // row) and the scale rows (fp32, gpr per row): box *_full covers a whole
  // stage (SR rows x one chunk), box *_row a single row of it.
  CUtensorMap tw_full, tw_row, ts_full, ts_row;
  const uint8_t* w;   // weight rows, row_bytes each
  const float* ws;    // per-row group scales (M x gpr) or nullptr
  const void* x;      // activations (format-specific)
  const float* xs;    // activation group scales or nullptr
  float* y;
  int m, k, gs, gpr;  // gpr: groups (ggml: blocks) per row
  int row_bytes;
  int G;              // groups per chunk (multiple of 4)
  int SR;             // rows per stage (<= 32)
  int RP;             // rows per pass (term-matrix height), <= kMaxRowsPerPass
  int stages;
  int bulk;           // 1: tensor-map (TMA) staging, 0: plain loads
  int tstride;        // floats per term-matrix row
  int x_bytes;        // shared bytes for the staged activations
  int off_w, off_s, off_t, off_b;  // shared-memory offsets
  int slice_pitch;    // shared bytes per weight row slice (G groups, 128-byte multiple)
  int spitch;         // shared floats per scale row slice (spitch * 4: 128-byte multiple)
  int stage_w_bytes, stage_s_bytes;
  float neg_zero;     // -0.0f, passed at run time (see mul2_rn)
};

constexpr int kMaxRowsPerPass = 128;  // four running totals per folder lane

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

// Byte offset of group g inside a weight row.  Exact: chunk starts are
// multiples of G (even), so packed 4-bit rows split on whole bytes.
__device__ __forceinline__ int64_t group_byte(const GemvParams& p, int g) {
  return static_cast<int64_t>(g) * p.row_bytes / p.gpr;
}

// The schedule all three roles walk: for each pass of up to RP rows, for
// each chunk, the pass's rows in stages of SR.
struct Sched {
  int row_end;
  int pass_r0, pass_rows;  // current pass
  int chunk, nchunks;
  int sb, nsb;             // stage within the chunk
  __device__ __forceinline__ void start(const GemvParams& p, int rb, int re) {
    row_end = re;
    pass_r0 = rb;
    pass_rows = min(p.RP, re - rb);
    chunk = 0;
    nchunks = (p.gpr + p.G - 1) / p.G;
    sb = 0;
    nsb = (pass_rows + p.SR - 1) / p.SR;
  }
  __device__ __forceinline__ bool done() const { return pass_r0 >= row_end; }
  __device__ __forceinline__ bool last_sb() const { return sb == nsb - 1; }
  __device__ __forceinline__ bool last_chunk() const { return chunk == nchunks - 1; }
  __device__ __forceinline__ void next(const GemvParams& p) {
    if (++sb < nsb) return;
    sb = 0;
    if (++chunk < nchunks) return;
    chunk = 0;
    pass_r0 += pass_rows;
    pass_rows = min(p.RP, row_end - pass_r0);
    nsb = (pass_rows + p.SR - 1) / p.SR;
  }
};

// ------------------------------------------------------------- folds
// Folds `n` terms of a chunk into the running state of up to four rows per
// lane (rows lane + 32 j, term rows `ts` floats apart), in group order.
// Serial: st[j][0] += t.  Lanes4: st[j][g & 3] += t (chunks start on
// multiples of 4 groups, so the local index has the global lane).
template <Fold F>
__device__ __forceinline__ void fold_chunk(const float* T, int ts, int nrows_lane, int n,
                                           float (&st)[4][4]) {
  const int n4 = n & ~3;
  for (int g = 0; g < n4; g += 4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < nrows_lane) {
        const float4 v = *reinterpret_cast<const float4*>(T + j * 32 * ts + g);
        if (F == Fold::Serial) {
          st[j][0] = fadd(st[j][0], v.x);
          st[j][0] = fadd(st[j][0], v.y);
          st[j][0] = fadd(st[j][0], v.z);
          st[j][0] = fadd(st[j][0], v.w);
        } else {
          st[j][0] = fadd(st[j][0], v.x);
          st[j][1] = fadd(st[j][1], v.y);
          st[j][2] = fadd(st[j][2], v.z);
          st[j][3] = fadd(st[j][3], v.w);
        }
      }
    }
  }
  for (int g = n4; g < n; ++g) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < nrows_lane) {
        const float t = T[j * 32 * ts + g];
        if (F == Fold::Serial) {
          st[j][0] = fadd(st[j][0], t);
        } else {
          const int l = g & 3;
          if (l == 0) st[j][0] = fadd(st[j][0], t);
          else if (l == 1) st[j][1] = fadd(st[j][1], t);
          else st[j][2] = fadd(st[j][2], t);
        }
      }
    }
  }
}

// ----------------------------------------------------------- the kernel
template <class Fmt, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 2), 1)
    gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ volatile int s_abort;
  // Every TMA destination below is 128-byte aligned relative to this base;
  // align the base itself rather than rely on the declaration (the launch
  // reserves the 128 bytes this may skip).
  uint8_t* smem = smem_raw + ((128u - (saddr(smem_raw) & 127u)) & 127u);
  uint8_t* xsm = smem;
  uint8_t* stw = smem + p.off_w;
  uint8_t* sts = smem + p.off_s;
  float* terms = reinterpret_cast<float*>(smem + p.off_t);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_b);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* tfull = bars + 2 * p.stages;
  uint64_t* tempty = tfull + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row_begin = static_cast<int>((static_cast<int64_t>(p.m) * blockIdx.x) / gridDim.x);
  const int row_end = static_cast<int>((static_cast<int64_t>(p.m) * (blockIdx.x + 1)) / gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], NCW);
      mbar_init(&tempty[b], 1);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (row_end <= row_begin) return;

  Sched sc;
  sc.start(p, row_begin, row_end);

  if (warp == 0) {
    // ------------------------------------------------------ producer
    // Weights never come from the kernel this launch may overlap with (see
    // launch_gemv), so the stream starts before the grid dependency is
    // resolved; the activations wait for it in the consumer warps.
    const uint64_t pol = l2_evict_first();
    if (p.bulk && lane == 0) {
      tma_prefetch_desc(&p.tw_full);
      tma_prefetch_desc(&p.tw_row);
    }
    int t = 0;
    for (; !sc.done(); sc.next(p), ++t) {
      const int s = t % p.stages;
      if (t == p.stages) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
      if (t >= p.stages && !mbar_wait(&empty[s], ((t / p.stages) - 1) & 1, &s_abort)) break;
      if (s_abort) break;
      const int r0 = sc.pass_r0 + sc.sb * p.SR;
      const int rows = min(p.SR, sc.pass_r0 + sc.pass_rows - r0);
      const int g0 = sc.chunk * p.G;
      const int gc = min(p.G, p.gpr - g0);
      const int64_t gb0 = group_byte(p, g0);
      const uint32_t slice = static_cast<uint32_t>(group_byte(p, g0 + gc) - gb0);
      const uint32_t sslice = Fmt::kScales ? static_cast<uint32_t>(gc) * 4u : 0u;
      uint8_t* dw = stw + s * p.stage_w_bytes;
      float* ds = reinterpret_cast<float*>(sts + s * p.stage_s_bytes);
      const uint8_t* gw = p.w + static_cast<int64_t>(r0) * p.row_bytes + gb0;
      const float* gsc = Fmt::kScales ? p.ws + static_cast<int64_t>(r0) * p.gpr + g0 : nullptr;
      if (p.bulk) {
        // Boxes are a full chunk wide (columns past the row end read as 0)
        // and count full-width bytes.
        const int c0 = static_cast<int>(gb0 >> 3);
        if (rows == p.SR) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[s], p.SR * (p.slice_pitch + (Fmt::kScales ? p.spitch * 4 : 0)));
            tma_load_2d(dw, &p.tw_full, c0, r0, &full[s], pol);
            if (Fmt::kScales) tma_load_2d(ds, &p.ts_full, g0, r0, &full[s], pol);
          }
        } else {
          if (lane == 0)
            mbar_arrive_expect_tx(&full[s], rows * (p.slice_pitch + (Fmt::kScales ? p.spitch * 4 : 0)));
          __syncwarp();
          if (lane < rows) {
            tma_load_2d(dw + lane * p.slice_pitch, &p.tw_row, c0, r0 + lane, &full[s], pol);
            if (Fmt::kScales) tma_load_2d(ds + lane * p.spitch, &p.ts_row, g0, r0 + lane, &full[s], pol);
          }
        }
        (void)slice;
        (void)sslice;
        (void)gw;
        (void)gsc;
      } else {
        for (int r = 0; r < rows; ++r) {
          for (uint32_t i = lane; i < slice; i += 32)
            dw[r * p.slice_pitch + i] = gw[static_cast<int64_t>(r) * p.row_bytes + i];
          if (Fmt::kScales)
            for (int i = lane; i < gc; i += 32) ds[r * p.spitch + i] = gsc[static_cast<int64_t>(r) * p.gpr + i];
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
    }
    if (t <= p.stages) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // Drain: never leave the CTA with a bulk copy still landing in shared.
    if (p.bulk && lane == 0) {
      for (int u = max(0, t - p.stages); u < t; ++u)
        mbar_wait(&full[u % p.stages], (u / p.stages) & 1);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- folder
    float st[4][4];
    int kc = 0;  // chunks folded by this CTA (term-buffer parity)
    for (; !sc.done(); sc.next(p)) {
      if (!sc.last_sb()) continue;  // one fold per chunk, after its last stage
      if (sc.chunk == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int l = 0; l < 4; ++l) st[j][l] = 0.0f;
      }
      const int tb = kc & 1;
      if (!mbar_wait(&tfull[tb], (kc >> 1) & 1, &s_abort)) break;
      if (s_abort) break;
      const int gc = min(p.G, p.gpr - sc.chunk * p.G);
      const int nrl = (sc.pass_rows - lane + 31) / 32;  // rows of this lane: lane + 32 j
      const float* T = terms + (tb * p.RP + lane) * p.tstride;
      fold_chunk<Fmt::kFold>(T, p.tstride, nrl, gc, st);
      if (sc.last_chunk()) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j < nrl) {
            const float out = Fmt::kFold == Fold::Serial
                                  ? st[j][0]
                                  : fadd(fadd(st[j][0], st[j][1]), fadd(st[j][2], st[j][3]));
            p.y[sc.pass_r0 + lane + 32 * j] = out;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[tb]);
      ++kc;
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
    const int gl = ct % p.G;  // group within the chunk
    const int ra = 2 * (ct / p.G);  // first row of this thread's pair in a stage
    int t = 0, kc = 0;
    for (; !sc.done(); sc.next(p), ++t) {
      const int s = t % p.stages;
      const int tb = kc & 1;
      bool ok = mbar_wait(&full[s], (t / p.stages) & 1, &s_abort);
      if (ok && sc.sb == 0 && kc >= 2) ok = mbar_wait(&tempty[tb], ((kc >> 1) - 1) & 1, &s_abort);
      if (!ok || s_abort) break;
      const int r0 = sc.pass_r0 + sc.sb * p.SR;
      const int rows = min(p.SR, sc.pass_r0 + sc.pass_rows - r0);
      const int g0 = sc.chunk * p.G;
      const int gc = min(p.G, p.gpr - g0);
      if (gl < gc && ra < rows) {
        const int rb = min(ra + 1, rows - 1);
        // Pointers rebased so that the absolute group index g addresses this
        // chunk's slice: the policies index weights, scales and x by g.
        const int64_t wb = group_byte(p, g0);
        const uint8_t* W = stw + s * p.stage_w_bytes;
        const float* S = reinterpret_cast<const float*>(sts + s * p.stage_s_bytes);
        float ta, tbv;
        f.term2(p, xsm, W + ra * p.slice_pitch - wb, W + rb * p.slice_pitch - wb,
                S + ra * p.spitch - g0, S + rb * p.spitch - g0, g0 + gl, ta, tbv);
        float* T = terms + (tb * p.RP + sc.sb * p.SR + ra) * p.tstride + gl;
        T[0] = ta;
        if (ra + 1 < rows) T[p.tstride] = tbv;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        if (sc.last_sb()) mbar_arrive(&tfull[tb]);
      }
      if (sc.last_sb()) ++kc;
    }
  }
}

}  // namespace lp
